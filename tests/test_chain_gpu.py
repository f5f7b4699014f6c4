"""Chained decode GEMV (one persistent launch for a list of M <= 16 matmuls) against the CPU oracle:
independent ops over the decode shapes, dependent chains (an op reading the previous op's output),
ragged shapes (N not a multiple of 128, an op with fewer 128 x 64 chunks than SMs, K not a multiple
of 64), repeated runs (counters reset, results identical), CUDA-graph replay and argument errors.
Tolerance: the north star's max relative error 2e-3 and per-row cosine 0.99999."""
import numpy as np
import pytest

from oracle import s4ref

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _weights(ctx, rng, K, N):
    packed, scales = s4ref.config_weights(rng, K, N)
    return ctx.upload(packed, scales, N, K), packed, scales


def _x(rng, M, K):
    return torch.from_numpy(s4ref.config_x(rng, M, K)).cuda()


DECODE = [(2048, 8224), (2048, 3072), (2048, 12288), (6144, 2048)]


def test_independent_decode_ops_match_oracle(ctx):
    rng = np.random.default_rng(1)
    ops, refs = [], []
    for K, N in DECODE:
        W, packed, scales = _weights(ctx, rng, K, N)
        deq = s4ref.dequant(packed, scales)
        for M in (1, 3, 8, 16):
            x = _x(rng, M, K)
            y = torch.empty((M, N), dtype=torch.float16, device="cuda")
            ops.append((x, W, y))
            refs.append(s4ref.matmul(x.cpu().numpy(), packed, scales, deq)[1])
    chain = ctx.chain(ops)
    chain.run()
    torch.cuda.synchronize()
    assert ctx.check_errors() == 0
    for (x, W, y), ref in zip(ops, refs):
        ok, mr, mc = s4ref.check(y.cpu().numpy(), ref)
        assert ok, (x.shape[0], W.K, W.N, mr, mc)
    first = [o[2].clone() for o in ops]
    for _ in range(3):  # counters and tickets reset between runs; results bit-identical
        chain.run()
    torch.cuda.synchronize()
    assert ctx.check_errors() == 0
    for (x, W, y), y0 in zip(ops, first):
        assert torch.equal(y, y0)


@pytest.mark.parametrize("M", [1, 5, 16])
def test_dependent_chain_matches_sequential_oracle(ctx, M):
    """x -> W0 (2048 -> 2048) -> W1 (2048 -> 6144) -> W2 (6144 -> 2048), each op reading the last
    op's fp16 output inside the same launch."""
    rng = np.random.default_rng(10 + M)
    dims = [(2048, 2048), (2048, 6144), (6144, 2048)]
    ws = [_weights(ctx, rng, K, N) for K, N in dims]
    x0 = _x(rng, M, 2048)
    ys = [torch.empty((M, N), dtype=torch.float16, device="cuda") for _, N in dims]
    ops = [(x0, ws[0][0], ys[0], -1), (ys[0], ws[1][0], ys[1], 0), (ys[1], ws[2][0], ys[2], 1)]
    chain = ctx.chain(ops)
    for _ in range(2):
        ys[0].zero_(), ys[1].zero_(), ys[2].zero_()
        chain.run()
        torch.cuda.synchronize()
        assert ctx.check_errors() == 0
        h = x0.cpu().numpy()
        for i, (W, packed, scales) in enumerate(ws):
            ref16, ref32 = s4ref.matmul(h, packed, scales)
            # each stage compared with the oracle on the GPU's own fp16 input of that stage
            got_in = h if i == 0 else ys[i - 1].cpu().numpy()
            _, ref_i = s4ref.matmul(got_in, packed, scales)
            ok, mr, mc = s4ref.check(ys[i].cpu().numpy(), ref_i)
            assert ok, (i, mr, mc)
            h = ref16
        ok, mr, mc = s4ref.check(ys[2].cpu().numpy(), ref32)
        assert ok, ("end to end", mr, mc)


def test_ragged_shapes(ctx):
    rng = np.random.default_rng(7)
    shapes = [(96, 100, 2), (64, 128, 1), (32, 8, 3), (2048, 8224, 16), (160, 1000, 9), (6144, 130, 4)]
    ops, refs = [], []
    for K, N, M in shapes:
        W, packed, scales = _weights(ctx, rng, K, N)
        x = _x(rng, M, K)
        y = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
        ops.append((x, W, y))
        refs.append(s4ref.matmul(x.cpu().numpy(), packed, scales)[1])
    ctx.chain(ops).run()
    torch.cuda.synchronize()
    assert ctx.check_errors() == 0
    for (x, W, y), ref in zip(ops, refs):
        ok, mr, mc = s4ref.check(y.cpu().numpy(), ref)
        assert ok, (W.K, W.N, x.shape[0], mr, mc)


def test_chain_graph_replay(ctx):
    rng = np.random.default_rng(3)
    W, packed, scales = _weights(ctx, rng, 2048, 3072)
    x = _x(rng, 4, 2048)
    y1 = torch.empty((4, 3072), dtype=torch.float16, device="cuda")
    W2, p2, s2 = _weights(ctx, rng, 3072, 2048)
    y2 = torch.empty((4, 2048), dtype=torch.float16, device="cuda")
    chain = ctx.chain([(x, W, y1), (y1, W2, y2, 0)])
    chain.run()
    torch.cuda.synchronize()
    eager = y2.clone()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        chain.run()
    y2.zero_()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert ctx.check_errors() == 0
    assert torch.equal(y2, eager)


def test_chain_argument_errors(ctx, pkg):
    rng = np.random.default_rng(4)
    W, _, _ = _weights(ctx, rng, 64, 128)
    x17 = _x(rng, 17, 64)
    y17 = torch.empty((17, 128), dtype=torch.float16, device="cuda")
    with pytest.raises(pkg.S4Error):
        ctx.chain([(x17, W, y17)])
    x = _x(rng, 2, 64)
    y = torch.empty((2, 128), dtype=torch.float16, device="cuda")
    with pytest.raises(pkg.S4Error):
        ctx.chain([(x, W, y, 0)])  # an op cannot depend on itself
    with pytest.raises(pkg.S4Error):
        ctx.chain([(x, W, y), (x, W, y, 5)])  # nor on a later op


def test_chain_run_host_matches_device_run(ctx):
    """s4_chain_run_host: inputs copied from pinned host memory, the chained launch, outputs copied
    back, on one stream; equals the device-buffer run bit for bit."""
    rng = np.random.default_rng(12)
    (W1, p1, s1), (W2, p2, s2) = _weights(ctx, rng, 2048, 3072), _weights(ctx, rng, 6144, 2048)
    xdev = torch.empty(3 * 2048 + 2 * 6144, dtype=torch.float16, device="cuda")
    ydev = torch.empty(3 * 3072 + 2 * 2048, dtype=torch.float16, device="cuda")
    x1, x2 = xdev[:3 * 2048].view(3, 2048), xdev[3 * 2048:].view(2, 6144)
    y1, y2 = ydev[:3 * 3072].view(3, 3072), ydev[3 * 3072:].view(2, 2048)
    chain = ctx.chain([(x1, W1, y1), (x2, W2, y2)])
    hx = torch.from_numpy(np.concatenate([s4ref.config_x(rng, 3, 2048).ravel(),
                                          s4ref.config_x(rng, 2, 6144).ravel()])).pin_memory()
    hy = torch.empty(ydev.shape, dtype=torch.float16).pin_memory()
    stream = torch.cuda.current_stream()
    chain.run_host(hx, xdev, hy, ydev, stream)
    stream.synchronize()
    assert ctx.check_errors() == 0
    got = hy.clone()
    chain.run()
    torch.cuda.synchronize()
    assert torch.equal(got, ydev.cpu())
    _, ref1 = s4ref.matmul(hx[:3 * 2048].view(3, 2048).numpy(), p1, s1)
    ok, mr, mc = s4ref.check(got[:3 * 3072].view(3, 3072).numpy(), ref1)
    assert ok, (mr, mc)
    _, ref2 = s4ref.matmul(hx[3 * 2048:].view(2, 6144).numpy(), p2, s2)
    ok, mr, mc = s4ref.check(got[3 * 3072:].view(2, 2048).numpy(), ref2)
    assert ok, (mr, mc)


def test_mixed_chain_phases_match_oracle(ctx):
    """A (indep), B (indep), C (reads A), D (indep), E (reads C), F (indep, long K): phases break at
    the dependencies, independent neighbours share a phase; every output against the oracle on the
    GPU's own input of that op."""
    rng = np.random.default_rng(21)
    M = 4
    WA, pA, sA = _weights(ctx, rng, 2048, 3072)
    WB, pB, sB = _weights(ctx, rng, 2048, 8224)
    WC, pC, sC = _weights(ctx, rng, 3072, 2048)
    WD, pD, sD = _weights(ctx, rng, 2048, 12288)
    WE, pE, sE = _weights(ctx, rng, 2048, 6144)
    WF, pF, sF = _weights(ctx, rng, 6144, 2048)
    xA, xB, xD = _x(rng, M, 2048), _x(rng, M, 2048), _x(rng, M, 2048)
    xF = _x(rng, M, 6144)
    yA = torch.empty((M, 3072), dtype=torch.float16, device="cuda")
    yB = torch.empty((M, 8224), dtype=torch.float16, device="cuda")
    yC = torch.empty((M, 2048), dtype=torch.float16, device="cuda")
    yD = torch.empty((M, 12288), dtype=torch.float16, device="cuda")
    yE = torch.empty((M, 6144), dtype=torch.float16, device="cuda")
    yF = torch.empty((M, 2048), dtype=torch.float16, device="cuda")
    chain = ctx.chain([(xA, WA, yA), (xB, WB, yB), (yA, WC, yC, 0), (xD, WD, yD), (yC, WE, yE, 2), (xF, WF, yF)])
    for _ in range(2):
        chain.run()
        torch.cuda.synchronize()
        assert ctx.check_errors() == 0
        for x, y, pk, sc in ((xA, yA, pA, sA), (xB, yB, pB, sB), (yA, yC, pC, sC), (xD, yD, pD, sD),
                             (yC, yE, pE, sE), (xF, yF, pF, sF)):
            _, ref = s4ref.matmul(x.cpu().numpy(), pk, sc)
            ok, mr, mc = s4ref.check(y.cpu().numpy(), ref)
            assert ok, (y.shape, mr, mc)


def test_chain_runs_back_to_back_on_one_stream(ctx):
    """Chained runs issued back to back on one stream overlap (programmatic dependent launch): run i
    reads what run i-1 wrote, and one chain run repeatedly reuses its counters and scratch. Each
    run is checked against the oracle on the GPU's own input (teacher-forced), and repeated runs of
    one chain are bitwise identical."""
    rng = np.random.default_rng(77)
    K, H = 2048, 3072
    p1, s1 = s4ref.config_weights(rng, K, H)
    p2, s2 = s4ref.config_weights(rng, H, K)
    W1, W2 = ctx.upload(p1, s1, H, K), ctx.upload(p2, s2, K, H)
    d1, d2 = s4ref.dequant(p1, s1), s4ref.dequant(p2, s2)
    R, M = 6, 4
    xs = [torch.zeros((M, K), dtype=torch.float16, device="cuda") for _ in range(R + 1)]
    mids = [torch.zeros((M, H), dtype=torch.float16, device="cuda") for _ in range(R)]
    xs[0].copy_(torch.from_numpy(s4ref.config_x(rng, M, K)))
    chains = [ctx.chain([(xs[i], W1, mids[i]), (mids[i], W2, xs[i + 1], 0)]) for i in range(R)]
    stream = torch.cuda.current_stream()
    for ch in chains:
        ch.run(stream)
    torch.cuda.synchronize()
    for i in range(R):
        x = xs[i].cpu().numpy()
        _, r1 = s4ref.matmul(x, p1, s1, d1)
        ok, mr, mc = s4ref.check(mids[i].cpu().numpy(), r1)
        assert ok, f"run {i} op 0: max_rel={mr:.2e} min_cos={mc:.7f}"
        _, r2 = s4ref.matmul(mids[i].cpu().numpy(), p2, s2, d2)
        ok, mr, mc = s4ref.check(xs[i + 1].cpu().numpy(), r2)
        assert ok, f"run {i} op 1: max_rel={mr:.2e} min_cos={mc:.7f}"
    first = xs[1].cpu().numpy().copy()
    for _ in range(5):
        chains[0].run(stream)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(xs[1].cpu().numpy().view(np.uint16), first.view(np.uint16))
    assert ctx.check_errors() == 0
    for ch in chains:
        ch.free()


@pytest.mark.parametrize("big_m", [7, 16])
def test_dynamic_op_ragged_and_deterministic(ctx, big_m):
    """A dependency-free chain whose op with the most n-blocks (17, the last one ragged: N = 2125,
    K = 1024) is claimed n-block by n-block at run time, next to static ops; 1 and 2 token groups.
    Every run matches the oracle and repeated runs are bitwise identical (a claimed n-block is summed
    by one CTA in k order, whichever CTA claims it)."""
    rng = np.random.default_rng(300 + big_m)
    specs = [(1024, 2125, big_m), (2048, 2048, 3), (2048, 384, 2), (96, 200, 5), (2048, 1000, 9)]
    ops, refs = [], []
    for K, N, M in specs:
        W, packed, scales = _weights(ctx, rng, K, N)
        x = _x(rng, M, K)
        y = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
        ops.append((x, W, y))
        refs.append(s4ref.matmul(x.cpu().numpy(), packed, scales)[1])
    chain = ctx.chain(ops)
    outs = []
    for _ in range(4):
        for o in ops:
            o[2].fill_(float("nan"))
        chain.run()
        torch.cuda.synchronize()
        assert ctx.check_errors() == 0
        for (x, W, y), ref in zip(ops, refs):
            ok, mr, mc = s4ref.check(y.cpu().numpy(), ref)
            assert ok, (x.shape[0], W.K, W.N, mr, mc)
        outs.append([o[2].clone() for o in ops])
    for later in outs[1:]:
        for a, b in zip(outs[0], later):
            assert torch.equal(a, b)
    chain.free()
