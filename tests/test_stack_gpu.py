"""The linear stack (configs 4/5 wiring, with the engine's residual adds and RMSNorms) on the GPU
against the CPU oracle stack: per projection with the same fp16 input (max
relative error 2e-3, per-row cosine 0.99999), end to end over two layers (the same tolerance), and
the residual add + RMSNorm kernel on its own."""
import importlib

import numpy as np
import pytest

from conftest import load_package
from oracle import s4ref

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def serve():
    load_package()
    return importlib.import_module("strands_decider_web_b200.serve")


def _oracle_layers(serve, n_layers):
    out = []
    for li, kind in enumerate(serve.layer_kinds(n_layers)):
        out.append({name: serve.synthetic_projection(serve.projection_seed(li, name), K, N)
                    for name, K, N in serve.projection_shapes(kind)})
    return out


def _add_norm(x, y):
    xn, h = s4ref.add_rmsnorm(x.numpy(), None if y is None else y.numpy())
    return torch.from_numpy(xn), torch.from_numpy(h)


def _cpu_ops(serve):
    return serve.Ops(matmul=lambda x, w: torch.from_numpy(s4ref.matmul(x.numpy(), *w)[0]),
                     silu_mul=lambda big, I: torch.from_numpy(s4ref.silu_mul(big.numpy(), I)),
                     all_gather=None,
                     add_norm=_add_norm,
                     cols=lambda x, c0, c1: x[:, c0:c1].contiguous(),
                     to_f32=lambda x: x.float())


@pytest.mark.parametrize("M", [8, 64, 300])
@pytest.mark.parametrize("fuse_norm", [False, True])
def test_stack_two_layers_matches_oracle(ctx, serve, M, fuse_norm):
    stack = serve.CudaStack(ctx, n_layers=4, host_gen=True, fuse_norm=fuse_norm)  # layers: L L L A
    stack.layers = [stack.layers[0], stack.layers[3]]
    x = s4ref.config_x(np.random.default_rng(M), M, serve.HIDDEN)
    y = stack.forward(torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    ol = _oracle_layers(serve, 4)
    ref = serve.stack_forward(torch.from_numpy(x), [ol[0], ol[3]], _cpu_ops(serve)).numpy()
    ok, mr, mc = s4ref.check(y.cpu().numpy(), ref.astype(np.float32))
    assert ok, (mr, mc)


def test_stack_projections_teacher_forced(ctx, serve):
    stack = serve.CudaStack(ctx, n_layers=4, host_gen=True)
    ol = _oracle_layers(serve, 4)
    rng = np.random.default_rng(3)
    for li in (0, 3):
        for name, K, N in serve.projection_shapes(serve.layer_kinds(4)[li]):
            x = s4ref.config_x(rng, 48, K)
            y = ctx.matmul(torch.from_numpy(x).cuda(), stack.layers[li][name])
            torch.cuda.synchronize()
            y16, ref = s4ref.matmul(x, *ol[li][name])
            if name == "gate_up" and stack.fuse_silu:  # the fused weight's matmul writes SiLU*mul
                ref = s4ref.silu_mul(y16, N // 2).astype(np.float32)
            ok, mr, mc = s4ref.check(y.cpu().numpy(), ref)
            assert ok, (li, name, mr, mc)


def test_device_generated_weights_are_deterministic(ctx, serve):
    a = serve.synthetic_projection_torch(5, 64, 256, torch.device("cuda", 0))
    b = serve.synthetic_projection_torch(5, 64, 256, torch.device("cuda", 0))
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
    assert int(a[0].max()) > 200 and float(a[1].float().abs().max()) > 0


@pytest.mark.parametrize("M,D,with_y,with_w", [(1, 2048, False, False), (37, 2048, True, False),
                                               (300, 2048, True, True), (5, 1000, True, True)])
def test_add_rmsnorm_matches_oracle(ctx, M, D, with_y, with_w):
    rng = np.random.default_rng(M * 7 + D)
    x = (rng.standard_normal((M, D)) * 4).astype(np.float32)
    y = (rng.standard_normal((M, D)) * 2).astype(np.float16) if with_y else None
    w = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32) if with_w else None
    xd = torch.from_numpy(x).cuda()
    h = ctx.add_rmsnorm(xd, None if y is None else torch.from_numpy(y).cuda(),
                        None if w is None else torch.from_numpy(w).cuda())
    torch.cuda.synchronize()
    xr, hr = s4ref.add_rmsnorm(x, y, w)
    np.testing.assert_array_equal(xd.cpu().numpy(), xr)          # fp32 add: one rounding, bit-exact
    # the fp32 sum of squares differs only in summation order: at most one fp16 ulp on h
    np.testing.assert_allclose(h.cpu().numpy().astype(np.float32), hr.astype(np.float32), rtol=1e-3, atol=1e-3)


# (K, N, M, norm weight, forced tcgen05 shape): out_proj / down shapes on the GEMV and tcgen05 paths,
# split tiles (fix-up kernel) and whole tiles, a ragged last n-block (N % 128 == 32) and an N that is
# not a multiple of 32 (matmul into h, then ADD_NORM in place)
ADDNORM_CASES = [(2048, 2048, 1, False, None), (2048, 2048, 8, True, None), (2048, 2048, 64, True, None),
                 (6144, 2048, 300, True, None), (6144, 2048, 2048, False, None),
                 (2048, 2048, 300, True, ("tc", 64, 148)), (2048, 2048, 300, True, ("tc", 64, 80)),
                 (512, 2080, 100, True, None), (512, 2056, 100, True, None)]


@pytest.mark.parametrize("K,N,M,with_w,force", ADDNORM_CASES)
def test_matmul_add_rmsnorm_matches_oracle(ctx, K, N, M, with_w, force):
    """s4_matmul_add_rmsnorm against the oracle's matmul then ADD_NORM, and against the GPU's own
    two-call form (s4_matmul, s4_add_rmsnorm): same fp16 y, so the residual agrees bit for bit."""
    rng = np.random.default_rng(K + N + M)
    packed, scales = s4ref.config_weights(rng, K, N)
    x = s4ref.config_x(rng, M, K)
    resid = (rng.standard_normal((M, N)) * 0.5).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(N)).astype(np.float32) if with_w else None
    W = ctx.upload(packed, scales, N, K)
    if force:
        ctx.force(*force)
    try:
        xd = torch.from_numpy(x).cuda()
        wd = None if w is None else torch.from_numpy(w).cuda()
        r1 = torch.from_numpy(resid).cuda()
        h1 = ctx.matmul_add_rmsnorm(xd, W, r1, wd)
        r2 = torch.from_numpy(resid).cuda()
        h2 = ctx.add_rmsnorm(r2, ctx.matmul(xd, W), wd)
        torch.cuda.synchronize()
        assert ctx.check_errors() == 0
    finally:
        ctx.force()
        W.free()
    y16, _ = s4ref.matmul(x, packed, scales)
    xr, hr = s4ref.add_rmsnorm(resid, y16, w)
    # the residual: y's fp16 rounding may differ by one ulp from the oracle's (fp32 sums in another order)
    tol = 2e-3 * float(np.abs(y16.astype(np.float32)).max()) + 1e-6
    np.testing.assert_allclose(r1.cpu().numpy(), xr, rtol=0, atol=tol)
    ok, mr, mc = s4ref.check(h1.cpu().numpy(), hr.astype(np.float32))
    assert ok, (mr, mc)
    np.testing.assert_array_equal(r1.cpu().numpy(), r2.cpu().numpy())
    # the sums of squares differ only in order: at most one fp16 ulp on h
    np.testing.assert_allclose(h1.cpu().numpy().astype(np.float32), h2.cpu().numpy().astype(np.float32),
                               rtol=1e-3, atol=1e-3)


def test_matmul_add_rmsnorm_rejects_bad_arguments(ctx):
    rng = np.random.default_rng(1)
    packed, scales = s4ref.config_weights(rng, 256, 256)
    W = ctx.upload(packed, scales, 256, 256)
    G = ctx.upload_glu(packed, scales, 128, 256)
    try:
        x = torch.zeros((4, 256), dtype=torch.float16, device="cuda")
        with pytest.raises(Exception):
            ctx.matmul_add_rmsnorm(x, W, torch.zeros((4, 256), dtype=torch.float16, device="cuda"))
        with pytest.raises(Exception):
            ctx.matmul_add_rmsnorm(x, W, torch.zeros((4, 128), dtype=torch.float32, device="cuda"))
        with pytest.raises(Exception):
            ctx.matmul_add_rmsnorm(x, G, torch.zeros((4, 128), dtype=torch.float32, device="cuda"))
    finally:
        W.free()
        G.free()


def test_fused_stack_one_gpu_eager_graph_and_plain_agree(ctx, serve):
    """World size 1: the fused-gather stack (matmul_gather into its own buffers, no barriers) equals
    the plain stack bit for bit, eagerly and replayed from a CUDA graph."""
    M = 64
    fused = serve.FusedColshardStack(ctx, None, 0, 1, max_tokens=M, n_layers=2)
    try:
        x = torch.from_numpy(s4ref.config_x(np.random.default_rng(9), M, serve.HIDDEN)).cuda()
        y_eager = fused.forward(x).clone()
        plain = serve.stack_forward(x, fused.stack.layers, fused.stack.ops())
        y_graph = fused.capture(x)
        fused.replay()
        torch.cuda.synchronize()
        np.testing.assert_array_equal(y_eager.cpu().numpy(), plain.cpu().numpy())
        np.testing.assert_array_equal(y_eager.cpu().numpy(), y_graph.cpu().numpy())
        assert ctx.check_errors() == 0
    finally:
        fused.close()


def test_split_barrier_consumers_on_one_rank(ctx):
    """The split barrier's API on one GPU (nranks = 1): a signal, then the waiting GEMM and ADD_NORM
    give exactly what their plain forms give, and no wait expires."""
    rng = np.random.default_rng(21)
    K, N, M = 2048, 2048, 200
    packed, scales = s4ref.config_weights(rng, K, N)
    W = ctx.upload(packed, scales, N, K)
    flags = ctx.buffer_alloc(64)
    try:
        x = torch.from_numpy(s4ref.config_x(rng, M, K)).cuda()
        y1 = torch.zeros((M, N), dtype=torch.float16, device="cuda")
        y2 = torch.zeros_like(y1)
        ctx.matmul_gather(x.data_ptr(), K, M, W, [y1.data_ptr()], N, 0)
        for _ in range(3):  # several epochs in a row
            ctx.peer_signal([flags], 0)
            ctx.matmul_gather(x.data_ptr(), K, M, W, [y2.data_ptr()], N, 0, wait_flags=flags, nranks=1)
        r = (torch.randn((M, N), device="cuda") * 0.5)
        r1, r2 = r.clone(), r.clone()
        h1 = ctx.add_rmsnorm(r1, y1)
        ctx.peer_signal([flags], 0)
        h2 = ctx.add_rmsnorm(r2, y2, wait_flags=flags, nranks=1)
        torch.cuda.synchronize()
        assert ctx.check_errors() == 0
        assert torch.equal(y1, y2)
        assert torch.equal(r1, r2) and torch.equal(h1, h2)
        _, ref = s4ref.matmul(x.cpu().numpy(), packed, scales)
        ok, mr, mc = s4ref.check(y2.cpu().numpy(), ref)
        assert ok, (mr, mc)
    finally:
        W.free()
        ctx.buffer_free(flags)
