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
def test_stack_two_layers_matches_oracle(ctx, serve, M):
    stack = serve.CudaStack(ctx, n_layers=4, host_gen=True)  # layers 0-3: linear, linear, linear, attn
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
