"""The linear stack (configs 4/5 wiring) on the GPU against the CPU oracle stack: per projection with
the same fp16 input (max relative error 2e-3, per-row cosine 0.99999) and end
to end over two layers (the same tolerance; errors do not compound visibly at two layers)."""
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


def _cpu_ops(serve):
    return serve.Ops(matmul=lambda x, w: torch.from_numpy(s4ref.matmul(x.numpy(), *w)[0]),
                     silu_mul=lambda big, I: torch.from_numpy(s4ref.silu_mul(big.numpy(), I)),
                     all_gather=None,
                     add=lambda a, b: (a.float() + b.float()).half(),
                     cols=lambda x, c0, c1: x[:, c0:c1].contiguous())


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
            _, ref = s4ref.matmul(x, *ol[li][name])
            ok, mr, mc = s4ref.check(y.cpu().numpy(), ref)
            assert ok, (li, name, mr, mc)


def test_device_generated_weights_are_deterministic(ctx, serve):
    a = serve.synthetic_projection_torch(5, 64, 256, torch.device("cuda", 0))
    b = serve.synthetic_projection_torch(5, 64, 256, torch.device("cuda", 0))
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
    assert int(a[0].max()) > 200 and float(a[1].float().abs().max()) > 0
