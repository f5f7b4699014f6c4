"""Parity of the CUDA path (through the C ABI) with the CPU oracle, on a B200.

Tolerance: max relative error max|y - ref| / max|ref| <= 2e-3 and per-row
cosine >= 0.99999 against the fp32 dequantise-then-matmul oracle. Integer work (the repacked
layout) is compared bit-exactly.
"""
import os

import numpy as np
import pytest

from oracle import s4ref

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
TOL, COS = s4ref.TOL_MAX_REL, s4ref.TOL_MIN_COSINE

FUSED_SHAPES = {  # (K, N) of the fused projections
    "qkvz_ab": (2048, 8224),
    "attn_qkv": (2048, 3072),
    "gate_up": (2048, 12288),
    "down": (6144, 2048),
}


def run(ctx, W, x16: np.ndarray, **kw):
    x = torch.from_numpy(x16).cuda()
    y = ctx.matmul(x, W, **kw)
    torch.cuda.synchronize()
    return y.cpu().numpy()


def assert_parity(y, ref, what=""):
    ok, mr, mc = s4ref.check(y, ref, TOL, COS)
    assert ok, f"{what}: max_rel={mr:.3e} (tol {TOL}), min_row_cos={mc:.7f} (tol {COS})"
    assert np.isfinite(y.astype(np.float32)).all()


@pytest.fixture(scope="module")
def weights(ctx):
    rng = np.random.default_rng(0)
    out = {}
    for name, (K, N) in FUSED_SHAPES.items():
        packed, scales = s4ref.config_weights(rng, K, N)
        out[name] = (packed, scales, s4ref.dequant(packed, scales), ctx.upload(packed, scales, N, K))
    return out


# ---- upload / repack ----------------------------------------------------------------------------
@pytest.mark.parametrize("N,K", [(8224, 2048), (2048, 6144), (130, 96), (1, 32), (16, 64), (300, 160)])
def test_repack_layout_bit_exact(ctx, N, K):
    rng = np.random.default_rng(N + K)
    packed, scales = s4ref.config_weights(rng, K, N)
    W = ctx.upload(packed, scales, N, K)
    wq, ws = W.layout()
    rq, rs = s4ref.repack_device(packed, scales, N, K)
    np.testing.assert_array_equal(wq, rq.ravel())
    np.testing.assert_array_equal(ws.view(np.uint16), rs.ravel().view(np.uint16))
    p2, s2 = s4ref.unrepack_device(wq, ws, N, K)
    np.testing.assert_array_equal(p2, packed)


def test_upload_from_device_pointers(ctx):
    rng = np.random.default_rng(11)
    packed, scales = s4ref.config_weights(rng, 256, 200)
    Wh = ctx.upload(packed, scales, 200, 256)
    Wd = ctx.upload(torch.from_numpy(packed).cuda(), torch.from_numpy(scales).cuda(), 200, 256)
    for a, b in zip(Wh.layout(), Wd.layout()):
        np.testing.assert_array_equal(a.view(np.uint8), b.view(np.uint8))


# ---- golden fixtures (reference quantiser + fp32 nn.Linear) -------------------------------------
def _golden_names():
    z = np.load(os.path.join(GOLDEN, "matmul_cases.npz"))
    return sorted({k.split("/")[0] for k in z.files})


@pytest.mark.parametrize("name", _golden_names())
def test_matches_reference_golden(ctx, name):
    z = np.load(os.path.join(GOLDEN, "matmul_cases.npz"))
    x, packed, scales, y32 = (z[f"{name}/{k}"] for k in ("x", "packed", "scales", "y32"))
    N, K = packed.shape[0], packed.shape[1] * 32
    W = ctx.upload(packed, scales, N, K)
    assert_parity(run(ctx, W, x), y32, name)


# ---- BASELINE config shapes -----------------------------------------------------------------------
@pytest.mark.parametrize("M", [1, 2, 4, 8])
@pytest.mark.parametrize("shape", list(FUSED_SHAPES))
def test_decode_sweep_config2(ctx, weights, shape, M):
    packed, scales, deq, W = weights[shape]
    x = s4ref.config_x(np.random.default_rng(M), M, FUSED_SHAPES[shape][0])
    _, ref = s4ref.matmul(x, packed, scales, deq)
    assert_parity(run(ctx, W, x), ref, f"{shape} M={M}")


def test_gate_up_m64_config1(ctx, weights):
    packed, scales, deq, W = weights["gate_up"]
    x = s4ref.config_x(np.random.default_rng(64), 64, 2048)
    _, ref = s4ref.matmul(x, packed, scales, deq)
    assert_parity(run(ctx, W, x), ref, "gate_up M=64")


@pytest.mark.parametrize("M", [16, 64, 128, 512, 2048])
@pytest.mark.parametrize("shape", ["down", "gate_up"])
def test_prefill_sweep_config3(ctx, weights, shape, M):
    packed, scales, deq, W = weights[shape]
    x = s4ref.config_x(np.random.default_rng(1000 + M), M, FUSED_SHAPES[shape][0])
    _, ref = s4ref.matmul(x, packed, scales, deq)
    assert_parity(run(ctx, W, x), ref, f"{shape} M={M}")


# ---- ragged shapes and edge cases ---------------------------------------------------------------
@pytest.mark.parametrize("N,K", [(1, 32), (15, 96), (17, 64), (130, 32), (8224, 96), (256, 6176)])
@pytest.mark.parametrize("M", [1, 3, 9, 31, 33, 70])
def test_ragged_shapes(ctx, N, K, M):
    rng = np.random.default_rng(N * 31 + K * 7 + M)
    packed, scales = s4ref.config_weights(rng, K, N)
    W = ctx.upload(packed, scales, N, K)
    x = s4ref.config_x(rng, M, K)
    _, ref = s4ref.matmul(x, packed, scales)
    assert_parity(run(ctx, W, x), ref, f"N={N} K={K} M={M}")


def test_zero_rows_and_m0(ctx, weights):
    _, _, _, W = weights["down"]
    y = torch.full((3, W.N), 7.0, dtype=torch.float16, device="cuda")
    ctx.matmul(torch.zeros((3, W.K), dtype=torch.float16, device="cuda"), W, 3, y)
    torch.cuda.synchronize()
    assert float(y.abs().max()) == 0.0
    ctx.matmul(torch.zeros((1, W.K), dtype=torch.float16, device="cuda"), W, 0, y)  # M == 0: no-op


def test_reference_quantised_weights_negative_scales(ctx):
    rng = np.random.default_rng(21)
    Wf = (rng.standard_normal((384, 2048)) * 0.02).astype(np.float32)
    packed, scales, deq = s4ref.quant(Wf)
    assert (scales < 0).any() and (scales > 0).any()
    W = ctx.upload(packed, scales, 384, 2048)
    for M in (1, 8, 40):
        x = s4ref.config_x(rng, M, 2048)
        _, ref = s4ref.matmul(x, packed, scales, deq)
        assert_parity(run(ctx, W, x), ref, f"quant M={M}")


def test_deterministic(ctx, weights):
    packed, scales, deq, W = weights["qkvz_ab"]
    x = s4ref.config_x(np.random.default_rng(5), 8, 2048)
    a = run(ctx, W, x)
    b = run(ctx, W, x)
    np.testing.assert_array_equal(a.view(np.uint16), b.view(np.uint16))


@pytest.mark.parametrize("split", [1, 3, 7, 16, 0])
def test_forced_gemv_splits(ctx, weights, split):
    packed, scales, deq, W = weights["attn_qkv"]
    x = s4ref.config_x(np.random.default_rng(split), 5, 2048)
    _, ref = s4ref.matmul(x, packed, scales, deq)
    ctx.force("gemv", 0, split)
    try:
        assert ctx.plan(5)[0] == "gemv"
        assert_parity(run(ctx, W, x), ref, f"split={split}")
    finally:
        ctx.force("auto")


# ---- host-buffer path and the Gemm object -------------------------------------------------------
def test_host_path_equals_device_path(ctx, weights):
    packed, scales, deq, W = weights["gate_up"]
    x = s4ref.config_x(np.random.default_rng(8), 8, 2048)
    yd = run(ctx, W, x)
    yh = ctx.matmul_host(x, W)
    np.testing.assert_array_equal(yd.view(np.uint16), yh.view(np.uint16))


def test_gemm_object_mirror_with_bench_check(ctx, pkg):
    """The gemmbench flow (bench.js:37-54): make_gemm weights, sin() activations, setA/encode/
    readY, and the fp32 CPU check on columns {0, 1, N/2, N-1}."""
    rng = np.random.default_rng(0)
    K, N = 2048, 6144
    packed, scales = s4ref.make_gemm_weights(rng, K, N)
    g = pkg.Gemm(ctx, K=K, N=N, B=packed, Sc=scales.view(np.uint16))
    for M in (1, 8, 16, 64):
        A = (np.sin(np.arange(M * K) * 12.9898) * 0.5).astype(np.float16)
        g.setA(M, A.view(np.uint16))
        g.encode()
        y = g.readY().view(np.float16).reshape(M, N)
        pts = s4ref.cpu_check_columns(A.reshape(M, K), packed, scales, [0, 1, N >> 1, N - 1])
        err = max(abs(float(y[m, n]) - v) for (m, n), v in pts.items())
        mag = max(abs(v) for v in pts.values())
        assert err / mag <= TOL, (M, err / mag)


# ---- SiLU * mul -----------------------------------------------------------------------------------
@pytest.mark.parametrize("M,I", [(1, 6144), (64, 6144), (3, 13), (2048, 6144)])
def test_silu_mul(ctx, M, I):
    rng = np.random.default_rng(M + I)
    big = (rng.standard_normal((M, 2 * I)) * 3).astype(np.float16)
    mid = ctx.silu_mul(torch.from_numpy(big).cuda(), I)
    torch.cuda.synchronize()
    ref = s4ref.silu_mul(big, I)
    got = mid.cpu().numpy().astype(np.float32)
    np.testing.assert_allclose(got, ref.astype(np.float32), rtol=2e-3, atol=2e-3)


# ---- dispatcher -----------------------------------------------------------------------------------
def test_dispatch_table(pkg):
    c = pkg.Context(0)
    try:
        c.set_table({"buckets": [{"max_m": 8, "family": "gemv", "split": 12}, {"max_m": 1 << 30, "family": "gemv"}]})
        assert c.plan(4) == ("gemv", 0, 12)
        assert c.plan(100)[0] == "gemv"
        with pytest.raises(pkg.S4Error):
            c.set_table('{"buckets": [{"max_m": 8, "family": "nope"}]}')
        with pytest.raises(pkg.S4Error):
            c.set_table('{"buckets": [{"max_m": 8, "family": "gemv"}, {"max_m": 4, "family": "gemv"}]}')
    finally:
        c.close()


def test_no_device_errors_and_launches_counted(ctx):
    assert ctx.check_errors() == 0
    assert ctx.launch_count > 0
