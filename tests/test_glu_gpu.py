"""Fused gate|up projections whose matmul writes SiLU*mul (s4_weight_upload_glu): y[M][I] =
silu(x W_gate^T) * (x W_up^T) (wgsl.js:81-90 in the GEMM epilogue) against the oracle's fp32
dequantise-then-matmul followed by its SiLU*mul, within the north-star tolerance, for the GEMV
(M <= 16), whole-tile and split-tile (fix-up) tcgen05 paths and the multi-destination gather; and
against the unfused GPU path (matmul, then s4_silu_mul), which computes from the same fp16 values."""
import numpy as np
import pytest

from oracle import s4ref

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _gate_up(rng, I, K):
    return s4ref.config_weights(rng, K, 2 * I)


@pytest.mark.parametrize("I,K", [(6144, 2048), (1536, 2048), (192, 1024)])
def test_glu_matches_oracle_and_unfused(ctx, I, K):
    rng = np.random.default_rng(I + K)
    packed, scales = _gate_up(rng, I, K)
    W = ctx.upload_glu(packed, scales, I, K)
    Wp = ctx.upload(packed, scales, 2 * I, K)
    assert W.N == I
    deq = s4ref.dequant(packed, scales)
    for M in (1, 5, 16, 17, 300, 512, 2048):  # 512: two whole waves of 176-token tiles (I = 6144)
        x = s4ref.config_x(rng, M, K)
        xd = torch.from_numpy(x).cuda()
        y = ctx.matmul(xd, W)
        ref_big, _ = s4ref.matmul(x, packed, scales, deq)
        unfused = ctx.silu_mul(ctx.matmul(xd, Wp), I)
        torch.cuda.synchronize()
        assert y.shape == (M, I)
        got = y.cpu().numpy()
        ok, mr, mc = s4ref.check(got, s4ref.silu_mul(ref_big, I).astype(np.float32))
        assert ok, f"I={I} M={M}: max_rel={mr:.2e} min_cos={mc:.7f}"
        # same fp16 gate / up values up to fp32 summation order (which tiles are split differs)
        diff = got.view(np.uint16) != unfused.cpu().numpy().view(np.uint16)
        assert diff.mean() < 0.01, f"I={I} M={M}: {diff.mean():.4f} of outputs differ from the unfused path"
    assert ctx.check_errors() == 0
    W.free()
    Wp.free()


def test_glu_gather_and_cache(ctx, pkg, tmp_path):
    """Two local destinations through s4_matmul_gather (the column-sharded form) equal s4_matmul; a
    cached fused weight reloads as fused."""
    rng = np.random.default_rng(5)
    I, K, M = 768, 2048, 256
    packed, scales = _gate_up(rng, I, K)
    W = ctx.upload_glu(packed, scales, I, K)
    x = torch.from_numpy(s4ref.config_x(rng, M, K)).cuda()
    ref = ctx.matmul(x, W)
    ldy = 2 * I
    bufs = [torch.zeros((M, ldy), dtype=torch.float16, device="cuda") for _ in range(2)]
    ctx.matmul_gather(x.data_ptr(), K, M, W, [b.data_ptr() for b in bufs], ldy, I)
    torch.cuda.synchronize()
    for b in bufs:
        assert torch.equal(b[:, I:], ref)
        assert torch.count_nonzero(b[:, :I]) == 0
    path = str(tmp_path / "glu.s4w")
    W.save(path)
    L = ctx.load_weight(path)
    assert L.N == I
    y2 = ctx.matmul(x, L)
    torch.cuda.synchronize()
    assert torch.equal(y2, ref)
    W.free()
    L.free()


def test_glu_errors(ctx, pkg):
    rng = np.random.default_rng(6)
    packed, scales = _gate_up(rng, 96, 256)
    with pytest.raises(pkg.S4Error):  # I not a multiple of 64
        ctx.upload_glu(packed, scales, 96, 256)
    packed, scales = _gate_up(rng, 128, 256)
    W = ctx.upload_glu(packed, scales, 128, 256)
    x = torch.from_numpy(s4ref.config_x(rng, 2, 256)).cuda()
    y = torch.empty((2, 128), dtype=torch.float16, device="cuda")
    with pytest.raises(pkg.S4Error) as e:
        ctx.chain([(x, W, y)])
    assert e.value.code == pkg.s4mm.ERR_UNSUPPORTED
    lib = pkg.load_library()
    assert lib.s4_matmul_noalloc(W.handle, x.data_ptr(), 2, y.data_ptr(), None) == pkg.s4mm.ERR_UNSUPPORTED
    W.free()
    assert ctx.check_errors() == 0
