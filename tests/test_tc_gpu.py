"""The tcgen05 GEMM family forced through the dispatcher: every token count, tile size and
stream-K split must agree with the CPU oracle within the north-star tolerance (max relative
error 2e-3, per-row cosine 0.99999)."""
import numpy as np
import pytest

from oracle import s4ref

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _run(ctx, W, x):
    y = ctx.matmul(torch.from_numpy(x).cuda(), W)
    torch.cuda.synchronize()
    return y.cpu().numpy()


def _check(y, ref, what):
    ok, mr, mc = s4ref.check(y, ref)
    assert ok, f"{what}: max_rel={mr:.3e} min_cos={mc:.7f}"


@pytest.fixture(scope="module")
def shapes(ctx):
    rng = np.random.default_rng(77)
    out = {}
    for K, N in [(2048, 3072), (6144, 2048), (96, 200), (2048, 8224)]:
        packed, scales = s4ref.config_weights(rng, K, N)
        out[(K, N)] = (packed, scales, s4ref.dequant(packed, scales), ctx.upload(packed, scales, N, K))
    return out


@pytest.fixture
def forced(ctx):
    def f(tile=0, split=0):
        ctx.force("tc", tile, split)
    yield f
    ctx.force("auto")


@pytest.mark.parametrize("M", [1, 5, 16, 33, 100, 256, 257, 600])
@pytest.mark.parametrize("KN", [(2048, 3072), (6144, 2048), (96, 200)])
def test_tc_all_m(ctx, shapes, forced, KN, M):
    packed, scales, deq, W = shapes[KN]
    forced()
    x = s4ref.config_x(np.random.default_rng(M + KN[0]), M, KN[0])
    _, ref = s4ref.matmul(x, packed, scales, deq)
    _check(_run(ctx, W, x), ref, f"tc K,N={KN} M={M}")


@pytest.mark.parametrize("tile", [16, 64, 128, 256])
def test_tc_tiles(ctx, shapes, forced, tile):
    packed, scales, deq, W = shapes[(2048, 8224)]
    forced(tile=tile)
    x = s4ref.config_x(np.random.default_rng(tile), 300, 2048)
    _, ref = s4ref.matmul(x, packed, scales, deq)
    _check(_run(ctx, W, x), ref, f"tile={tile}")


@pytest.mark.parametrize("split", [1, 3, 7, 64, 148])
def test_tc_stream_k_splits(ctx, shapes, forced, split):
    packed, scales, deq, W = shapes[(6144, 2048)]
    forced(split=split)
    x = s4ref.config_x(np.random.default_rng(split), 70, 6144)
    _, ref = s4ref.matmul(x, packed, scales, deq)
    _check(_run(ctx, W, x), ref, f"split={split}")


def test_tc_deterministic(ctx, shapes, forced):
    packed, scales, deq, W = shapes[(2048, 3072)]
    forced()
    x = s4ref.config_x(np.random.default_rng(3), 200, 2048)
    a, b = _run(ctx, W, x), _run(ctx, W, x)
    np.testing.assert_array_equal(a.view(np.uint16), b.view(np.uint16))


def test_tc_and_gemv_agree(ctx, shapes):
    packed, scales, deq, W = shapes[(2048, 3072)]
    x = s4ref.config_x(np.random.default_rng(9), 24, 2048)
    ctx.force("gemv")
    a = _run(ctx, W, x)
    ctx.force("tc")
    b = _run(ctx, W, x)
    ctx.force("auto")
    _check(b, a.astype(np.float32), "tc vs gemv")
    assert ctx.check_errors() == 0


@pytest.mark.parametrize("K,N,M", [(6144, 2048, 2048), (2048, 2048, 2048), (2048, 12288, 512), (2048, 12288, 768)])
def test_whole_wave_tile_shapes(ctx, K, N, M):
    """Automatic shapes that pack whole tiles into whole waves: one wave of 240-token tiles (16 n-blocks
    at M = 2048) and two exact waves of 176- / 256-token tiles (96 n-blocks at M = 512 / 768)."""
    rng = np.random.default_rng(K + N + M)
    packed, scales = s4ref.config_weights(rng, K, N)
    W = ctx.upload(packed, scales, N, K)
    x = s4ref.config_x(rng, M, K)
    _, ref = s4ref.matmul(x, packed, scales)
    _check(_run(ctx, W, x), ref, f"K={K} N={N} M={M}")
    W.free()


@pytest.mark.parametrize("K,N", [(6144, 2048), (2048, 12288), (2048, 3072)])
@pytest.mark.parametrize("M", [16, 64, 130, 300])
@pytest.mark.parametrize("grid", [148, 37])
def test_tc_fixup_modes(ctx, K, N, M, grid):
    """Split tiles summed by the fix-up kernel or by their last CTA (in-kernel, either straight from
    TMEM or from the published partials): both meet the tolerance and are bitwise identical, since
    both add the parts in CTA order."""
    rng = np.random.default_rng(K + N + M + grid)
    packed, scales = s4ref.config_weights(rng, K, N)
    W = ctx.upload(packed, scales, N, K)
    x = s4ref.config_x(rng, M, K)
    _, ref = s4ref.matmul(x, packed, scales)
    outs = {}
    try:
        for fx in ("kernel", "cta"):
            ctx.set_table({"buckets": [{"max_m": 1 << 30, "family": "tc", "split": grid, "fixup": fx}]})
            for rep in range(2):  # twice: the tickets must be back at zero after each call
                outs[(fx, rep)] = _run(ctx, W, x)
                _check(outs[(fx, rep)], ref, f"K={K} N={N} M={M} grid={grid} fixup={fx} call {rep}")
    finally:
        ctx.set_table(None)
    for k, v in outs.items():
        np.testing.assert_array_equal(v.view(np.uint16), outs[("kernel", 0)].view(np.uint16), err_msg=str(k))
    assert ctx.check_errors() == 0
    W.free()


def test_table_shape_buckets(ctx):
    """Buckets with K / N apply to their shape only; other shapes fall through to the general ones;
    s4_plan reports the tile and CTA count a tcgen05 call launches with."""
    try:
        ctx.set_table({"buckets": [
            {"max_m": 64, "K": 6144, "N": 2048, "family": "tc", "tile": 32, "split": 100, "fixup": "cta"},
            {"max_m": 16, "family": "gemv"}, {"max_m": 1 << 30, "family": "tc"}]})
        assert ctx.plan(64, 2048, 6144) == ("tc", 32, 100)
        assert ctx.plan(65, 2048, 6144)[0] == "tc" and ctx.plan(65, 2048, 6144)[1] == 80
        assert ctx.plan(8, 2048, 6144) == ("tc", 32, 100)
        assert ctx.plan(8, 3072, 2048)[0] == "gemv"
        assert ctx.plan(64, 3072, 2048)[0] == "tc"
        with pytest.raises(Exception):
            ctx.set_table({"buckets": [{"max_m": 64, "K": 6144, "family": "tc"}]})  # no general bucket
        with pytest.raises(Exception):
            ctx.set_table({"buckets": [{"max_m": 64, "family": "tc", "fixup": "sometimes"}]})
    finally:
        ctx.set_table(None)


def test_tc_few_leftover_units(ctx):
    """Fewer leftover stream-K units than CTAs (65 n-blocks x 16 token blocks of 128 on 148 CTAs: 4
    leftover tiles of 32 k-tiles): one wave of whole tiles joins the stream-K part so that no CTA
    inside a split tile's span has an empty range, with either fix-up."""
    K, N, M = 2048, 8224, 2048
    rng = np.random.default_rng(5)
    packed, scales = s4ref.config_weights(rng, K, N)
    W = ctx.upload(packed, scales, N, K)
    x = s4ref.config_x(rng, M, K)
    _, ref = s4ref.matmul(x, packed, scales)
    try:
        for fx in ("kernel", "cta"):
            ctx.set_table({"buckets": [{"max_m": 1 << 30, "family": "tc", "tile": 128, "split": 148, "fixup": fx}]})
            _check(_run(ctx, W, x), ref, f"tile 128 fixup={fx}")
    finally:
        ctx.set_table(None)
    assert ctx.check_errors() == 0
    W.free()
