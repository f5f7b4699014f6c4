"""On-disk cache of repacked weights (s4_weight_save / s4_weight_load): a loaded weight has the saved
device layout and gives bit-identical matmuls; a missing, truncated, corrupt or other-version file is
reported as S4_ERR_IO so the caller uploads from the shard again (WeightCache.get)."""
import numpy as np
import pytest

from oracle import s4ref

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _weights(ctx, rng, K, N, asym):
    if not asym:
        packed, scales = s4ref.config_weights(rng, K, N)
        return ctx.upload(packed, scales, N, K)
    words = s4ref.pack_format(rng.integers(0, 8, (N, K)), 3)
    sc = (np.abs(rng.standard_normal((N, K // 64))) * 0.005).astype(np.float16)
    return ctx.upload_format(words, sc, N, K, 3, 64, bias=(-3.5 * sc).astype(np.float16))


@pytest.mark.parametrize("asym", [False, True])
def test_save_load_round_trip(ctx, tmp_path, asym):
    rng = np.random.default_rng(3 + asym)
    K, N = 2048, 1000
    W = _weights(ctx, rng, K, N, asym)
    path = str(tmp_path / "w.s4w")
    W.save(path)
    L = ctx.load_weight(path)
    assert (L.N, L.K, L.device_bytes) == (N, K, W.device_bytes)
    for a, b in zip(W.layout(), L.layout()):
        np.testing.assert_array_equal(a, b)
    for M in (1, 300):
        x = torch.from_numpy(s4ref.config_x(rng, M, K)).cuda()
        ya, yb = ctx.matmul(x, W), ctx.matmul(x, L)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(ya.cpu().numpy().view(np.uint16), yb.cpu().numpy().view(np.uint16))
    W.free()
    L.free()


def test_bad_entries_are_io_errors(ctx, pkg, tmp_path):
    rng = np.random.default_rng(9)
    W = _weights(ctx, rng, 256, 200, False)
    good = tmp_path / "good.s4w"
    W.save(str(good))
    data = good.read_bytes()
    cases = {"missing": None, "truncated": data[:-7], "corrupt": data[:100] + bytes([data[100] ^ 1]) + data[101:],
             "version": data[:4] + (99).to_bytes(4, "little") + data[8:], "trailing": data + b"\0",
             "header": data[:30]}
    for name, content in cases.items():
        p = tmp_path / f"{name}.s4w"
        if content is not None:
            p.write_bytes(content)
        with pytest.raises(pkg.S4Error) as e:
            ctx.load_weight(str(p))
        assert e.value.code == pkg.s4mm.ERR_IO, name
    W.free()


def test_weight_cache_get(ctx, pkg, tmp_path):
    rng = np.random.default_rng(11)
    packed, scales = s4ref.config_weights(rng, 1024, 512)
    cache = pkg.WeightCache(str(tmp_path), pkg.cache_prefix("rev1", "base/", "{}", "{}"))
    calls = []

    def upload():
        calls.append(1)
        return ctx.upload(packed, scales, 512, 1024)

    W1, hit1 = cache.get(ctx, "layers.0.mlp.down_proj", upload)
    W2, hit2 = cache.get(ctx, "layers.0.mlp.down_proj", upload)
    assert (hit1, hit2, len(calls)) == (False, True, 1)
    for a, b in zip(W1.layout(), W2.layout()):
        np.testing.assert_array_equal(a, b)
    W1.free()
    W2.free()
    assert ctx.check_errors() == 0
