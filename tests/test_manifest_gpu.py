"""Projections uploaded by name from an exported engine's shards (s4_weight_upload_named: the shard
upload + w(name) binding of Engine.create, web/public/engine/engine.js:76-84, 175-180), from host and
from device shard buffers, then multiplied and checked against the CPU oracle (max relative error
2e-3, per-row cosine 0.99999); the device layout equals a direct upload of the same bytes."""
import numpy as np
import pytest

from oracle import s4ref

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _engine():
    rng = np.random.default_rng(11)
    tensors = [
        ("layers.0.in_norm", (1 + 0.01 * rng.standard_normal(2048)).astype(np.float32)),
        ("layers.0.in_proj", "q", (0.02 * rng.standard_normal((8224, 2048))).astype(np.float32)),  # -> 8256 rows
        ("layers.0.out_proj", "q", (0.02 * rng.standard_normal((2048, 2048))).astype(np.float32)),
        ("layers.0.gate_up", "q", (0.02 * rng.standard_normal((1024, 512))).astype(np.float32)),
        ("layers.0.down", "q", (0.02 * rng.standard_normal((512, 1024))).astype(np.float32)),
    ]
    return s4ref.export_engine(tensors, shard_limit=6 << 20)


@pytest.mark.parametrize("where", ["host", "device"])
def test_upload_named(pkg, ctx, where):
    manifest, shards, quantised = _engine()
    assert len(shards) > 1
    m = pkg.Manifest(manifest)
    bufs = [np.frombuffer(s, np.uint8) for s in shards]
    if where == "device":
        bufs = [torch.from_numpy(b.copy()).cuda() for b in bufs]
    for name, (packed, scales) in quantised.items():
        W = ctx.upload_named(m, bufs, name)
        N, K = packed.shape[0], packed.shape[1] * 32
        assert (W.N, W.K) == (N, K)
        ref_w = ctx.upload(packed, scales, N, K)
        a, b = W.layout(), ref_w.layout()
        np.testing.assert_array_equal(a[0], b[0])
        np.testing.assert_array_equal(a[1].view(np.uint16), b[1].view(np.uint16))
        for M in (1, 37):
            x = s4ref.config_x(np.random.default_rng(M), M, K)
            y = ctx.matmul(torch.from_numpy(x).cuda(), W)
            torch.cuda.synchronize()
            _, ref = s4ref.matmul(x, packed, scales)
            ok, mr, mc = s4ref.check(y.cpu().numpy(), ref)
            assert ok, f"{name} M={M}: max_rel={mr:.2e} min_cos={mc:.7f}"
        W.free()
        ref_w.free()
    with pytest.raises(pkg.S4Error, match="no tensor"):
        ctx.upload_named(m, bufs, "layers.7.in_proj")
    with pytest.raises(pkg.S4Error):
        ctx.upload_named(m, bufs, "layers.0.in_norm")  # not a projection: no .q / .s pair
