"""The weight manifest reader (s4_manifest_*): the exporter's tensor index and shard layout
(convert/export_engine.py:29-43, 70-85, restated in the oracle to build fixtures) resolved like the
engine's w(name) (web/public/engine/engine.js:175-180). No GPU needed."""
import json

import numpy as np
import pytest

from oracle import s4ref


def _engine(shard_limit):
    rng = np.random.default_rng(3)
    tensors = [
        ("layers.0.in_norm", (1 + 0.01 * rng.standard_normal(2048)).astype(np.float32)),
        ("layers.0.in_proj", "q", rng.standard_normal((200, 256)).astype(np.float32)),  # N pads to 256
        ("layers.0.conv", rng.standard_normal((37, 4)).astype(np.float32)),              # odd size: padding
        ("layers.0.out_proj", "q", rng.standard_normal((128, 192)).astype(np.float32)),
        ("layers.0.down", "q", rng.standard_normal((64, 512)).astype(np.float32)),
    ]
    return s4ref.export_engine(tensors, shard_limit=shard_limit, config={"hidden_size": 2048})


@pytest.mark.parametrize("limit,nshards", [(512 << 20, 1), (40000, 3), (9000, 7)])
def test_manifest_resolves_like_the_engine(pkg, limit, nshards):
    manifest, shards, quantised = _engine(limit)
    assert len(shards) == nshards
    m = pkg.Manifest(manifest)
    assert [b for _, b in m.shards] == [len(s) for s in shards]
    assert [p for p, _ in m.shards] == [s["path"] for s in manifest["shards"]]
    for name, t in manifest["tensors"].items():
        got = m.tensor(name)
        shard, off = s4ref.resolve_tensor(manifest, name)
        assert (got["shard"], got["offset"], got["bytes"]) == (shard, off, t["bytes"])
        assert (got["N"], got["K"]) == (t.get("N", -1), t.get("K", -1))
        # the bytes at the resolved range are the tensor's own
        base, kind = name.rsplit(".", 1)
        if base in quantised:
            arr = quantised[base][0 if kind == "q" else 1]
            assert shards[shard][off:off + t["bytes"]] == arr.tobytes()
    q = m.tensor("layers.0.in_proj.q")
    assert q["N"] == 256 and q["K"] == 256  # padded to a multiple of 64 rows (export_engine.py:37-38)
    m.close()


def test_manifest_errors(pkg):
    manifest, _, _ = _engine(512 << 20)
    m = pkg.Manifest(json.dumps(manifest))
    with pytest.raises(pkg.S4Error, match="no tensor layers.9.in_proj.q"):
        m.tensor("layers.9.in_proj.q")
    for bad in ('{"tensors": {}}', '{"shards": [{"path": "a", "start": 0, "bytes": 4}]}', "{", '{"shards": [],',
                '{"shards": [{"path": "a", "start": 0, "bytes": 4}], "tensors": {"x": {"bytes": 4}}}',
                '{"shards": [{"path": "a", "start": 0, "bytes": 4.5}], "tensors": {}}'):
        with pytest.raises(pkg.S4Error):
            pkg.Manifest(bad)
    # a tensor that would run past its shard's end
    broken = json.loads(json.dumps(manifest))
    broken["tensors"]["layers.0.down.s"]["bytes"] = 1 << 30
    mb = pkg.Manifest(broken)
    with pytest.raises(pkg.S4Error, match="runs past the end"):
        mb.tensor("layers.0.down.s")
