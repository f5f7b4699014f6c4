"""The measured dispatch table (strands-decider-web_b200/dispatch_table.json, written by tune.py and
compiled into the library as its built-in table): s4_plan follows it, and a matmul at both edges of
every shape-specific bucket meets the north-star tolerance against the CPU oracle (max relative
error 2e-3, per-row cosine 0.99999) - the reference's tuner only requires every forced candidate to
run (web/public/engine/tune.html:14-21); this one also requires the numbers to be right."""
import json
import os

import numpy as np
import pytest

from oracle import s4ref

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TABLE = json.load(open(os.path.join(ROOT, "strands-decider-web_b200", "dispatch_table.json")))
SHAPE_BUCKETS = [b for b in TABLE["buckets"] if b.get("K") and b.get("N")]


def _edges():
    out, prev = [], {}
    for b in SHAPE_BUCKETS:
        key = (b["K"], b["N"])
        lo = prev.get(key, 0) + 1
        prev[key] = b["max_m"]
        for M in sorted({lo, min(b["max_m"], 300)}):
            if M >= lo:
                out.append((b["K"], b["N"], M, b))
    return out


@pytest.fixture(scope="module")
def weights(ctx):
    rng = np.random.default_rng(31)
    out = {}
    for b in SHAPE_BUCKETS:
        key = (b["K"], b["N"])
        if key not in out:
            packed, scales = s4ref.config_weights(rng, *key)
            out[key] = (packed, scales, s4ref.dequant(packed, scales), ctx.upload(packed, scales, key[1], key[0]))
    return out


@pytest.mark.parametrize("K,N,M,bucket", _edges(), ids=lambda v: str(v) if not isinstance(v, dict) else "")
def test_builtin_bucket(ctx, weights, K, N, M, bucket):
    ctx.set_table(None)  # the built-in (compiled-in) table
    fam, tile, split = ctx.plan(M, N, K)
    assert fam == bucket["family"]
    if fam == "tc":
        if bucket.get("tile"):
            assert tile == bucket["tile"]
        if bucket.get("split"):
            assert split == min(bucket["split"], ctx.sm_count)
    elif bucket.get("split"):
        assert split == bucket["split"]
    packed, scales, deq, W = weights[(K, N)]
    x = s4ref.config_x(np.random.default_rng(M), M, K)
    y = ctx.matmul(torch.from_numpy(x).cuda(), W)
    torch.cuda.synchronize()
    _, ref = s4ref.matmul(x, packed, scales, deq)
    ok, mr, mc = s4ref.check(y.cpu().numpy(), ref)
    assert ok, f"K={K} N={N} M={M} {bucket}: max_rel={mr:.2e} min_cos={mc:.7f}"
