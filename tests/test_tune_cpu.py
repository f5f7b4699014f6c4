"""The tuner's deterministic half on the CPU (the timing half needs a GPU): the committed dispatch
table is exactly what tune.py builds from the candidate timings recorded beside it (its --from-json
path), the built-in C string is that table, and the tie rule that lets buckets merge (the reference's
tuner keeps the fastest forced candidate per L, web/public/engine/tune.html:8-24)."""
import importlib
import json
import os

from conftest import load_package

load_package()
tune = importlib.import_module("strands_decider_web_b200.tune")
HERE = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "strands-decider-web_b200")


def test_committed_table_rebuilds_from_its_recorded_timings():
    old = json.load(open(os.path.join(HERE, "dispatch_table.json")))
    shapes = {k: tuple(v) for k, v in old["measured_on"]["shapes"].items()}
    ms = old["measured_on"]["M"]
    res = {}
    for name, (K, N) in shapes.items():
        prev = None
        for M in ms:
            key = f"{name}/M{M}"
            if key in old["candidates"]:
                res[(name, M)] = prev = tune.measured(name, K, N, M, old["candidates"][key], prev)
    table = tune.build_table(res, shapes, ms, old["measured_on"]["sm_count"])
    assert table["buckets"] == old["buckets"]
    # every kept candidate is one that ran and passed the oracle check
    for (name, M), r in res.items():
        assert isinstance(old["candidates"][f"{name}/M{M}"][tune._label(r["best"])], (int, float))


def test_builtin_string_is_written_from_the_table(tmp_path):
    old = json.load(open(os.path.join(HERE, "dispatch_table.json")))
    out = tmp_path / "t.inc"
    tune.write_inc(old, str(out))
    assert out.read_text() == open(os.path.join(HERE, "csrc", "dispatch_table.inc")).read()


def test_pick_prefers_previous_then_automatic_within_ties():
    t = {"tc/t0/g0/kernel": 10.2, "tc/t0/g148/kernel": 10.0, "tc/t128/g148/cta": 12.0, "gemv/s2": "FAIL max_rel"}
    # the fastest wins when nothing else is within 3 %
    assert tune.pick({"tc/t0/g148/kernel": 10.0, "tc/t0/g0/kernel": 11.0}, None) == \
        {"family": "tc", "tile": 0, "split": 148, "fixup": "kernel"}
    # within 3 %: the automatic candidate
    assert tune.pick(t, None) == {"family": "tc", "tile": 0, "split": 0, "fixup": "kernel"}
    # within 3 %: the previous M's choice before the automatic one (so consecutive Ms merge)
    prev = {"family": "tc", "tile": 0, "split": 148, "fixup": "kernel"}
    assert tune.pick(t, prev) == prev
    # a failed candidate is never kept, however it is labelled
    assert tune.pick({"gemv/s2": "FAIL", "gemv/s0": 5.0}, {"family": "gemv", "split": 2}) == \
        {"family": "gemv", "split": 0}


def test_has_split_matches_the_work_split():
    # gate|up at M = 64 on 96 CTAs: 96 whole tiles, nothing split; on 148 CTAs: stream-K splits tiles
    assert not tune.has_split(64, 2048, 12288, 64, 96)
    assert tune.has_split(64, 2048, 12288, 64, 148)
    # down at M = 2048, 240-token tiles on 144 CTAs: 144 whole tiles
    assert not tune.has_split(2048, 6144, 2048, 240, 144)
