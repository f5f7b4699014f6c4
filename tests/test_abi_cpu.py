"""C-ABI checks that need no GPU: the library loads, exports every declared entry point, and
rejects bad arguments with a status and a message instead of crashing."""
import ctypes as C
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "s4mm.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^S4_API\s+[\w\s\*]+?\b(s4_\w+)\(", text, flags=re.M)))


def test_header_declares_the_boundary():
    syms = declared_symbols()
    for must in ("s4_init", "s4_destroy", "s4_weight_upload", "s4_matmul", "s4_matmul_host", "s4_silu_mul",
                 "s4_plan", "s4_force", "s4_set_table", "s4_last_error"):
        assert must in syms


def test_library_exports_every_declared_symbol(pkg):
    lib = pkg.load_library()
    raw = C.CDLL(pkg.LIB_PATH)
    for name in declared_symbols():
        assert hasattr(raw, name), name
    assert set(declared_symbols()) == set(pkg.s4mm._SIGS), "ctypes bindings out of sync with the header"
    assert lib.s4_version() >> 16 == 1


def test_errors_without_work(pkg):
    lib = pkg.load_library()
    h = C.c_void_p()
    # NULL out-pointer -> invalid argument, with a message
    assert lib.s4_init(0, None) == pkg.s4mm.ERR_INVALID
    assert b"NULL" in lib.s4_last_error()
    # null context / weight handles
    assert lib.s4_matmul(None, None, None, 1, None, None) == pkg.s4mm.ERR_INVALID
    assert lib.s4_weight_upload(None, None, None, 16, 64, 0, C.byref(h)) == pkg.s4mm.ERR_INVALID
    assert lib.s4_set_table(None, b"{}") == pkg.s4mm.ERR_INVALID
    assert lib.s4_weight_free(None) == 0
    assert lib.s4_destroy(None) == 0


def test_init_without_gpu_fails_cleanly(pkg):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(pkg.S4Error) as e:
        pkg.Context(0)
    assert e.value.code in (pkg.s4mm.ERR_UNSUPPORTED, pkg.s4mm.ERR_CUDA)


def test_missing_library_is_loud(pkg, tmp_path):
    saved = pkg.s4mm._lib
    pkg.s4mm._lib = None
    try:
        with pytest.raises(pkg.S4Error):
            pkg.s4mm.load_library(str(tmp_path / "missing.so"))
    finally:
        pkg.s4mm._lib = saved


def test_new_entry_points_reject_null_arguments(pkg, tmp_path):
    """The format, wire, FWHT, fused gate|up and cache entry points fail with a status on NULL handles
    before touching a device."""
    lib = pkg.load_library()
    h = C.c_void_p()
    INV = pkg.s4mm.ERR_INVALID
    assert lib.s4_weight_upload_format(None, None, None, None, 16, 64, 2, 32, 0, C.byref(h)) == INV
    assert lib.s4_weight_upload_glu(None, None, None, 64, 64, 0, C.byref(h)) == INV
    assert lib.s4_weight_upload_wire(None, None, None, 16, 64, 0, C.byref(h)) == INV
    assert lib.s4_decode_wire_scales(None, None, 4, 4, None, None) == INV
    assert lib.s4_fwht(None, None, 1, 64, 64, None) == INV
    assert lib.s4_weight_save(None, str(tmp_path / "w").encode()) == INV
    assert lib.s4_weight_load(None, str(tmp_path / "w").encode(), C.byref(h)) == INV
    assert b"NULL" in lib.s4_last_error()


def test_wrappers_refuse_tensors_the_kernels_would_overrun(pkg):
    """Context.matmul / silu_mul / chain / matmul_host check dtype, device, contiguity and shape
    against the weight before passing raw pointers to the library (ERR_INVALID, no library call):
    a wrong width or row count would be read or written out of bounds by the kernels."""
    import numpy as np
    torch = pytest.importorskip("torch")
    m = pkg.s4mm
    ctx = m.Context.__new__(m.Context)  # no device: the checks raise before any library call
    ctx.handle, ctx.device = None, 0
    W = m.Weight(ctx, None, 128, 64)
    cpu16 = torch.zeros((2, 64), dtype=torch.float16)
    cases = [
        lambda: ctx.matmul(cpu16, W),                                        # host tensor
        lambda: ctx.silu_mul(torch.zeros((2, 256), dtype=torch.float16), 128),
        lambda: ctx.chain([(cpu16, W, torch.zeros((2, 128), dtype=torch.float16))]),
        lambda: ctx.matmul_host(np.zeros((2, 32), np.float16), W),          # K mismatch
        lambda: ctx.matmul_host(np.zeros((2, 64), np.float32), W),          # dtype
        lambda: ctx.matmul_host(np.zeros((2, 64), np.float16), W, np.zeros((2, 64), np.float16)),  # y width
    ]
    for i, case in enumerate(cases):
        with pytest.raises(m.S4Error) as e:
            case()
        assert e.value.code == m.ERR_INVALID, i


def test_builtin_table_is_the_committed_json():
    """csrc/dispatch_table.inc (the library's built-in table) holds exactly the buckets of
    dispatch_table.json, and every bucket is well formed."""
    import json
    pkg_dir = os.path.join(ROOT, "strands-decider-web_b200")
    table = json.load(open(os.path.join(pkg_dir, "dispatch_table.json")))
    inc = open(os.path.join(pkg_dir, "csrc", "dispatch_table.inc")).read()
    text = "".join(re.findall(r'^\s*"(.*)"', inc, flags=re.M)).replace('\\"', '"').replace("\\\\", "\\")
    assert json.loads(text) == {"buckets": table["buckets"]}
    general = [b for b in table["buckets"] if not b.get("K") and not b.get("N")]
    assert general and general[-1]["max_m"] >= 1 << 30
    for b in table["buckets"]:
        assert b["family"] in ("gemv", "tc")
        assert b.get("fixup", "kernel") in ("auto", "kernel", "cta")
