"""Python host side of the int4 MatMulNBits path: ctypes bindings over ``libs4mm.so``.

The classes mirror the reference's JavaScript call surface so that code written against it maps
one to one:

* :class:`Gemm` is the standalone ``Gemm`` object of web/public/gemmbench/kernels.js:83-104
  (``constructor(device, {K, N, B, Sc})`` uploads, ``setA(M, A16)``, ``encode()``, ``readY()``).
* :meth:`Context.matmul` is the engine's ``matmul(A, wname, Y)`` closure
  (web/public/engine/engine.js:236-246) on device tensors, with the weight resolved beforehand
  (:meth:`Context.upload`, the engine's shard upload + ``w(name)``, engine.js:63-87,175-180).
* :meth:`Context.silu_mul` is the ``SILU_MUL`` step between gate|up and down (wgsl.js:81-90).

Errors: every C call returns a status; a non-zero one raises :class:`S4Error` with
``s4_last_error()``, as the reference throws ``Error`` (engine.js:177, 228). There is no CPU
fallback: if the library or a B200 is missing, construction raises.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libs4mm.so")

FAMILY_AUTO, FAMILY_GEMV, FAMILY_TC = 0, 1, 2
FAMILY_NAMES = {FAMILY_AUTO: "auto", FAMILY_GEMV: "gemv", FAMILY_TC: "tc"}
ERR_INVALID, ERR_CUDA, ERR_NOMEM, ERR_DEVICE, ERR_UNSUPPORTED, ERR_IO = 1, 2, 3, 4, 5, 6
UPLOAD_DEVICE = 1  # s4_weight_upload_format: pointers are device memory
UPLOAD_DECODE_LAYOUT = 2  # s4_weight_upload_format: symmetric 2-bit, also the native 2-bit decode layout

# Every symbol include/s4mm.h declares, with its ctypes signature.
_P = C.c_void_p
_SIGS = {
    "s4_version": (C.c_int, []),
    "s4_last_error": (C.c_char_p, []),
    "s4_init": (C.c_int, [C.c_int, C.POINTER(_P)]),
    "s4_destroy": (C.c_int, [_P]),
    "s4_weight_upload": (C.c_int, [_P, _P, _P, C.c_int, C.c_int, C.c_uint32, C.POINTER(_P)]),
    "s4_weight_upload_device": (C.c_int, [_P, _P, _P, C.c_int, C.c_int, C.c_uint32, C.POINTER(_P)]),
    "s4_decode_wire_scales": (C.c_int, [_P, _P, C.c_int, C.c_int, _P, _P]),
    "s4_weight_upload_wire": (C.c_int, [_P, _P, _P, C.c_int, C.c_int, C.c_uint32, C.POINTER(_P)]),
    "s4_weight_upload_format": (C.c_int, [_P, _P, _P, _P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_uint32,
                                          C.POINTER(_P)]),
    "s4_fwht": (C.c_int, [_P, _P, C.c_int, C.c_int, C.c_int, _P]),
    "s4_weight_upload_glu": (C.c_int, [_P, _P, _P, C.c_int, C.c_int, C.c_uint32, C.POINTER(_P)]),
    "s4_weight_free": (C.c_int, [_P]),
    "s4_manifest_open": (C.c_int, [C.c_char_p, C.POINTER(_P)]),
    "s4_manifest_free": (C.c_int, [_P]),
    "s4_manifest_counts": (C.c_int, [_P, C.POINTER(C.c_int), C.POINTER(C.c_int)]),
    "s4_manifest_shard": (C.c_int, [_P, C.c_int, C.POINTER(C.c_char_p), C.POINTER(C.c_size_t)]),
    "s4_manifest_tensor": (C.c_int, [_P, C.c_char_p, C.POINTER(C.c_int), C.POINTER(C.c_size_t), C.POINTER(C.c_size_t),
                                     C.POINTER(C.c_int), C.POINTER(C.c_int)]),
    "s4_weight_upload_named": (C.c_int, [_P, _P, C.POINTER(_P), C.c_char_p, C.c_uint32, C.POINTER(_P)]),
    "s4_weight_save": (C.c_int, [_P, C.c_char_p]),
    "s4_weight_load": (C.c_int, [_P, C.c_char_p, C.POINTER(_P)]),
    "s4_weight_info": (C.c_int, [_P, C.POINTER(C.c_int), C.POINTER(C.c_int), C.POINTER(C.c_size_t)]),
    "s4_weight_layout_bytes": (C.c_int, [_P, C.POINTER(C.c_size_t), C.POINTER(C.c_size_t)]),
    "s4_weight_download_layout": (C.c_int, [_P, _P, C.c_size_t, _P, C.c_size_t]),
    "s4_matmul": (C.c_int, [_P, _P, _P, C.c_int, _P, _P]),
    "s4_matmul_host": (C.c_int, [_P, _P, _P, C.c_int, _P]),
    "s4_matmul_host_async": (C.c_int, [_P, _P, _P, C.c_int, _P, _P]),
    "s4_matmul_noalloc": (C.c_int, [_P, _P, C.c_int, _P, _P]),
    "s4_noalloc_check_errors": (C.c_int, [C.c_int, C.POINTER(C.c_uint32), C.c_int]),
    "s4_silu_mul": (C.c_int, [_P, _P, C.c_int, C.c_int, _P, _P]),
    "s4_add_rmsnorm": (C.c_int, [_P, _P, _P, _P, C.c_int, C.c_int, C.c_float, _P, _P]),
    "s4_matmul_add_rmsnorm": (C.c_int, [_P, _P, _P, C.c_int, _P, _P, C.c_float, _P, _P]),
    "s4_chain_create": (C.c_int, [_P, C.c_int, C.POINTER(_P), C.POINTER(_P), C.POINTER(_P), C.POINTER(C.c_int),
                                  C.POINTER(C.c_int), C.POINTER(_P)]),
    "s4_chain_run": (C.c_int, [_P, _P, _P]),
    "s4_chain_run_host": (C.c_int, [_P, _P, _P, _P, C.c_size_t, _P, _P, C.c_size_t, _P]),
    "s4_chain_info": (C.c_int, [_P, C.POINTER(C.c_int), C.POINTER(C.c_int), C.POINTER(C.c_int)]),
    "s4_chain_free": (C.c_int, [_P]),
    "s4_buffer_alloc": (C.c_int, [_P, C.c_size_t, C.POINTER(_P)]),
    "s4_buffer_free": (C.c_int, [_P, _P]),
    "s4_ipc_handle": (C.c_int, [_P, _P, _P]),
    "s4_ipc_open": (C.c_int, [_P, _P, C.POINTER(_P)]),
    "s4_ipc_close": (C.c_int, [_P, _P]),
    "s4_matmul_gather": (C.c_int, [_P, _P, _P, C.c_int, C.c_int, C.POINTER(_P), C.c_int, C.c_int, C.c_int, _P]),
    "s4_silu_mul_gather": (C.c_int, [_P, _P, C.c_int, C.c_int, C.POINTER(_P), C.c_int, C.c_int, C.c_int, _P]),
    "s4_peer_barrier": (C.c_int, [_P, C.POINTER(_P), C.c_int, C.c_int, C.c_uint32, _P]),
    "s4_peer_signal": (C.c_int, [_P, C.POINTER(_P), C.c_int, C.c_int, _P]),
    "s4_matmul_gather_wait": (C.c_int, [_P, _P, _P, C.c_int, C.c_int, C.POINTER(_P), C.c_int, C.c_int, C.c_int,
                                        _P, C.c_int, _P]),
    "s4_add_rmsnorm_wait": (C.c_int, [_P, _P, _P, _P, C.c_int, C.c_int, C.c_float, _P, _P, C.c_int, _P]),
    "s4_plan": (C.c_int, [_P, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_int), C.POINTER(C.c_int),
                          C.POINTER(C.c_int)]),
    "s4_force": (C.c_int, [_P, C.c_int, C.c_int, C.c_int]),
    "s4_set_table": (C.c_int, [_P, C.c_char_p]),
    "s4_check_errors": (C.c_int, [_P, C.POINTER(C.c_uint32)]),
    "s4_clear_errors": (C.c_int, [_P]),
    "s4_launch_count": (C.c_int, [_P, C.POINTER(C.c_uint64)]),
    "s4_device_info": (C.c_int, [_P, C.POINTER(C.c_int), C.POINTER(C.c_int)]),
}


class S4Error(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"s4mm error {code}: {msg}")
        self.code = code


_lib = None
_lib_lock = threading.Lock()


def load_library(path: str = LIB_PATH):
    """Load ``libs4mm.so`` and bind every declared entry point. Raises if it is missing."""
    global _lib
    with _lib_lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            raise S4Error(ERR_UNSUPPORTED, f"{path} is not built (run __graft_entry__.build())")
        lib = C.CDLL(path)
        for name, (res, args) in _SIGS.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def _check(rc: int):
    if rc != 0:
        raise S4Error(rc, _lib.s4_last_error().decode(errors="replace"))


def _ptr(a) -> int:
    """Device or host address of a torch tensor or numpy array."""
    if hasattr(a, "data_ptr"):
        return a.data_ptr()
    if isinstance(a, np.ndarray):
        return a.ctypes.data
    raise TypeError(f"expected a torch tensor or numpy array, got {type(a)}")


def _stream_handle(stream) -> int | None:
    if stream is None:
        try:
            import torch
            return torch.cuda.current_stream().cuda_stream
        except Exception:
            return None
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


class Chain:
    """A bound list of decode matmuls run by one persistent launch (``s4_chain_*``)."""

    def __init__(self, ctx: "Context", handle: int, ops):
        self.ctx, self.handle, self.ops = ctx, handle, ops

    def run(self, stream=None):
        _check(_lib.s4_chain_run(self.ctx.handle, self.handle, _stream_handle(stream)))

    def run_host(self, x_host, x_dev, y_host, y_dev, stream=None):
        """Host-buffer run: ``x_host`` (pinned CPU tensor) -> ``x_dev``, the chain, ``y_dev`` ->
        ``y_host``; asynchronous on ``stream``. ``x_dev``/``y_dev`` cover the bound buffers."""
        xb = x_host.numel() * x_host.element_size()
        yb = y_host.numel() * y_host.element_size()
        if x_dev.numel() * x_dev.element_size() < xb or y_dev.numel() * y_dev.element_size() < yb:
            raise S4Error(1, "run_host: device buffers smaller than the host buffers")
        _check(_lib.s4_chain_run_host(self.ctx.handle, self.handle, x_host.data_ptr(), x_dev.data_ptr(), xb,
                                      y_host.data_ptr(), y_dev.data_ptr(), yb, _stream_handle(stream)))

    def info(self):
        g, s, m = C.c_int(), C.c_int(), C.c_int()
        _check(_lib.s4_chain_info(self.handle, C.byref(g), C.byref(s), C.byref(m)))
        return {"grid": g.value, "slots": s.value, "smem_bytes": m.value}

    def free(self):
        if self.handle:
            _check(_lib.s4_chain_free(self.handle))
            self.handle = None

    def __del__(self):
        try:  # valid after the context closed too (the library frees chains without it)
            if self.handle and _lib is not None:
                _lib.s4_chain_free(self.handle)
        except Exception:
            pass


def _dev_f16(name: str, t, device: int, rows: int, cols: int):
    """Require a contiguous ``[>= rows, cols]`` CUDA fp16 tensor on the context's device. The
    kernels take raw pointers and sizes, so a wrong dtype, width, row count or device would be read
    or written out of bounds; the wrapper refuses it with ERR_INVALID instead."""
    import torch
    if not isinstance(t, torch.Tensor) or t.dtype != torch.float16 or not t.is_cuda:
        raise S4Error(ERR_INVALID, f"{name} must be a CUDA fp16 tensor")
    if t.device.index != device:
        raise S4Error(ERR_INVALID, f"{name} is on cuda:{t.device.index}, the context on cuda:{device}")
    if t.dim() != 2 or not t.is_contiguous() or t.shape[1] != cols or t.shape[0] < rows:
        raise S4Error(ERR_INVALID, f"{name} must be a contiguous [>= {rows}, {cols}] tensor, got "
                                   f"{tuple(t.shape)}{'' if t.is_contiguous() else ' (strided)'}")


def _dev_buf(name: str, t, device: int, nbytes: int, dtype=None):
    """Require a contiguous CUDA tensor on the context's device holding at least ``nbytes`` (of
    ``dtype`` when given): the upload kernels read that many bytes from its pointer."""
    import torch
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise S4Error(ERR_INVALID, f"{name} must be a CUDA tensor when the weight is uploaded from the device")
    if t.device.index != device:
        raise S4Error(ERR_INVALID, f"{name} is on cuda:{t.device.index}, the context on cuda:{device}")
    if dtype is not None and t.dtype != dtype:
        raise S4Error(ERR_INVALID, f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous() or t.numel() * t.element_size() < nbytes:
        raise S4Error(ERR_INVALID, f"{name} must be contiguous with at least {nbytes} bytes, got "
                                   f"{t.numel() * t.element_size()}{'' if t.is_contiguous() else ' (strided)'}")


class Manifest:
    """The weight manifest of an exported engine (``manifest.json`` of convert/export_engine.py:29-34,
    83-85), parsed by the library (``s4_manifest_open``); :meth:`tensor` is the engine's ``w(name)``
    (web/public/engine/engine.js:175-180). Needs no GPU."""

    def __init__(self, manifest):
        import json
        load_library()
        text = manifest if isinstance(manifest, (str, bytes)) else json.dumps(manifest)
        h = _P()
        _check(_lib.s4_manifest_open(text.encode() if isinstance(text, str) else text, C.byref(h)))
        self.handle = h.value

    @property
    def shards(self):
        """[(path, bytes)] in shard order."""
        ns, nt = C.c_int(), C.c_int()
        _check(_lib.s4_manifest_counts(self.handle, C.byref(ns), C.byref(nt)))
        out = []
        for i in range(ns.value):
            p, b = C.c_char_p(), C.c_size_t()
            _check(_lib.s4_manifest_shard(self.handle, i, C.byref(p), C.byref(b)))
            out.append((p.value.decode(), b.value))
        return out

    def tensor(self, name: str) -> dict:
        """``{shard, offset, bytes, N, K}`` of a tensor (offset inside its shard; N / K -1 unless it is a
        projection's ``.q``). Raises S4Error ``no tensor <name>`` when absent (engine.js:177)."""
        sh, off, nb, n, k = C.c_int(), C.c_size_t(), C.c_size_t(), C.c_int(), C.c_int()
        _check(_lib.s4_manifest_tensor(self.handle, name.encode(), C.byref(sh), C.byref(off), C.byref(nb), C.byref(n),
                                       C.byref(k)))
        return {"shard": sh.value, "offset": off.value, "bytes": nb.value, "N": n.value, "K": k.value}

    def close(self):
        if self.handle:
            _lib.s4_manifest_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Weight:
    """An uploaded, device-repacked int4 weight (the engine's resolved ``.q``/``.s`` pair)."""

    def __init__(self, ctx: "Context", handle: int, N: int, K: int):
        self.ctx, self.handle, self.N, self.K = ctx, handle, N, K

    @property
    def device_bytes(self) -> int:
        n, k, b = C.c_int(), C.c_int(), C.c_size_t()
        _check(_lib.s4_weight_info(self.handle, C.byref(n), C.byref(k), C.byref(b)))
        return b.value

    def save(self, path: str):
        """Write the repacked device layout to a cache file (``s4_weight_save``)."""
        _check(_lib.s4_weight_save(self.handle, os.fsencode(path)))

    def layout(self):
        """Download the device layout: ``(wq uint32, ws float16)`` flat arrays."""
        qb, sb = C.c_size_t(), C.c_size_t()
        _check(_lib.s4_weight_layout_bytes(self.handle, C.byref(qb), C.byref(sb)))
        wq = np.empty(qb.value // 4, np.uint32)
        ws = np.empty(sb.value // 2, np.float16)
        _check(_lib.s4_weight_download_layout(self.handle, wq.ctypes.data, qb.value, ws.ctypes.data, sb.value))
        return wq, ws

    def free(self):
        if self.handle:
            _check(_lib.s4_weight_free(self.handle))
            self.handle = None

    def __del__(self):
        try:  # valid after the context closed too (the library frees weights without it)
            if self.handle and _lib is not None:
                _lib.s4_weight_free(self.handle)
        except Exception:
            pass


class Context:
    """One library context on one CUDA device (the device side of ``Engine.create``)."""

    def __init__(self, device: int = 0):
        load_library()
        h = _P()
        _check(_lib.s4_init(int(device), C.byref(h)))
        self.handle = h.value
        self.device = int(device)
        self._weights = []

    # -- weights ---------------------------------------------------------------------------------
    def upload(self, packed, scales, N: int, K: int) -> Weight:
        """Upload MatMulNBits bytes (``packed`` uint8 [N][K/32][16], ``scales`` fp16 [N][K/32]).

        Host numpy arrays go through ``s4_weight_upload``; CUDA tensors through
        ``s4_weight_upload_device``. Synchronous."""
        h = _P()
        if hasattr(packed, "is_cuda") and packed.is_cuda:
            import torch
            _dev_buf("packed", packed, self.device, N * (K // 32) * 16, torch.uint8)
            _dev_buf("scales", scales, self.device, N * (K // 32) * 2, torch.float16)
            _check(_lib.s4_weight_upload_device(self.handle, packed.data_ptr(), scales.data_ptr(), N, K, 0,
                                                C.byref(h)))
        else:
            p = np.ascontiguousarray(np.asarray(packed, dtype=np.uint8))
            s = np.ascontiguousarray(np.asarray(scales, dtype=np.float16))
            if p.size != N * (K // 32) * 16 or s.size != N * (K // 32):
                raise S4Error(ERR_INVALID, f"packed/scales sizes do not match N={N} K={K}")
            _check(_lib.s4_weight_upload(self.handle, p.ctypes.data, s.ctypes.data, N, K, 0, C.byref(h)))
        return Weight(self, h.value, N, K)

    def upload_named(self, manifest: "Manifest", shards, name: str) -> Weight:
        """Upload projection ``name`` (``name.q`` / ``name.s`` of the manifest) from the engine's shard
        buffers (``s4_weight_upload_named``): ``shards`` lists every shard's bytes in manifest order, as
        host uint8 arrays or as CUDA uint8 tensors on this context's device (all on one side). Synchronous."""
        import torch
        expect = manifest.shards
        if len(shards) != len(expect):
            raise S4Error(ERR_INVALID, f"{len(shards)} shard buffers for a manifest of {len(expect)} shards")
        on_dev = [hasattr(b, "is_cuda") and b.is_cuda for b in shards]
        if any(on_dev) and not all(on_dev):
            raise S4Error(ERR_INVALID, "shard buffers must all be host arrays or all CUDA tensors")
        keep, ptrs = [], []
        for b, (path, nbytes) in zip(shards, expect):
            if on_dev[0]:
                _dev_buf(f"shard {path}", b, self.device, nbytes, torch.uint8)
                ptrs.append(b.data_ptr())
            else:
                a = np.ascontiguousarray(np.frombuffer(b, dtype=np.uint8) if isinstance(b, (bytes, bytearray))
                                         else np.asarray(b, dtype=np.uint8).reshape(-1))
                if a.size < nbytes:
                    raise S4Error(ERR_INVALID, f"shard {path}: {a.size} bytes, the manifest says {nbytes}")
                keep.append(a)
                ptrs.append(a.ctypes.data)
        arr = (_P * len(ptrs))(*[_P(p) for p in ptrs])
        h = _P()
        _check(_lib.s4_weight_upload_named(self.handle, manifest.handle, arr, name.encode(),
                                           UPLOAD_DEVICE if on_dev[0] else 0, C.byref(h)))
        t = manifest.tensor(name + ".q")
        return Weight(self, h.value, t["N"], t["K"])

    def upload_glu(self, packed, scales, I: int, K: int) -> Weight:
        """Upload a fused gate|up weight ([2I][K] MatMulNBits bytes, gate rows first) whose matmul
        writes silu(gate) * up, [M][I] (``s4_weight_upload_glu``). Host arrays or CUDA tensors."""
        h = _P()
        if hasattr(packed, "is_cuda") and packed.is_cuda:
            import torch
            _dev_buf("packed", packed, self.device, 2 * I * (K // 32) * 16, torch.uint8)
            _dev_buf("scales", scales, self.device, 2 * I * (K // 32) * 2, torch.float16)
            _check(_lib.s4_weight_upload_glu(self.handle, packed.data_ptr(), scales.data_ptr(), I, K, UPLOAD_DEVICE,
                                             C.byref(h)))
        else:
            p = np.ascontiguousarray(np.asarray(packed, dtype=np.uint8))
            s = np.ascontiguousarray(np.asarray(scales, dtype=np.float16))
            if p.size != 2 * I * (K // 32) * 16 or s.size != 2 * I * (K // 32):
                raise S4Error(ERR_INVALID, f"packed/scales sizes do not match 2I={2 * I} K={K}")
            _check(_lib.s4_weight_upload_glu(self.handle, p.ctypes.data, s.ctypes.data, I, K, 0, C.byref(h)))
        return Weight(self, h.value, I, K)

    def upload_wire(self, packed, wire, N: int, K: int) -> Weight:
        """Upload int4 bytes with download-format scales (``wire``: 4*N header bytes then N*(K/32)
        codes, as the export tooling writes them) through ``s4_weight_upload_wire``. Synchronous."""
        p = np.ascontiguousarray(np.asarray(packed, dtype=np.uint8))
        w = np.frombuffer(bytes(wire), dtype=np.uint8) if isinstance(wire, (bytes, bytearray)) else \
            np.ascontiguousarray(np.asarray(wire, dtype=np.uint8))
        G = K // 32
        if p.size != N * G * 16 or w.size != 4 * N + N * G:
            raise S4Error(ERR_INVALID, f"packed/wire sizes do not match N={N} K={K}")
        h = _P()
        _check(_lib.s4_weight_upload_wire(self.handle, p.ctypes.data, w.ctypes.data, N, K, 0, C.byref(h)))
        return Weight(self, h.value, N, K)

    def upload_format(self, q, scales, N: int, K: int, bits: int, group: int = 32, bias=None,
                      decode_layout: bool = False) -> Weight:
        """Upload a weight in one of the engine's formats (``{bits, group, asym}``): ``q`` u32
        [N][K/32][bits], ``scales`` fp16 [N][K/group], ``bias`` fp16 [N][K/group] or None. Host numpy
        arrays, or CUDA tensors (all on the device). Synchronous. ``decode_layout`` (symmetric 2-bit
        only): also keep the native 2-bit layout the decode GEMV streams (``S4_UPLOAD_DECODE_LAYOUT``)."""
        h = _P()
        extra = UPLOAD_DECODE_LAYOUT if decode_layout else 0
        if hasattr(q, "is_cuda") and q.is_cuda:
            import torch
            ng = N * (K // group) if group else 0
            _dev_buf("q", q, self.device, N * (K // 32) * bits * 4)
            _dev_buf("scales", scales, self.device, ng * 2, torch.float16)
            if bias is not None:
                _dev_buf("bias", bias, self.device, ng * 2, torch.float16)
            _check(_lib.s4_weight_upload_format(self.handle, q.data_ptr(), scales.data_ptr(),
                                                None if bias is None else bias.data_ptr(), N, K, bits, group,
                                                UPLOAD_DEVICE | extra, C.byref(h)))
        else:
            qa = np.ascontiguousarray(np.asarray(q, dtype=np.uint32))
            sa = np.ascontiguousarray(np.asarray(scales, dtype=np.float16))
            ba = None if bias is None else np.ascontiguousarray(np.asarray(bias, dtype=np.float16))
            if qa.size != N * (K // 32) * bits or sa.size != N * (K // group if group else 0) or \
                    (ba is not None and ba.size != sa.size):
                raise S4Error(ERR_INVALID, f"q/scales/bias sizes do not match N={N} K={K} bits={bits} group={group}")
            _check(_lib.s4_weight_upload_format(self.handle, qa.ctypes.data, sa.ctypes.data,
                                                None if ba is None else ba.ctypes.data, N, K, bits, group, extra,
                                                C.byref(h)))
        return Weight(self, h.value, N, K)

    def fwht(self, a, n: int, stream=None):
        """In-place orthonormal Walsh-Hadamard transform of every contiguous n-block of the CUDA fp16
        tensor ``a`` [M][K] (the engine's online rotation of ``had`` tensors). Returns ``a``."""
        M, K = (a.shape[0], a.shape[1]) if a.dim() == 2 else (1, a.numel())
        _check(_lib.s4_fwht(self.handle, a.data_ptr(), int(M), int(K), int(n), _stream_handle(stream)))
        return a

    def load_weight(self, path: str) -> Weight:
        """A weight from a cache file written by :meth:`Weight.save` (``s4_weight_load``); raises
        S4Error with code ERR_IO when the entry is missing, corrupt or of another layout version."""
        h = _P()
        _check(_lib.s4_weight_load(self.handle, os.fsencode(path), C.byref(h)))
        n, k = C.c_int(), C.c_int()
        _check(_lib.s4_weight_info(h.value, C.byref(n), C.byref(k), None))
        return Weight(self, h.value, n.value, k.value)

    def decode_wire_scales(self, wire_dev, N: int, G: int, out=None, stream=None):
        """Decode a device-resident wire scale tensor (uint8 CUDA tensor of 4*N + N*G bytes) to fp16
        ``[N, G]`` on the device (``decodeScales``), asynchronous on ``stream``."""
        import torch
        _dev_buf("wire", wire_dev, self.device, 4 * N + N * G)
        if out is None:
            out = torch.empty((N, G), dtype=torch.float16, device=wire_dev.device)
        _dev_buf("out", out, self.device, N * G * 2, torch.float16)
        _check(_lib.s4_decode_wire_scales(self.handle, wire_dev.data_ptr(), int(N), int(G), out.data_ptr(),
                                          _stream_handle(stream)))
        return out

    # -- compute ---------------------------------------------------------------------------------
    def matmul(self, x, W: Weight, M: int | None = None, y=None, stream=None):
        """``y[M][N] = x[M][K] @ W^T`` on CUDA fp16 tensors (the engine's matmul(A, wname, Y))."""
        import torch
        if M is None:
            M = x.shape[0]
        _dev_f16("x", x, self.device, M, W.K)
        if y is None:
            y = torch.empty((M, W.N), dtype=torch.float16, device=x.device)
        _dev_f16("y", y, self.device, M, W.N)
        _check(_lib.s4_matmul(self.handle, W.handle, x.data_ptr(), int(M), y.data_ptr(), _stream_handle(stream)))
        return y

    def matmul_host(self, x: np.ndarray, W: Weight, y: np.ndarray | None = None) -> np.ndarray:
        """Synchronous host-buffer matmul (``Gemm.setA`` + ``encode`` + ``readY``); fp16 arrays
        or their uint16 bit patterns."""
        x = np.ascontiguousarray(x)
        if x.dtype not in (np.float16, np.uint16) or x.ndim != 2 or x.shape[1] != W.K:
            raise S4Error(ERR_INVALID, f"x must be [M, {W.K}] fp16 (or its uint16 bits), got {x.dtype} {x.shape}")
        M = x.shape[0]
        if y is None:
            y = np.empty((M, W.N), dtype=np.float16)
        if (not isinstance(y, np.ndarray) or y.dtype not in (np.float16, np.uint16) or y.shape != (M, W.N)
                or not y.flags.c_contiguous or not y.flags.writeable):
            raise S4Error(ERR_INVALID, f"y must be a writable contiguous [{M}, {W.N}] fp16 array")
        _check(_lib.s4_matmul_host(self.handle, W.handle, x.ctypes.data, int(M), y.ctypes.data))
        return y

    def matmul_host_ptr(self, x_ptr: int, M: int, W: Weight, y_ptr: int):
        _check(_lib.s4_matmul_host(self.handle, W.handle, x_ptr, int(M), y_ptr))

    def matmul_host_async(self, x, W: Weight, y, M: int | None = None, stream=None):
        """Enqueue host->device copy, matmul and device->host copy on ``stream`` (pinned host
        tensors or arrays ``x`` [M][K] and ``y`` [M][N], fp16); returns without waiting."""
        if M is None:
            M = x.shape[0]
        _check(_lib.s4_matmul_host_async(self.handle, W.handle, _ptr(x), int(M), _ptr(y), _stream_handle(stream)))

    def silu_mul(self, big, I: int, mid=None, stream=None):
        """``mid = silu(big[:, :I]) * big[:, I:2I]`` on CUDA fp16 tensors."""
        import torch
        M = big.shape[0]
        _dev_f16("big", big, self.device, M, 2 * I)
        if mid is None:
            mid = torch.empty((M, I), dtype=torch.float16, device=big.device)
        _dev_f16("mid", mid, self.device, M, I)
        _check(_lib.s4_silu_mul(self.handle, big.data_ptr(), int(M), int(I), mid.data_ptr(), _stream_handle(stream)))
        return mid

    def add_rmsnorm(self, x, y=None, w=None, eps: float = 1e-6, h=None, stream=None, wait_flags=None,
                    nranks: int = 0):
        """``x += y`` (fp32 residual, in place; skipped when y is None), then
        ``h = f16(x * rsqrt(mean(x^2) + eps) * w)`` (w None = ones). Returns h. With ``wait_flags``
        (this rank's flag array) the kernel first waits for all ``nranks`` ranks' latest signal
        (``s4_add_rmsnorm_wait``)."""
        import torch
        M, D = x.shape
        if x.dtype != torch.float32 or not x.is_contiguous():
            raise S4Error(1, "add_rmsnorm: x must be a contiguous fp32 tensor")
        if y is not None and (y.dtype != torch.float16 or not y.is_contiguous() or tuple(y.shape) != (M, D)):
            raise S4Error(1, "add_rmsnorm: y must be a contiguous fp16 tensor shaped like x")
        if h is None:
            h = torch.empty((M, D), dtype=torch.float16, device=x.device)
        if wait_flags is not None:
            _check(_lib.s4_add_rmsnorm_wait(self.handle, x.data_ptr(), y.data_ptr() if y is not None else None,
                                            w.data_ptr() if w is not None else None, int(M), int(D), float(eps),
                                            h.data_ptr(), wait_flags, int(nranks), _stream_handle(stream)))
            return h
        _check(_lib.s4_add_rmsnorm(self.handle, x.data_ptr(), y.data_ptr() if y is not None else None,
                                   w.data_ptr() if w is not None else None, int(M), int(D), float(eps), h.data_ptr(),
                                   _stream_handle(stream)))
        return h

    def matmul_add_rmsnorm(self, x, W: Weight, resid, w=None, eps: float = 1e-6, h=None, stream=None):
        """A projection followed by ADD_NORM in one call: ``resid += f16(x @ W^T)`` (fp32, in
        place) and ``h = f16(resid * rsqrt(mean(resid^2) + eps) * w)`` (w None = ones); y itself is
        not stored. Returns h."""
        import torch
        M = x.shape[0]
        _dev_f16("x", x, self.device, M, W.K)
        if (resid.dtype != torch.float32 or not resid.is_contiguous() or tuple(resid.shape) != (M, W.N)
                or resid.device != torch.device("cuda", self.device)):
            raise S4Error(ERR_INVALID, f"matmul_add_rmsnorm: resid must be a contiguous [{M}, {W.N}] fp32 "
                                       f"tensor on cuda:{self.device}")
        if w is not None and (w.dtype != torch.float32 or not w.is_contiguous() or w.numel() != W.N):
            raise S4Error(ERR_INVALID, f"matmul_add_rmsnorm: w must be a contiguous fp32 tensor of {W.N} values")
        if h is None:
            h = torch.empty((M, W.N), dtype=torch.float16, device=x.device)
        _dev_f16("h", h, self.device, M, W.N)
        _check(_lib.s4_matmul_add_rmsnorm(self.handle, W.handle, x.data_ptr(), int(M), resid.data_ptr(),
                                          w.data_ptr() if w is not None else None, float(eps), h.data_ptr(),
                                          _stream_handle(stream)))
        return h

    # -- column-sharded prefill over peer memory --------------------------------------------------
    def buffer_alloc(self, nbytes: int) -> int:
        p = _P()
        _check(_lib.s4_buffer_alloc(self.handle, int(nbytes), C.byref(p)))
        return p.value

    def buffer_free(self, ptr: int):
        _check(_lib.s4_buffer_free(self.handle, ptr))

    def ipc_handle(self, ptr: int) -> bytes:
        h = C.create_string_buffer(64)
        _check(_lib.s4_ipc_handle(self.handle, ptr, h))
        return h.raw

    def ipc_open(self, handle: bytes) -> int:
        p = _P()
        hb = C.create_string_buffer(handle, 64)
        _check(_lib.s4_ipc_open(self.handle, hb, C.byref(p)))
        return p.value

    def ipc_close(self, ptr: int):
        _check(_lib.s4_ipc_close(self.handle, ptr))

    @staticmethod
    def _ptr_array(ptrs):
        return (_P * len(ptrs))(*[_P(int(p)) for p in ptrs])

    def matmul_gather(self, x_ptr: int, ldx: int, M: int, W: Weight, dst_ptrs, ldy: int, col0: int, stream=None,
                      wait_flags=None, nranks: int = 0):
        """``s4_matmul_gather``; with ``wait_flags`` (this rank's flag array) the activation loads first
        wait for all ``nranks`` ranks' latest signal (``s4_matmul_gather_wait``)."""
        arr = self._ptr_array(dst_ptrs)
        if wait_flags is not None:
            _check(_lib.s4_matmul_gather_wait(self.handle, W.handle, x_ptr, int(ldx), int(M), arr, len(dst_ptrs),
                                              int(ldy), int(col0), wait_flags, int(nranks), _stream_handle(stream)))
            return
        _check(_lib.s4_matmul_gather(self.handle, W.handle, x_ptr, int(ldx), int(M), arr, len(dst_ptrs), int(ldy),
                                     int(col0), _stream_handle(stream)))

    def silu_mul_gather(self, big, Is: int, dst_ptrs, ldd: int, col0: int, stream=None):
        arr = self._ptr_array(dst_ptrs)
        _check(_lib.s4_silu_mul_gather(self.handle, big.data_ptr(), int(big.shape[0]), int(Is), arr, len(dst_ptrs),
                                       int(ldd), int(col0), _stream_handle(stream)))

    def peer_signal(self, flag_ptrs, rank: int, stream=None):
        arr = self._ptr_array(flag_ptrs)
        _check(_lib.s4_peer_signal(self.handle, arr, len(flag_ptrs), int(rank), _stream_handle(stream)))

    def peer_barrier(self, flag_ptrs, rank: int, epoch: int, stream=None):
        arr = self._ptr_array(flag_ptrs)
        _check(_lib.s4_peer_barrier(self.handle, arr, len(flag_ptrs), int(rank), int(epoch) & 0xFFFFFFFF,
                                    _stream_handle(stream)))

    # -- chained decode GEMV ------------------------------------------------------------------------
    def chain(self, ops):
        """Bind a list of decode matmuls into one persistent launch (``s4_chain_create``).

        ``ops``: sequence of ``(x, W, y)`` or ``(x, W, y, dep)`` with CUDA fp16 tensors ``x [M, K]``
        and ``y [M, N]`` (1 <= M <= 16) and ``dep`` the index of an earlier op whose output ``x``
        is (or -1). The tensors are held by the returned :class:`Chain` so they stay alive."""
        n = len(ops)
        ws = (_P * n)(*[_P(o[1].handle) for o in ops])
        xs = (_P * n)(*[_P(o[0].data_ptr()) for o in ops])
        ys = (_P * n)(*[_P(o[2].data_ptr()) for o in ops])
        ms = (C.c_int * n)(*[int(o[0].shape[0]) for o in ops])
        deps = (C.c_int * n)(*[int(o[3]) if len(o) > 3 else -1 for o in ops])
        for i, o in enumerate(ops):
            if o[0].shape[0] != o[2].shape[0] or o[0].shape[1] != o[1].K or o[2].shape[1] != o[1].N:
                raise S4Error(1, "chain op shapes must be x [M, K], y [M, N] of its weight")
            _dev_f16(f"op {i} x", o[0], self.device, o[0].shape[0], o[1].K)
            _dev_f16(f"op {i} y", o[2], self.device, o[0].shape[0], o[1].N)
        h = _P()
        _check(_lib.s4_chain_create(self.handle, n, ws, xs, ys, ms, deps, C.byref(h)))
        return Chain(self, h.value, list(ops))

    # -- dispatcher ------------------------------------------------------------------------------
    def plan(self, M: int, N: int = 0, K: int = 0):
        f, t, s = C.c_int(), C.c_int(), C.c_int()
        _check(_lib.s4_plan(self.handle, int(M), int(N), int(K), C.byref(f), C.byref(t), C.byref(s)))
        return FAMILY_NAMES[f.value], t.value, s.value

    def force(self, family=FAMILY_AUTO, tile: int = 0, split: int = 0):
        if isinstance(family, str):
            family = {v: k for k, v in FAMILY_NAMES.items()}[family]
        _check(_lib.s4_force(self.handle, int(family), int(tile), int(split)))

    def set_table(self, table):
        """Load a dispatch table (dict or JSON text, the format of ``dispatch_table.json``); None
        restores the library's built-in table."""
        import json
        if table is None:
            _check(_lib.s4_set_table(self.handle, None))
            return
        text = table if isinstance(table, str) else json.dumps(table)
        _check(_lib.s4_set_table(self.handle, text.encode()))

    # -- diagnostics -----------------------------------------------------------------------------
    def check_errors(self) -> int:
        f = C.c_uint32()
        _check(_lib.s4_check_errors(self.handle, C.byref(f)))
        return f.value

    def clear_errors(self):
        _check(_lib.s4_clear_errors(self.handle))

    @property
    def launch_count(self) -> int:
        c = C.c_uint64()
        _check(_lib.s4_launch_count(self.handle, C.byref(c)))
        return c.value

    @property
    def sm_count(self) -> int:
        d, s = C.c_int(), C.c_int()
        _check(_lib.s4_device_info(self.handle, C.byref(d), C.byref(s)))
        return s.value

    def close(self):
        if self.handle:
            _check(_lib.s4_destroy(self.handle))
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()


class Gemm:
    """The reference's standalone GEMM object (web/public/gemmbench/kernels.js:83-104).

    ``Gemm(ctx, K=, N=, B=packed bytes, Sc=fp16 scale bits)`` uploads; ``setA(M, A16)`` stages
    fp16 activations (uint16 bit patterns, as ``Uint16Array``); ``encode()`` runs the matmul on
    the device; ``readY()`` returns the fp16 output bits (uint16, ``[M*N]``)."""

    def __init__(self, ctx: Context, K: int, N: int, B, Sc):
        import torch
        self.ctx, self.K, self.N = ctx, int(K), int(N)
        B = np.frombuffer(np.ascontiguousarray(B).tobytes(), np.uint8)
        Sc = np.frombuffer(np.ascontiguousarray(Sc).tobytes(), np.uint16).view(np.float16)
        self.W = ctx.upload(B, Sc, self.N, self.K)
        self._dev = torch.device("cuda", ctx.device)
        self.M = 0

    def setA(self, M: int, A16):
        import torch
        a = np.ascontiguousarray(np.asarray(A16).view(np.uint16)).reshape(M, self.K)
        self.M = int(M)
        self.A = torch.from_numpy(a.view(np.int16)).to(self._dev).view(torch.float16)
        self.Y = torch.empty((self.M, self.N), dtype=torch.float16, device=self._dev)

    def encode(self, stream=None):
        self.ctx.matmul(self.A, self.W, self.M, self.Y, stream)

    def readY(self) -> np.ndarray:
        import torch
        torch.cuda.synchronize(self._dev)
        return self.Y.view(torch.int16).cpu().numpy().view(np.uint16).reshape(-1)


# ------------------------------------------------------------------------------------------------
# On-disk weight cache keyed like the reference worker's asset cache (web/public/js/worker.js:27-44,
# 82-88, 100): entry names carry the prefix ``<rev>__<fnv(base + config + manifest)>__`` so new
# weights get fresh entries even at the same location, and entries under any other prefix are
# removed after a load. Entries hold the repacked device layout (``s4_weight_save``).
# ------------------------------------------------------------------------------------------------
def fnv1a32(text: str) -> str:
    """The worker's ``fnv`` (worker.js:31): FNV-1a 32, one step per code point on its first UTF-16
    unit (``for (const c of s) ... c.charCodeAt(0)``: the high surrogate of a non-BMP character), 8 hex
    digits."""
    h = 0x811C9DC5
    for ch in text:
        cp = ord(ch)
        unit = cp if cp < 0x10000 else 0xD800 + ((cp - 0x10000) >> 10)
        h = ((h ^ unit) * 0x01000193) & 0xFFFFFFFF
    return f"{h:08x}"


def cache_prefix(rev: str, base: str, config_text: str, manifest_text: str) -> str:
    """``cachePrefix`` of worker.js:100."""
    return f"{rev}__{fnv1a32(base + config_text + manifest_text)}__"


class WeightCache:
    """Repacked weights on disk under one fingerprint prefix."""

    SUFFIX = ".s4w"

    def __init__(self, directory: str, prefix: str):
        self.dir = directory
        self.prefix = prefix
        os.makedirs(directory, exist_ok=True)

    def path(self, name: str) -> str:
        return os.path.join(self.dir, self.prefix + name.replace("/", "_") + self.SUFFIX)

    def get(self, ctx: "Context", name: str, upload):
        """The cached weight ``name``, or ``upload()``'s result saved for the next load.
        Returns ``(weight, hit)``."""
        try:
            return ctx.load_weight(self.path(name)), True
        except S4Error as e:
            if e.code != ERR_IO:
                raise
        w = upload()
        w.save(self.path(name))
        return w, False

    def prune(self) -> int:
        """Remove entries under any other prefix (``pruneCache``, worker.js:82-88). Returns the count."""
        n = 0
        for f in os.listdir(self.dir):
            if f.endswith(self.SUFFIX) and not f.startswith(self.prefix):
                os.remove(os.path.join(self.dir, f))
                n += 1
        return n
