"""numpy restatement of the reference's int4 MatMulNBits path (TEST INFRASTRUCTURE ONLY).

Every function cites the reference file:line it restates. Conventions of the format
(convert/export_engine.py:3-4, web/public/gemmbench/kernels.js:1-3):

* weights ``W[N, K]`` are quantised in blocks of 32 consecutive K values of one output row;
* ``packed[N][K/32][16]`` bytes: element ``2i`` of a block in the low nibble of byte ``i``,
  element ``2i+1`` in the high nibble; nibble value ``q`` means ``q - 8`` (zero point 8);
* ``scales[N][K/32]`` fp16, one per block, any sign (``quant`` produces negative ones);
* ``Y[M, N] = X[M, K] @ dequant(W).T`` computed in fp32 and rounded once to fp16.

The product never imports this module; tests compare the CUDA path against it.
"""
from __future__ import annotations

import hashlib

import numpy as np

BLOCK = 32


# --------------------------------------------------------------------------------------------
# quantiser / packer  (convert/export_engine.py:17-26)
# --------------------------------------------------------------------------------------------
def quant(W: np.ndarray):
    """Symmetric round-to-nearest int4 quantiser, restating ``quant`` (export_engine.py:17-26).

    Per block of 32: the element of largest magnitude (first one on ties, as torch.argmax) is
    divided by -8 to give the scale (so that element maps to nibble 0); a zero scale becomes 1;
    the scale is rounded to fp16 and that rounded value is used for ``q = clamp(round(w/s)+8)``
    (round half to even, as torch.round). Returns ``(packed u8 [N,K/32,16], scales f16 [N,K/32],
    deq f32 [N,K])``.
    """
    W = np.asarray(W, dtype=np.float32)
    N, K = W.shape
    assert K % BLOCK == 0
    b = W.reshape(N, K // BLOCK, BLOCK)
    idx = np.abs(b).argmax(-1)[..., None]                                   # :20
    scale = np.take_along_axis(b, idx, -1) / np.float32(-8.0)               # :21
    scale = np.where(scale == 0, np.float32(1.0), scale)                    # :22
    scale = scale.astype(np.float16).astype(np.float32)                     # :22
    q = np.clip(np.round(b / scale) + 8, 0, 15).astype(np.uint8)            # :23
    packed = pack_nibbles(q)                                                # :24
    deq = ((q.astype(np.float32) - 8) * scale).reshape(N, K)                # :25
    return packed, scale[..., 0].astype(np.float16), deq


def pack_nibbles(q: np.ndarray) -> np.ndarray:
    """``q[N,B,32]`` nibble values -> ``packed[N,B,16]`` (export_engine.py:24, make_gemm.py:9)."""
    q = np.asarray(q, dtype=np.uint8)
    return np.ascontiguousarray(q[..., 0::2] | (q[..., 1::2] << 4)).astype(np.uint8)


def unpack_nibbles(packed: np.ndarray) -> np.ndarray:
    """Inverse of :func:`pack_nibbles`: element ``e`` of a block is nibble ``e % 2`` of byte
    ``e // 2`` (kernels.js:2-3, ``decodeBlock`` kernels.js:23-38)."""
    p = np.asarray(packed, dtype=np.uint8)
    q = np.empty(p.shape[:-1] + (p.shape[-1] * 2,), dtype=np.uint8)
    q[..., 0::2] = p & 15
    q[..., 1::2] = p >> 4
    return q


def dequant(packed: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """fp32 ``(q - 8) * scale`` (export_engine.py:25; the per-element formula of kernels.js:35
    and of the CPU checks in gemmbench/bench.js:49 and portable.js:62)."""
    q = unpack_nibbles(packed).astype(np.float32) - 8.0
    s = np.asarray(scales).astype(np.float32)[..., None]
    N, B, _ = q.shape
    return (q * s).reshape(N, B * BLOCK)


def dequant_torch(packed, scales):
    """``dequant`` in torch (CPU tensors in, fp32 ``[N, K]`` out), for timing the dequantise-per-call
    variant of the CPU baseline: the reference's own quantiser is torch code (export_engine.py:17-26),
    byte i of a block holding elements 2i (low nibble) and 2i + 1 (high nibble)."""
    import torch
    p = torch.as_tensor(packed)
    N, B, _ = p.shape
    q = torch.stack((p & 0xF, p >> 4), dim=-1).reshape(N, B, BLOCK).to(torch.float32) - 8.0
    s = torch.as_tensor(scales).to(torch.float32).unsqueeze(-1)
    return (q * s).reshape(N, B * BLOCK)


def matmul(x: np.ndarray, packed: np.ndarray, scales: np.ndarray, deq: np.ndarray | None = None):
    """The reference CPU path: fp32 dequantise-then-matmul, one fp16 rounding at the end.

    Restates the fake-quant fp32 route (export_engine.py:88-103: dequantised weights copied into
    an fp32 model, so each projection is ``x.float() @ deq.T``) and the fp32 dot of the GEMM
    benches (bench.js:49). Returns ``(y f16 [M,N], y32 f32 [M,N])``.
    """
    if deq is None:
        deq = dequant(packed, scales)
    y32 = np.asarray(x, dtype=np.float16).astype(np.float32) @ deq.T
    return y32.astype(np.float16), y32


def cpu_check_columns(x16: np.ndarray, packed: np.ndarray, scales: np.ndarray, cols, rows=None):
    """Element-wise fp32 dot products on a few output columns, restating the spot check of
    gemmbench/bench.js:47-52 (all rows, columns {0, 1, N/2, N-1}) and portable.js:59-66
    (rows {0, M/2, M-1}). Returns a dict ``{(m, n): fp32 value}``."""
    M = x16.shape[0]
    rows = range(M) if rows is None else rows
    xf = x16.astype(np.float32)
    out = {}
    for n in cols:
        w = dequant(packed[n:n + 1], scales[n:n + 1])[0]
        for m in rows:
            out[(m, n)] = float(np.dot(xf[m].astype(np.float64), w.astype(np.float64)))
    return out


# --------------------------------------------------------------------------------------------
# metrics  (chain.js:12, bench.js:50-51)
# --------------------------------------------------------------------------------------------
def max_rel(y, ref) -> float:
    """max |y - ref| / max |ref| over all elements (chain.js:12, bench.js:50-51)."""
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    mag = np.abs(ref).max()
    return float(np.abs(y - ref).max() / mag) if mag > 0 else float(np.abs(y - ref).max())


def min_row_cosine(y, ref) -> float:
    """Smallest per-row cosine similarity between ``y`` and ``ref`` (rows = tokens)."""
    y = np.asarray(y, dtype=np.float64).reshape(ref.shape[0], -1)
    r = np.asarray(ref, dtype=np.float64).reshape(ref.shape[0], -1)
    num = (y * r).sum(1)
    den = np.sqrt((y * y).sum(1) * (r * r).sum(1))
    cos = np.where(den > 0, num / np.where(den > 0, den, 1), 1.0)
    return float(cos.min())


TOL_MAX_REL = 2e-3       # max relative error
TOL_MIN_COSINE = 0.99999  # per-row cosine


def check(y, ref, tol=TOL_MAX_REL, cos=TOL_MIN_COSINE):
    """(ok, max_rel, min_row_cosine) under the north-star tolerance."""
    mr = max_rel(y, ref)
    mc = min_row_cosine(y, ref)
    return (mr <= tol and mc >= cos), mr, mc


# --------------------------------------------------------------------------------------------
# synthetic inputs  (convert/make_gemm.py:4-10, convert/make_chain.py:22-29)
# --------------------------------------------------------------------------------------------
MAKE_GEMM_SHAPES = [(2048, 6144), (2048, 2048), (6144, 2048), (2048, 12288)]   # make_gemm.py:5


def make_gemm_weights(rng, K: int, N: int):
    """One shape of the GEMM bench generator (make_gemm.py:7-10): uniform nibbles, signed scales
    N(0,1)*0.02 in fp16. Draw order matters: nibbles first, then scales."""
    blocks = K // BLOCK
    q = rng.integers(0, 16, size=(N, blocks, 32), dtype=np.uint8)
    packed = pack_nibbles(q)
    scales = (rng.standard_normal((N, blocks)) * 0.02).astype(np.float16)
    return packed, scales


def make_chain_weights(rng, K: int, N: int):
    """One layer of the chain generator (make_chain.py:27-29): scales N(0,1)/(sqrt(K)*4.6)."""
    q = rng.integers(0, 16, size=(N, K // BLOCK, 32), dtype=np.uint8)
    packed = pack_nibbles(q)
    scales = (rng.standard_normal((N, K // BLOCK)) * (1.0 / (np.sqrt(K) * 4.6))).astype(np.float16)
    return packed, scales


def config_weights(rng, K: int, N: int):
    """Weights of the BASELINE configs: nibbles uniform (q-8 uniform in [-8,7]), fp16 scales
    |N(0, 0.02)| / 7. Nibbles are drawn before scales, as in make_gemm.py:8-10."""
    q = rng.integers(0, 16, size=(N, K // BLOCK, 32), dtype=np.uint8)
    packed = pack_nibbles(q)
    scales = (np.abs(rng.standard_normal((N, K // BLOCK)) * 0.02) / 7.0).astype(np.float16)
    return packed, scales


def config_x(rng, M: int, K: int):
    """Activations of the BASELINE configs: fp16 N(0, 1)."""
    return rng.standard_normal((M, K)).astype(np.float16)


def sha256(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


# --------------------------------------------------------------------------------------------
# SiLU * mul  (web/public/engine/wgsl.js:81-90)
# --------------------------------------------------------------------------------------------
def silu_mul(big: np.ndarray, I: int) -> np.ndarray:
    """``mid[t, j] = silu(g) * u`` with ``big[t] = [g (I) | u (I)]``; f32 math, f16 out
    (wgsl.js:81-90)."""
    b = np.asarray(big, dtype=np.float16).astype(np.float32)
    g, u = b[:, :I], b[:, I:2 * I]
    return (g / (1.0 + np.exp(-g)) * u).astype(np.float16)


# --------------------------------------------------------------------------------------------
# residual add + RMSNorm  (web/public/engine/wgsl.js:55-78)
# --------------------------------------------------------------------------------------------
def add_rmsnorm(x: np.ndarray, y=None, w=None, eps: float = 1e-6):
    """ADD_NORM: fp32 residual ``x += y`` (y fp16, optional), then ``h = f16(x * (mean(x^2) + eps)^-1/2
    * w)`` per row (wgsl.js:55-78; ``w`` is the stored 1 + weight). Returns (x_new f32, h f16)."""
    x = np.asarray(x, dtype=np.float32)
    if y is not None:
        x = x + np.asarray(y, dtype=np.float16).astype(np.float32)
    inv = 1.0 / np.sqrt((x.astype(np.float64) ** 2).mean(1, keepdims=True) + eps)
    h = x * inv.astype(np.float32)
    if w is not None:
        h = h * np.asarray(w, dtype=np.float32)
    return x, h.astype(np.float16)


# --------------------------------------------------------------------------------------------
# non-default weight formats (web/public/gemmbench/kernels.js:5-12, 23-38) and FWHT (wgsl.js:94-110)
# --------------------------------------------------------------------------------------------
def pack_format(q: np.ndarray, bits: int) -> np.ndarray:
    """q [N][K] in [0, 2^bits) -> u32 [N][K/32][bits] in the layout kernels.js:5-9 documents: 4 bits:
    element e at bits 4(e%8) of word e/8; 2 bits: element e at bits 2(e%16) of word e/16; 3 bits:
    the low two bits as in the 2-bit layout in words 0-1, bit e of word 2 the high bit. (The
    exporter that writes these is not part of the reference checkout; this packs test data.)"""
    N, K = q.shape
    qb = q.reshape(N, K // BLOCK, BLOCK).astype(np.uint64)
    e = np.arange(BLOCK, dtype=np.uint64)
    if bits == 4:
        words = [(qb[..., 8 * w:8 * w + 8] << (4 * e[:8])).sum(-1) for w in range(4)]
    else:
        lo = qb & 3
        words = [(lo[..., 16 * w:16 * w + 16] << (2 * e[:16])).sum(-1) for w in range(2)]
        if bits == 3:
            words.append(((qb >> 2) << e).sum(-1))
    return np.stack(words, -1).astype(np.uint32)


def unpack_format(words: np.ndarray, bits: int) -> np.ndarray:
    """u32 [N][B][bits] -> q [N][B*32] (decodeBlock's extraction, kernels.js:31-34)."""
    w = words.astype(np.uint64)
    e = np.arange(BLOCK, dtype=np.uint64)
    if bits == 4:
        q = (w[..., e // 8] >> (4 * (e % 8))) & 15
    else:
        q = (w[..., e // 16] >> (2 * (e % 16))) & 3
        if bits == 3:
            q |= ((w[..., 2:3] >> e) & 1) << 2
    N, B = words.shape[:2]
    return q.reshape(N, B * BLOCK).astype(np.int64)


def dequant_format(words: np.ndarray, scales: np.ndarray, bits: int, group: int, bias=None) -> np.ndarray:
    """fp32 weights [N][K] as decodeBlock computes them in f32 (kernels.js:28-36): one scale (and
    bias) per `group` values; symmetric ``(q - 2^(bits-1)) * sc``, asymmetric ``fma(q, sc, bi)``
    (one rounding: the float64 sum is exact here, then rounded to float32)."""
    q = unpack_format(words, bits)
    N, K = q.shape
    s = np.repeat(np.asarray(scales, dtype=np.float16).astype(np.float64).reshape(N, K // group), group, 1)
    if bias is None:
        return ((q - 2 ** (bits - 1)) * s).astype(np.float32)
    b = np.repeat(np.asarray(bias, dtype=np.float16).astype(np.float64).reshape(N, K // group), group, 1)
    return (q * s + b).astype(np.float32)


def transcode_sym(words: np.ndarray, scales: np.ndarray, bits: int, group: int):
    """A symmetric 2/3/4-bit, group-32/64 weight as MatMulNBits int4 bytes with [N][K/32] fp16 scales
    holding exactly the same weights: q4 = q - 2^(bits-1) + 8, each group scale repeated over its
    32-blocks. Returns ``(packed [N][K/32][16] u8, scales [N][K/32] f16)``."""
    q = unpack_format(words, bits) - 2 ** (bits - 1) + 8
    N, K = q.shape
    packed = pack_nibbles(q.reshape(N, K // BLOCK, BLOCK).astype(np.uint8))
    s = np.repeat(np.asarray(scales, dtype=np.float16).reshape(N, K // group), group // BLOCK, 1)
    return packed, s


def fwht(a: np.ndarray, n: int) -> np.ndarray:
    """In-place orthonormal Walsh-Hadamard transform of each contiguous n-block (wgsl.js:94-110):
    fp32 butterflies (x + y, x - y) over pairs (i, i + h) for h = 1, 2, 4, ... < n, then times
    f32(1/sqrt(n)) and rounded to fp16. Returns the transformed fp16 copy of ``a``."""
    sh = np.asarray(a, dtype=np.float16).astype(np.float32).reshape(-1, n).copy()
    h = 1
    while h < n:
        v = sh.reshape(sh.shape[0], n // (2 * h), 2, h)
        x, y = v[:, :, 0, :].copy(), v[:, :, 1, :].copy()
        v[:, :, 0, :] = x + y
        v[:, :, 1, :] = x - y
        h *= 2
    c = np.float32(1.0 / np.sqrt(float(n)))
    return (sh * c).astype(np.float16).reshape(np.shape(a))


# --------------------------------------------------------------------------------------------
# wire-format scale codec (web/public/engine/wire.js:1-33)
# --------------------------------------------------------------------------------------------
# 2^(-r/4096) for r in [0, 4096), correctly rounded: libm pow is exact to the last bit on all 4096 (a
# test checks them against 60-digit decimal values). 2^(-i/4096) = 2^-(i >> 12) * table[i & 4095], the
# power-of-two factor exact wherever the decoded scale is not flushed to zero anyway.
WIRE_POW = np.array([2.0 ** (-r / 4096) for r in range(4096)], dtype=np.float64)


def wire_from_half(h: np.ndarray) -> np.ndarray:
    """fromHalf (wire.js:5): fp16 bits -> float64, exponent 31 read as a finite power (no inf/NaN)."""
    h = h.astype(np.int64)
    e, f = (h >> 10) & 31, h & 1023
    v = np.where(e > 0, np.ldexp((1024 + f).astype(np.float64), (e - 25).astype(np.int32)),
                 np.ldexp(f.astype(np.float64), -24))
    return np.where(h & 0x8000, -v, v)


def wire_to_half(x: np.ndarray) -> np.ndarray:
    """toHalf (wire.js:8-15) bit for bit: float64 -> float32 (nearest even) -> fp16 bits by the JS
    integer steps (magnitude exponent rebased by 112, 13 dropped bits rounded half to even, overflow
    to 0x7c00, subnormals by floor arithmetic in units of 2^-24), stored mod 2^16 as the Uint16Array
    it lands in does."""
    f32 = np.asarray(x, dtype=np.float64).astype(np.float32)
    b = f32.view(np.uint32).astype(np.int64)
    e, rest = ((b >> 23) & 255) - 112, b & 0x1FFF
    h = (e << 10) | ((b >> 13) & 1023)
    normal = h + ((rest > 0x1000) | ((rest == 0x1000) & ((h & 1) == 1)))
    u = f32.astype(np.float64) * 2.0 ** 24
    fl = np.floor(u)
    d = u - fl
    fi = fl.astype(np.int64)
    sub = fi + ((d > 0.5) | ((d == 0.5) & ((fi & 1) == 1)))
    out = np.where((e > 0) & (e < 31), normal, np.where(e >= 31, 0x7C00, sub))
    return (out & 0xFFFF).astype(np.uint16)


def decode_wire_scales(wire: bytes | np.ndarray, N: int, G: int) -> np.ndarray:
    """8-bit log-coded scales -> fp16, restating ``decodeScales`` (wire.js:19-33).

    Layout (wire.js:1-3, 20-22): N row headers of 4 bytes (``m`` = fp16 bits of the row's largest
    magnitude, ``j`` = u16 step, both little-endian), then N*G codes ``sign << 7 | k``. A code
    decodes to ``toHalf(fromHalf(m) * 2^(-k*j/4096)) | sign << 15`` (the product in float64).
    Returns fp16 ``[N, G]``."""
    b = np.frombuffer(bytes(wire), dtype=np.uint8) if not isinstance(wire, np.ndarray) else wire.view(np.uint8).ravel()
    hdr = b[:4 * N].reshape(N, 4).astype(np.int64)
    codes = b[4 * N:4 * N + N * G].reshape(N, G).astype(np.int64)
    m = wire_from_half(hdr[:, 0] | hdr[:, 1] << 8)[:, None]
    j = (hdr[:, 2] | hdr[:, 3] << 8)[:, None]
    i = (codes & 127) * j
    p = np.ldexp(WIRE_POW[i & 4095], -(i >> 12).astype(np.int32))
    bits = wire_to_half(m * p) | ((codes & 128) << 8).astype(np.uint16)
    return bits.view(np.float16)


def encode_wire_scales(scales: np.ndarray) -> bytes:
    """A simple encoder for test data (the reference's pack_wire.py is not part of the checkout): per
    row m = largest |scale|, j spans the row's dynamic range over codes 0..127, k = nearest code."""
    s = np.asarray(scales, dtype=np.float16)
    N, G = s.shape
    a = np.abs(s.astype(np.float64))
    mx = a.max(1)
    m16 = np.where(mx > 0, mx, 1.0).astype(np.float16)
    mf = m16.astype(np.float64)
    nz = np.where(a > 0, a, np.inf).min(1)
    span = np.where(np.isfinite(nz) & (nz < mf), np.log2(mf / np.minimum(nz, mf)), 0.0)
    j = np.clip(np.ceil(span * 4096.0 / 127.0), 1, 65535).astype(np.uint16)
    with np.errstate(divide="ignore"):
        e = np.where(a > 0, -np.log2(a / mf[:, None]), np.inf)
    k = np.clip(np.rint(e * 4096.0 / j[:, None].astype(np.float64)), 0, 127).astype(np.uint8)
    codes = k | ((s.view(np.uint16) >> 8).astype(np.uint8) & 128)
    hdr = np.stack([m16.view(np.uint16), j], 1).astype(np.uint16)
    return hdr.tobytes() + codes.tobytes()


# --------------------------------------------------------------------------------------------
# device layout (the layout the upload kernel writes; checked bit-exactly against the GPU)
# --------------------------------------------------------------------------------------------
NB_ROWS = 128   # output rows (N) per n-block
KT_COLS = 64    # K per k-tile (two quant blocks)


def tiled_dims(N: int, K: int):
    nblk = (N + NB_ROWS - 1) // NB_ROWS
    kt = (K + KT_COLS - 1) // KT_COLS
    return nblk, kt


def _shuffle_word(w: np.ndarray) -> np.ndarray:
    """MatMulNBits u32 (nibble i = k_i, i=0..7) -> device u32: k0,k2,k4,k6 in nibbles 0-3 and
    k1,k3,k5,k7 in nibbles 4-7, so the magic-number fp16 conversion yields the pairs
    (k0,k1), (k2,k3), (k4,k5), (k6,k7)."""
    w = w.astype(np.uint32)
    out = np.zeros_like(w)
    for i in range(8):
        nib = (w >> np.uint32(4 * i)) & np.uint32(15)
        pos = (i // 2) if i % 2 == 0 else 4 + i // 2
        out |= nib << np.uint32(4 * pos)
    return out


def repack_device(packed: np.ndarray, scales: np.ndarray, N: int, K: int):
    """The B200 layout of one weight (what ``s4_weight_upload`` writes on the device).

    ``wq`` u32 ``[NBLK][KT][8 sub][32 lanes][4 words]``: sub-tile ``sub`` holds rows
    ``r0 = nb*128 + sub*16``; lane ``L = 4g + t`` word ``j = 2*blk + h`` holds the 8 values of row
    ``r0 + g + 8h`` at ``k = kt*64 + blk*32 + 8t .. +8``, shuffled by :func:`_shuffle_word`.
    ``ws`` f16 ``[NBLK][KT][8 sub][8 g][4]`` = scales of (row g, blk0), (row g+8, blk0),
    (row g, blk1), (row g+8, blk1). Rows >= N and K >= K are padded with nibble 8 and scale 0.
    """
    nblk, kt = tiled_dims(N, K)
    Np, Kp = nblk * NB_ROWS, kt * KT_COLS
    B = K // BLOCK
    q = np.full((Np, Kp // 2), 0x88, dtype=np.uint8)
    q[:N, :K // 2] = packed.reshape(N, B * 16)
    sc = np.zeros((Np, Kp // BLOCK), dtype=np.float16)
    sc[:N, :B] = scales
    words = q.view("<u4").reshape(Np, Kp // 8)           # word c of row r covers k 8c..8c+7
    words = _shuffle_word(words)
    # [nb, sub, h, g, kt, blk, t]
    w7 = words.reshape(nblk, 8, 2, 8, kt, 2, 4)
    wq = w7.transpose(0, 4, 1, 3, 6, 5, 2).reshape(nblk, kt, 8, 32, 4)   # lane = (g, t); word = (blk, h)
    s6 = sc.reshape(nblk, 8, 2, 8, kt, 2)                 # [nb, sub, h, g, kt, blk]
    ws = s6.transpose(0, 4, 1, 3, 5, 2).reshape(nblk, kt, 8, 8, 4)
    return np.ascontiguousarray(wq.astype(np.uint32)), np.ascontiguousarray(ws)


def unrepack_device(wq: np.ndarray, ws: np.ndarray, N: int, K: int):
    """Inverse of :func:`repack_device` (used by the round-trip tests)."""
    nblk, kt = tiled_dims(N, K)
    Np, Kp = nblk * NB_ROWS, kt * KT_COLS
    w7 = wq.reshape(nblk, kt, 8, 8, 4, 2, 2).transpose(0, 2, 6, 3, 1, 5, 4)  # -> nb, sub, h, g, kt, blk, t
    words = w7.reshape(Np, Kp // 8).astype(np.uint32)
    orig = np.zeros_like(words)
    for i in range(8):
        pos = (i // 2) if i % 2 == 0 else 4 + i // 2
        orig |= ((words >> np.uint32(4 * pos)) & np.uint32(15)) << np.uint32(4 * i)
    q = orig.astype("<u4").view(np.uint8).reshape(Np, Kp // 2)
    packed = q[:N, :K // 2].reshape(N, K // BLOCK, 16)
    s6 = ws.reshape(nblk, kt, 8, 8, 2, 2).transpose(0, 2, 5, 3, 1, 4)     # -> nb, sub, h, g, kt, blk
    sc = s6.reshape(Np, Kp // BLOCK)[:N, :K // BLOCK]
    return np.ascontiguousarray(packed), np.ascontiguousarray(sc)


# --------------------------------------------------------------------------------------------
# exported engine layout  (convert/export_engine.py:29-43, 70-85)
# --------------------------------------------------------------------------------------------
def export_engine(tensors, shard_limit: int = 512 << 20, config=None):
    """Restates the exporter's tensor index and shard split: tensors are appended in order to one byte
    sequence, each at the next 256-byte aligned offset (``add``, :29-34; the padding is its own piece);
    a quantised projection ``p`` becomes ``p.q`` (with ``N`` padded to a multiple of 64 by zero rows and
    ``K``) then ``p.s`` (``add_q``, :36-43); the pieces are cut into shards, a new shard starting at the
    piece that would push the current one past ``shard_limit`` (:70-78). ``tensors`` lists
    ``(name, array)`` for plain tensors and ``(name, "q", W f32 [N, K])`` for projections. Returns
    ``(manifest dict, [shard bytes], {name: (packed, scales)})``."""
    pieces, index, quantised = [], {}, {}
    offset = 0

    def add(name, arr, **meta):
        nonlocal offset
        arr = np.ascontiguousarray(arr)
        pad = (-offset) % 256
        if pad:
            pieces.append(b"\0" * pad)
            offset += pad
        index[name] = {"offset": offset, "bytes": arr.nbytes, "dtype": str(arr.dtype), "shape": list(arr.shape), **meta}
        pieces.append(arr.tobytes())
        offset += arr.nbytes

    for t in tensors:
        if len(t) == 3 and isinstance(t[1], str) and t[1] == "q":
            name, _, W = t
            N = W.shape[0]
            Np = (N + 63) // 64 * 64
            if Np != N:
                W = np.concatenate([W, np.zeros((Np - N, W.shape[1]), np.float32)])
            pk, sc, _ = quant(W)
            add(name + ".q", pk, N=Np, K=W.shape[1])
            add(name + ".s", sc)
            quantised[name] = (pk, sc)
        else:
            add(*t)
    shards, cur, cur_start, pos = [], [], 0, 0
    for b in pieces:
        if cur and pos + len(b) - cur_start > shard_limit:
            shards.append((cur_start, cur))
            cur, cur_start = [], pos
        cur.append(b)
        pos += len(b)
    shards.append((cur_start, cur))
    manifest = {"config": config or {},
                "shards": [{"path": f"weights.{n}.bin", "start": s, "bytes": sum(len(b) for b in bs)}
                           for n, (s, bs) in enumerate(shards)],
                "tensors": index}
    return manifest, [b"".join(bs) for _, bs in shards], quantised


def resolve_tensor(manifest: dict, name: str):
    """The engine's ``w(name)`` (web/public/engine/engine.js:175-180): the shard whose
    [start, start + bytes) holds the tensor's offset, and the offset inside it."""
    t = manifest["tensors"][name]
    for i, s in enumerate(manifest["shards"]):
        if s["start"] <= t["offset"] < s["start"] + s["bytes"]:
            return i, t["offset"] - s["start"]
    raise KeyError(name)
