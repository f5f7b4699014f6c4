"""The CPU oracle against the reference's own outputs (golden fixtures) and its own invariants."""
import json
import os

import numpy as np
import pytest

from oracle import s4ref

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _cases(fname):
    z = np.load(os.path.join(GOLDEN, fname))
    names = sorted({k.split("/")[0] for k in z.files})
    return z, names


QZ, QNAMES = _cases("quant_cases.npz")
MZ, MNAMES = _cases("matmul_cases.npz")


@pytest.mark.parametrize("name", QNAMES)
def test_quant_matches_reference_bit_exact(name):
    packed, scales, deq = s4ref.quant(QZ[f"{name}/W"])
    assert packed.dtype == np.uint8 and scales.dtype == np.float16
    np.testing.assert_array_equal(packed, QZ[f"{name}/packed"])
    np.testing.assert_array_equal(scales.view(np.uint16), QZ[f"{name}/scales"].view(np.uint16))
    np.testing.assert_array_equal(deq.view(np.uint32), QZ[f"{name}/deq"].view(np.uint32))


def test_quant_edge_rules():
    W = QZ["edges_8x64/W"]
    packed, scales, _ = s4ref.quant(W)
    assert scales[0, 0] == 1.0                        # zero block -> scale 1
    assert scales[1, 1] < 0 and scales[2, 1] > 0      # sign follows -max/8
    q = s4ref.unpack_nibbles(packed)
    # the element of largest magnitude always maps to nibble 0
    for r in range(1, 8):
        for b in range(2):
            blk = W[r, 32 * b:32 * b + 32]
            if np.abs(blk).max() > 0:
                assert q[r, b, np.abs(blk).argmax()] == 0


@pytest.mark.parametrize("name", QNAMES)
def test_dequant_of_packed_equals_reference_deq(name):
    deq = s4ref.dequant(QZ[f"{name}/packed"], QZ[f"{name}/scales"])
    np.testing.assert_array_equal(deq, QZ[f"{name}/deq"])


@pytest.mark.parametrize("name", QNAMES)
def test_torch_dequant_equals_reference_deq(name):
    """The torch restatement timed by the dequantise-per-call CPU baseline gives the reference's deq."""
    deq = s4ref.dequant_torch(QZ[f"{name}/packed"], QZ[f"{name}/scales"]).numpy()
    np.testing.assert_array_equal(deq, QZ[f"{name}/deq"])


@pytest.mark.parametrize("name", MNAMES)
def test_matmul_matches_reference_fake_quant(name):
    x = MZ[f"{name}/x"]
    y16, y32 = s4ref.matmul(x, MZ[f"{name}/packed"], MZ[f"{name}/scales"])
    ref = MZ[f"{name}/y32"]
    # same fp32 math, different summation order: fp32-level agreement
    assert s4ref.max_rel(y32, ref) < 1e-5
    ok, mr, mc = s4ref.check(y16, ref)
    assert ok, (mr, mc)


@pytest.mark.parametrize("name", MNAMES)
def test_cpu_check_columns_formula(name):
    x = MZ[f"{name}/x"]
    packed, scales = MZ[f"{name}/packed"], MZ[f"{name}/scales"]
    N = packed.shape[0]
    cols = sorted({0, 1, N >> 1, N - 1})
    pts = s4ref.cpu_check_columns(x, packed, scales, cols)
    ref = MZ[f"{name}/y32"]
    for (m, n), v in pts.items():
        assert abs(v - ref[m, n]) <= 1e-5 * max(1.0, np.abs(ref).max())


def test_generators_match_reference_recipe_hashes():
    gens = json.load(open(os.path.join(GOLDEN, "generators.json")))
    rng = np.random.default_rng(0)
    for g in gens["make_gemm"]:
        packed, scales = s4ref.make_gemm_weights(rng, g["K"], g["N"])
        assert s4ref.sha256(packed) == g["packed_sha256"]
        assert s4ref.sha256(scales) == g["scales_sha256"]
    rng = np.random.default_rng(0)
    for g in gens["make_chain"][:4]:
        packed, scales = s4ref.make_chain_weights(rng, g["K"], g["N"])
        assert s4ref.sha256(packed) == g["packed_sha256"]
        assert s4ref.sha256(scales) == g["scales_sha256"]


def test_pack_unpack_round_trip():
    rng = np.random.default_rng(5)
    q = rng.integers(0, 16, size=(7, 3, 32), dtype=np.uint8)
    np.testing.assert_array_equal(s4ref.unpack_nibbles(s4ref.pack_nibbles(q)), q)


@pytest.mark.parametrize("N,K", [(128, 64), (8224, 2048), (16, 96), (130, 32), (2048, 6144), (1, 32)])
def test_device_layout_round_trip(N, K):
    rng = np.random.default_rng(N * 7 + K)
    packed, scales = s4ref.config_weights(rng, K, N)
    wq, ws = s4ref.repack_device(packed, scales, N, K)
    nblk, kt = s4ref.tiled_dims(N, K)
    assert wq.shape == (nblk, kt, 8, 32, 4) and ws.shape == (nblk, kt, 8, 8, 4)
    p2, s2 = s4ref.unrepack_device(wq, ws, N, K)
    np.testing.assert_array_equal(p2, packed)
    np.testing.assert_array_equal(s2.view(np.uint16), scales.view(np.uint16))


def test_device_layout_fragment_semantics():
    """Decode the device layout the way the GEMV kernel's fragments do and compare with the
    row-major dequantised matrix: lane (g,t) word (blk,h) = row g+8h, k = 8t..8t+7 of block blk."""
    N, K = 256, 128
    rng = np.random.default_rng(3)
    packed, scales = s4ref.config_weights(rng, K, N)
    wq, ws = s4ref.repack_device(packed, scales, N, K)
    deq = s4ref.dequant(packed, scales)
    nblk, kt = s4ref.tiled_dims(N, K)
    for nb in range(nblk):
        for t_ in range(kt):
            for sub in range(8):
                for lane in range(32):
                    g, t = lane >> 2, lane & 3
                    for j in range(4):
                        blk, h = j >> 1, j & 1
                        w = int(wq[nb, t_, sub, lane, j])
                        lo = [(w >> (4 * i)) & 15 for i in range(4)]
                        hi = [(w >> (16 + 4 * i)) & 15 for i in range(4)]
                        vals = [v for pair in zip(lo, hi) for v in pair]     # k0..k7 in order
                        r = nb * 128 + sub * 16 + g + 8 * h
                        k0 = t_ * 64 + blk * 32 + 8 * t
                        s = np.float32(ws[nb, t_, sub, g, blk * 2 + h])
                        got = (np.array(vals, np.float32) - 8) * s
                        np.testing.assert_array_equal(got, deq[r, k0:k0 + 8])


def test_silu_mul_formula():
    rng = np.random.default_rng(2)
    big = rng.standard_normal((3, 8)).astype(np.float16)
    mid = s4ref.silu_mul(big, 4)
    g = big[:, :4].astype(np.float64)
    u = big[:, 4:].astype(np.float64)
    np.testing.assert_allclose(mid.astype(np.float64), g / (1 + np.exp(-g)) * u, rtol=2e-3, atol=1e-4)


def test_metrics():
    ref = np.array([[1.0, -2.0], [0.5, 4.0]], np.float32)
    assert s4ref.max_rel(ref, ref) == 0.0
    assert abs(s4ref.max_rel(ref + np.float32(0.004), ref) - 0.001) < 1e-7
    assert s4ref.min_row_cosine(ref, ref) > 0.999999
    ok, _, _ = s4ref.check(ref * 1.01, ref)
    assert not ok


def test_add_rmsnorm_restatement_matches_loop():
    """ADD_NORM (wgsl.js:55-78) restated with numpy vs a per-element Python loop of the WGSL body:
    fp32 residual add, sum of squares, inverseSqrt(mean + eps), fp16 store of v * inv * w."""
    rng = np.random.default_rng(5)
    M, D = 3, 40
    x = rng.standard_normal((M, D)).astype(np.float32)
    y = (rng.standard_normal((M, D)) * 3).astype(np.float16)
    w = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    xn, h = s4ref.add_rmsnorm(x, y, w, eps=1e-6)
    for m in range(M):
        row = [float(np.float32(x[m, c]) + np.float32(y[m, c])) for c in range(D)]
        inv = 1.0 / np.sqrt(sum(v * v for v in row) / D + 1e-6)
        for c in range(D):
            assert xn[m, c] == np.float32(row[c])
            assert abs(float(h[m, c]) - row[c] * inv * w[c]) <= 1e-3 * max(1.0, abs(row[c] * inv * w[c]))
    # no add, unit weight: rows come out with mean square ~1
    _, h1 = s4ref.add_rmsnorm(x)
    np.testing.assert_allclose((h1.astype(np.float64) ** 2).mean(1), 1.0, rtol=2e-3)


def _js_from_half(h):
    e, f = (h >> 10) & 31, h & 1023
    v = (1024 + f) * 2.0 ** (e - 25) if e else f * 2.0 ** -24
    return -v if h & 0x8000 else v


def _js_to_half(x):
    """Line-by-line port of toHalf (wire.js:8-15): x rounded to float32, then to fp16 bits."""
    b = int(np.array([x], dtype=np.float32).view(np.uint32)[0])
    f32 = float(np.float32(x))
    e, rest = ((b >> 23) & 255) - 112, b & 0x1FFF
    if 0 < e < 31:
        h = (e << 10) | ((b >> 13) & 1023)
        return h + 1 if rest > 0x1000 or (rest == 0x1000 and h & 1) else h
    if e >= 31:
        return 0x7C00
    u = f32 * 2.0 ** 24
    f = int(np.floor(u))
    return f + 1 if u - f > 0.5 or (u - f == 0.5 and f & 1) else f


def _js_decode(wire, N, G):
    """decodeScales (wire.js:19-33) as written, element by element."""
    b = np.frombuffer(wire, dtype=np.uint8)
    out = np.zeros(N * G, dtype=np.uint16)
    for r in range(N):
        m = _js_from_half(int(b[4 * r]) | int(b[4 * r + 1]) << 8)
        j = int(b[4 * r + 2]) | int(b[4 * r + 3]) << 8
        for g in range(G):
            c = int(b[4 * N + r * G + g])
            k = c & 127
            tab = _js_to_half(m * 2.0 ** (-(k * j) / 4096)) & 0xFFFF  # a Uint16Array element
            out[r * G + g] = (tab | ((c & 128) << 8)) & 0xFFFF
    return out.view(np.float16).reshape(N, G)


# row headers the exporter writes (positive normal and subnormal m) and the ones it never writes but a
# decoder still has to map like the JS does: m = 0, -0, exponent 31 (finite in fromHalf), negative m
WIRE_EDGE_M = [0x2C00, 0x1E66, 0x3555, 0x0400, 0x03FF, 0x0001, 0x7BFF, 0x0000, 0x8000, 0x7C00, 0x7FFF,
               0xAC00, 0x83FF, 0x8001]
WIRE_EDGE_J = [0, 1, 37, 4096, 4097, 20000, 65535]


def wire_case(seed, N, G):
    """Seeded wire bytes: headers from the edge lists and random ones, codes covering all 256 values."""
    rng = np.random.default_rng(seed)
    m = np.where(rng.random(N) < 0.5, rng.choice(WIRE_EDGE_M, N), rng.integers(0, 65536, N))
    j = np.where(rng.random(N) < 0.5, rng.choice(WIRE_EDGE_J, N), rng.integers(0, 4000, N))
    hdr = np.stack([m, j], 1).astype(np.uint16)
    codes = rng.integers(0, 256, N * G).astype(np.uint8)
    codes[:256] = np.arange(256, dtype=np.uint8)[:min(256, N * G)]
    return hdr.tobytes() + codes.tobytes()


def test_wire_pow_table_correctly_rounded():
    from decimal import Decimal, getcontext
    getcontext().prec = 60
    ln2 = Decimal(2).ln()
    exact = np.array([float((-(ln2 * r) / 4096).exp()) for r in range(4096)])
    np.testing.assert_array_equal(s4ref.WIRE_POW, exact)


def test_wire_scale_decode_matches_js_restatement():
    for seed, N, G in ((8, 24, 40), (10, 64, 64), (11, 3, 1)):
        wire = wire_case(seed, N, G)
        np.testing.assert_array_equal(s4ref.decode_wire_scales(wire, N, G).view(np.uint16),
                                      _js_decode(wire, N, G).view(np.uint16))


def test_wire_to_half_matches_rne_for_positive_floats():
    # on positive float32 values toHalf is IEEE round-to-nearest-even to fp16
    rng = np.random.default_rng(12)
    x = np.concatenate([np.abs(rng.standard_normal(20000)) * 10.0 ** rng.integers(-9, 5, 20000),
                        np.ldexp(1.0 + np.arange(64) / 1024, -25), [65504.0, 65519.9, 65520.0, 1e-30]])
    x32 = x.astype(np.float32)
    with np.errstate(over="ignore"):  # values above 65520 round to inf, as intended
        want = x32.astype(np.float16).view(np.uint16)
    np.testing.assert_array_equal(s4ref.wire_to_half(x32.astype(np.float64)), want)


def test_wire_scale_encoder_round_trip():
    rng = np.random.default_rng(9)
    sc = (rng.standard_normal((64, 64)) * 0.02).astype(np.float16)
    dec = s4ref.decode_wire_scales(s4ref.encode_wire_scales(sc), 64, 64).astype(np.float64)
    ref = sc.astype(np.float64)
    assert np.all(np.sign(dec) == np.sign(ref))
    # 127 log steps over each row's range: a nearest code is within half a step (plus fp16 rounding)
    b = s4ref.encode_wire_scales(sc)
    j = np.frombuffer(b[:4 * 64], dtype=np.uint16).reshape(64, 2)[:, 1].astype(np.float64)
    half_step = 2.0 ** (j / 8192.0) - 1.0
    big = np.abs(ref) > 1e-4
    rel = np.abs(dec / np.where(big, ref, 1.0) - 1)
    assert np.all(rel[big] <= (half_step[:, None] + 1e-3).repeat(64, 1)[big])


# ---- non-default weight formats and FWHT ----------------------------------------------------------
def _wgsl_decode_block(words, bits, group, scales, bias, n, b, blocks):
    """decodeBlock (kernels.js:23-38) for one block, element by element with the shader's shifts."""
    w = [int(v) for v in words]
    g = (n * blocks + b) // (group // 32)
    sc = np.float32(scales[g])
    out = []
    for i in range(8):
        e = 4 * i
        for c in range(4):
            if bits == 4:
                q = ((w[e >> 3] >> (4 * (e & 7))) >> (4 * c)) & 15
            else:
                q = ((w[e >> 4] >> (2 * (e & 15))) >> (2 * c)) & 3
                if bits == 3:
                    q |= ((w[2] >> e >> c) & 1) << 2
            if bias is None:
                out.append(np.float32(np.float32(q) - np.float32(2 ** (bits - 1))) * sc)
            else:  # fma: exact product and sum in float64, one rounding
                out.append(np.float32(float(q) * float(sc) + float(np.float32(bias[g]))))
    return np.array(out, dtype=np.float32)


@pytest.mark.parametrize("bits,group,asym", [(2, 32, False), (3, 32, False), (4, 64, False), (3, 64, False),
                                             (2, 64, True), (4, 32, True), (3, 32, True)])
def test_format_dequant_matches_wgsl_decode(bits, group, asym):
    rng = np.random.default_rng(bits * 100 + group + asym)
    N, K = 6, 256
    q = rng.integers(0, 2 ** bits, (N, K))
    words = s4ref.pack_format(q, bits)
    sc = (rng.standard_normal(N * K // group) * 0.03).astype(np.float16)
    bi = (rng.standard_normal(N * K // group) * 0.05).astype(np.float16) if asym else None
    deq = s4ref.dequant_format(words, sc, bits, group, bi)
    blocks = K // 32
    for n in range(N):
        for b in range(blocks):
            np.testing.assert_array_equal(deq[n, 32 * b:32 * b + 32],
                                          _wgsl_decode_block(words[n, b], bits, group, sc, bi, n, b, blocks))


@pytest.mark.parametrize("bits,group", [(2, 32), (3, 32), (2, 64), (3, 64), (4, 64)])
def test_transcode_sym_is_exact(bits, group):
    rng = np.random.default_rng(bits + group)
    N, K = 5, 192
    words = s4ref.pack_format(rng.integers(0, 2 ** bits, (N, K)), bits)
    sc = (rng.standard_normal((N, K // group)) * 0.03).astype(np.float16)
    packed, s32 = s4ref.transcode_sym(words, sc, bits, group)
    np.testing.assert_array_equal(s4ref.dequant(packed, s32), s4ref.dequant_format(words, sc, bits, group))


def test_fwht_matches_shader_loop():
    rng = np.random.default_rng(13)
    for n in (2, 8, 64):
        a = rng.standard_normal((3, 2 * n)).astype(np.float16)
        sh = a.astype(np.float32).reshape(-1, n).copy()
        for blk in sh:  # wgsl.js:100-108, one workgroup per block
            h = 1
            while h < n:
                for p in range(n // 2):
                    i = (p // h) * 2 * h + p % h
                    x, y = blk[i], blk[i + h]
                    blk[i], blk[i + h] = x + y, x - y
                h *= 2
        want = (sh * np.float32(1.0 / np.sqrt(float(n)))).astype(np.float16).reshape(a.shape)
        np.testing.assert_array_equal(s4ref.fwht(a, n).view(np.uint16), want.view(np.uint16))


def test_fwht_is_orthonormal():
    rng = np.random.default_rng(14)
    a = rng.standard_normal((4, 1024)).astype(np.float16)
    twice = s4ref.fwht(s4ref.fwht(a, 256), 256)  # H is its own inverse
    np.testing.assert_allclose(twice.astype(np.float32), a.astype(np.float32), atol=4e-3, rtol=4e-3)
