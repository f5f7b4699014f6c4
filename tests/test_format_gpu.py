"""The engine's non-default weight formats (kernels.js:5-12: 2/3/4 bits, group 32/64, symmetric and
asymmetric) uploaded through s4_weight_upload_format: a symmetric one's device layout is
byte-identical to an upload of the oracle's exact int4 rewrite, and matmuls through them (GEMV,
chained and tcgen05 families; asymmetric ones without the chain) meet the north-star tolerance
against the oracle's fp32 dequantise-then-matmul of the original format. The
online Hadamard rotation (s4_fwht, wgsl.js:94-110) is checked bit for bit against the oracle."""
import numpy as np
import pytest

from oracle import s4ref

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

FORMATS = [(2, 32), (3, 32), (2, 64), (3, 64), (4, 64)]


def _format_weight(rng, K, N, bits, group):
    words = s4ref.pack_format(rng.integers(0, 2 ** bits, (N, K)), bits)
    sc = (np.abs(rng.standard_normal((N, K // group))) * 0.02 / 2 ** (bits - 1)).astype(np.float16)
    sc = np.where(rng.random(sc.shape) < 0.2, -sc, sc).astype(np.float16)
    return words, sc


@pytest.mark.parametrize("bits,group", FORMATS)
def test_format_upload_layout_and_matmul(ctx, bits, group):
    K, N = 2048, 1536
    rng = np.random.default_rng(bits * 10 + group)
    words, sc = _format_weight(rng, K, N, bits, group)
    W = ctx.upload_format(words, sc, N, K, bits, group)
    packed, s32 = s4ref.transcode_sym(words, sc, bits, group)
    Wr = ctx.upload(packed, s32, N, K)
    for a, b in zip(W.layout(), Wr.layout()):
        np.testing.assert_array_equal(a, b)
    deq = s4ref.dequant_format(words, sc, bits, group)
    for M in (1, 7, 256):
        x = s4ref.config_x(rng, M, K)
        y = ctx.matmul(torch.from_numpy(x).cuda(), W)
        torch.cuda.synchronize()
        ref = x.astype(np.float32) @ deq.T
        ok, mr, mc = s4ref.check(y.cpu().numpy(), ref)
        assert ok, f"bits={bits} group={group} M={M}: max_rel={mr:.2e} min_cos={mc:.7f}"
    W.free()
    Wr.free()


def test_format_upload_from_device_and_chain(ctx):
    K, N = 1024, 640
    rng = np.random.default_rng(31)
    words, sc = _format_weight(rng, K, N, 3, 64)
    W = ctx.upload_format(torch.from_numpy(words.view(np.int32)).cuda(), torch.from_numpy(sc).cuda(), N, K, 3, 64)
    deq = s4ref.dequant_format(words, sc, 3, 64)
    x = torch.from_numpy(s4ref.config_x(rng, 4, K)).cuda()
    y = torch.empty((4, N), dtype=torch.float16, device="cuda")
    chain = ctx.chain([(x, W, y)])
    chain.run()
    torch.cuda.synchronize()
    ok, mr, mc = s4ref.check(y.cpu().numpy(), x.cpu().numpy().astype(np.float32) @ deq.T)
    assert ok, f"max_rel={mr:.2e} min_cos={mc:.7f}"
    chain.free()
    W.free()


def test_format_errors(ctx, pkg):
    for bits, group, K in ((5, 32, 64), (2, 128, 64), (2, 64, 96)):
        with pytest.raises(pkg.S4Error):
            ctx.upload_format(np.zeros(4 * (K // 32) * max(bits, 2), np.uint32), np.zeros(4 * (K // group), np.float16)
                              if K % group == 0 else np.zeros(8, np.float16), 4, K, bits, group)


def _asym_weight(rng, K, N, bits, group):
    """Min-max style asymmetric weights: scale = range / (2^bits - 1), bias near -range / 2."""
    words = s4ref.pack_format(rng.integers(0, 2 ** bits, (N, K)), bits)
    sc = (np.abs(rng.standard_normal((N, K // group))) * 0.04 / (2 ** bits - 1)).astype(np.float16)
    bi = (-(2 ** bits - 1) / 2 * sc.astype(np.float32) * (1 + 0.2 * rng.standard_normal(sc.shape))).astype(np.float16)
    return words, sc, bi


ASYM = [(4, 32), (2, 32), (3, 64), (4, 64)]


@pytest.mark.parametrize("bits,group", ASYM)
def test_asym_matmul(ctx, pkg, bits, group):
    """w = q * scale + bias (kernels.js:11, 36) through the GEMV (1 and 2 token groups) and tcgen05
    families, and the allocation-free entry point."""
    K, N = 2048, 1280
    rng = np.random.default_rng(100 + bits * 10 + group)
    words, sc, bi = _asym_weight(rng, K, N, bits, group)
    W = ctx.upload_format(words, sc, N, K, bits, group, bias=bi)
    deq = s4ref.dequant_format(words, sc, bits, group, bi)
    wq, ws = W.layout()
    packed = s4ref.pack_nibbles(s4ref.unpack_format(words, bits).reshape(N, K // 32, 32).astype(np.uint8))
    ref_wq, ref_ws = s4ref.repack_device(packed, np.repeat(sc, group // 32, 1), N, K)
    np.testing.assert_array_equal(wq, ref_wq.ravel())  # nibbles kept uncentered
    np.testing.assert_array_equal(ws.view(np.uint16), ref_ws.ravel().view(np.uint16))
    for M in (1, 9, 16, 300):
        x = s4ref.config_x(rng, M, K)
        xd = torch.from_numpy(x).cuda()
        y = ctx.matmul(xd, W)
        torch.cuda.synchronize()
        ref = x.astype(np.float32) @ deq.T
        ok, mr, mc = s4ref.check(y.cpu().numpy(), ref)
        assert ok, f"bits={bits} group={group} M={M}: max_rel={mr:.2e} min_cos={mc:.7f}"
    y2 = torch.full((300, N), float("nan"), dtype=torch.float16, device="cuda")
    lib = pkg.load_library()
    assert lib.s4_matmul_noalloc(W.handle, xd.data_ptr(), 300, y2.data_ptr(), None) == 0, lib.s4_last_error().decode()
    torch.cuda.synchronize()
    ok, mr, mc = s4ref.check(y2.cpu().numpy(), ref)
    assert ok, f"noalloc: max_rel={mr:.2e} min_cos={mc:.7f}"
    W.free()


def test_asym_from_device_and_chain_rejects(ctx, pkg):
    K, N = 1024, 384
    rng = np.random.default_rng(7)
    words, sc, bi = _asym_weight(rng, K, N, 2, 64)
    W = ctx.upload_format(torch.from_numpy(words.view(np.int32)).cuda(), torch.from_numpy(sc).cuda(), N, K, 2, 64,
                          bias=torch.from_numpy(bi).cuda())
    x = torch.from_numpy(s4ref.config_x(rng, 3, K)).cuda()
    y = ctx.matmul(x, W)
    torch.cuda.synchronize()
    ok, mr, mc = s4ref.check(y.cpu().numpy(), x.cpu().numpy().astype(np.float32)
                             @ s4ref.dequant_format(words, sc, 2, 64, bi).T)
    assert ok, f"max_rel={mr:.2e} min_cos={mc:.7f}"
    with pytest.raises(pkg.S4Error) as e:
        ctx.chain([(x, W, torch.empty((3, N), dtype=torch.float16, device="cuda"))])
    assert e.value.code == pkg.s4mm.ERR_UNSUPPORTED
    W.free()


# warp-per-block sizes (32..1024) and shared-memory sizes (2, 4096, 32768)
@pytest.mark.parametrize("n,M,K", [(2, 3, 64), (32, 4, 96), (64, 5, 2048), (128, 3, 384), (256, 17, 6144),
                                   (512, 2, 1024), (1024, 3, 2048), (4096, 2, 8192), (32768, 1, 32768)])
def test_fwht_bit_exact(ctx, n, M, K):
    rng = np.random.default_rng(n + M)
    a = rng.standard_normal((M, K)).astype(np.float16)
    d = torch.from_numpy(a).cuda()
    ctx.fwht(d, n)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(d.cpu().numpy().view(np.uint16), s4ref.fwht(a, n).view(np.uint16))


def test_fwht_unaligned_rows(ctx):
    """A 2-byte aligned (not 16-byte) tensor takes the shared-memory form: same bits."""
    rng = np.random.default_rng(2)
    a = rng.standard_normal((3, 512)).astype(np.float16)
    buf = torch.zeros(3 * 512 + 1, dtype=torch.float16, device="cuda")
    d = buf[1:].view(3, 512)
    d.copy_(torch.from_numpy(a))
    ctx.fwht(d, 256)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(d.cpu().numpy().view(np.uint16), s4ref.fwht(a, 256).view(np.uint16))


def test_fwht_then_matmul(ctx):
    """A `had` tensor: the weight was exported against rotated inputs, the engine rotates A first."""
    K, N, n = 2048, 1024, 128
    rng = np.random.default_rng(41)
    packed, scales = s4ref.config_weights(rng, K, N)
    W = ctx.upload(packed, scales, N, K)
    x = s4ref.config_x(rng, 3, K)
    d = torch.from_numpy(x).cuda()
    y = ctx.matmul(ctx.fwht(d, n), W)
    torch.cuda.synchronize()
    _, ref = s4ref.matmul(s4ref.fwht(x, n), packed, scales)
    ok, mr, mc = s4ref.check(y.cpu().numpy(), ref)
    assert ok, f"max_rel={mr:.2e} min_cos={mc:.7f}"


def test_fwht_errors(ctx, pkg):
    d = torch.zeros((2, 96), dtype=torch.float16, device="cuda")
    for n in (3, 1, 65536, 64):  # not a power of two, too small, too large, K % n != 0
        with pytest.raises(pkg.S4Error):
            ctx.fwht(d, n)
    assert ctx.check_errors() == 0


@pytest.mark.parametrize("group", [32, 64])
@pytest.mark.parametrize("K,N", [(2048, 1536), (1024, 2200), (6144, 2048), (1088, 384)])
def test_two_bit_decode_layout_streams_half_the_bytes(ctx, K, N, group):
    """A symmetric 2-bit weight uploaded with S4_UPLOAD_DECODE_LAYOUT also gets the native 2-bit decode
    layout (2048 bytes per 128 x 64 chunk instead of 4096), which the decode GEMV streams: its outputs
    match the oracle, and with the split forced equal they are bit-identical to the int4 layout's (the
    same fp16 fragments enter the same MMAs). Ragged N (not a multiple of 128) and a K whose last
    k-tile holds one 32-block (1088) included; the device footprint counts both layouts; the flag is
    refused for other formats."""
    rng = np.random.default_rng(K + N + group)
    words, sc = _format_weight(rng, K, N, 2, group)
    W = ctx.upload_format(words, sc, N, K, 2, group, decode_layout=True)
    packed, s32 = s4ref.transcode_sym(words, sc, 2, group)
    Wr = ctx.upload(packed, s32, N, K)
    nblk, kt = -(-N // 128), -(-K // 64)
    assert W.device_bytes == Wr.device_bytes + nblk * kt * 2048
    deq = s4ref.dequant_format(words, sc, 2, group)
    try:
        for M in (1, 5, 8, 16):
            x = torch.from_numpy(s4ref.config_x(rng, M, K)).cuda()
            y = ctx.matmul(x, W)
            torch.cuda.synchronize()
            ok, mr, mc = s4ref.check(y.cpu().numpy(), x.cpu().numpy().astype(np.float32) @ deq.T)
            assert ok, f"M={M}: max_rel={mr:.2e} min_cos={mc:.7f}"
            for split in (2, 4):
                ctx.force("gemv", 0, split)
                try:
                    a, b = ctx.matmul(x, W), ctx.matmul(x, Wr)
                    torch.cuda.synchronize()
                finally:
                    ctx.force()
                assert torch.equal(a, b), (M, split)
        assert ctx.check_errors() == 0
        w3, s3 = _format_weight(rng, K, 256, 3, group)
        with pytest.raises(Exception):
            ctx.upload_format(w3, s3, 256, K, 3, group, decode_layout=True)
    finally:
        W.free()
        Wr.free()
