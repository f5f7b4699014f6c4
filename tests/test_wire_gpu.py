"""Download-format ("wire") scales decoded on the device (decodeScales, wire.js:19-33) against the
oracle bit for bit, on headers the exporter writes and on the ones it never writes (m = 0, -0,
exponent 31, negative m), with codes covering all 256 values; and weights uploaded through the wire
path: their device layout is byte-identical to an upload of the oracle-decoded scales, and a matmul
through them meets the north-star tolerance against the oracle."""
import numpy as np
import pytest

from oracle import s4ref
from test_oracle import wire_case

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("seed,N,G", [(20, 1, 1), (21, 3, 7), (22, 257, 64), (23, 4096, 256), (24, 12288, 64)])
def test_decode_bit_exact(ctx, seed, N, G):
    wire = wire_case(seed, N, G)
    want = s4ref.decode_wire_scales(wire, N, G).view(np.uint16)
    # offset the wire bytes by one: the decoder reads bytes and needs no alignment
    buf = torch.zeros(len(wire) + 1, dtype=torch.uint8, device="cuda")
    buf[1:] = torch.frombuffer(bytearray(wire), dtype=torch.uint8).cuda()
    got = ctx.decode_wire_scales(buf[1:], N, G)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(got.cpu().numpy().view(np.uint16), want)


def test_decode_on_stream_repeated(ctx):
    N, G = 512, 128
    wire = wire_case(25, N, G)
    want = s4ref.decode_wire_scales(wire, N, G).view(np.uint16)
    dev = torch.frombuffer(bytearray(wire), dtype=torch.uint8).cuda()
    s = torch.cuda.Stream()
    out = torch.empty((N, G), dtype=torch.float16, device="cuda")
    with torch.cuda.stream(s):
        for _ in range(3):
            out.fill_(1.0)
            ctx.decode_wire_scales(dev, N, G, out=out, stream=s)
    s.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy().view(np.uint16), want)


@pytest.mark.parametrize("K,N", [(2048, 3072), (1024, 200), (6144, 2048)])
def test_upload_wire_matches_decoded_upload(ctx, K, N):
    rng = np.random.default_rng(K + N)
    packed, scales = s4ref.config_weights(rng, K, N)
    scales = np.where(rng.random(scales.shape) < 0.3, -scales, scales)  # the format carries a sign bit
    wire = s4ref.encode_wire_scales(scales.reshape(N, K // 32))
    dec = s4ref.decode_wire_scales(wire, N, K // 32)
    Ww = ctx.upload_wire(packed, wire, N, K)
    Wd = ctx.upload(packed, dec, N, K)
    for a, b in zip(Ww.layout(), Wd.layout()):
        np.testing.assert_array_equal(a, b)
    deq = s4ref.dequant(packed, dec)
    for M in (1, 5, 300):
        x = s4ref.config_x(rng, M, K)
        y = ctx.matmul(torch.from_numpy(x).cuda(), Ww)
        torch.cuda.synchronize()
        _, ref = s4ref.matmul(x, packed, dec, deq)
        ok, mr, mc = s4ref.check(y.cpu().numpy(), ref)
        assert ok, f"M={M}: max_rel={mr:.2e} min_cos={mc:.7f}"
    Ww.free()
    Wd.free()


def test_wire_argument_errors(ctx, pkg):
    dev = torch.zeros(64, dtype=torch.uint8, device="cuda")
    with pytest.raises(pkg.S4Error):
        ctx.decode_wire_scales(dev, 0, 4)
    with pytest.raises(pkg.S4Error):
        ctx.decode_wire_scales(dev, 4, 0)
    with pytest.raises(pkg.S4Error):
        ctx.decode_wire_scales(dev, 8, 8)  # 96 bytes needed, 64 given
    odd = torch.zeros(9, dtype=torch.float16, device="cuda")
    with pytest.raises(pkg.S4Error):  # fp16 output not 2-byte aligned
        ctx.decode_wire_scales(dev, 2, 2, out=odd.view(torch.uint8)[1:17].view(torch.uint8))
    packed = np.zeros(4 * 2 * 16, dtype=np.uint8)
    with pytest.raises(pkg.S4Error):
        ctx.upload_wire(packed, b"\0" * 11, 4, 64)  # 4*4 + 4*2 = 24 bytes expected
    with pytest.raises(pkg.S4Error):  # K not a multiple of 32 (sizes consistent for G = 1)
        ctx.upload_wire(np.zeros(4 * 16, dtype=np.uint8), b"\0" * 20, 4, 48)
    assert ctx.check_errors() == 0
