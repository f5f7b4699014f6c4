"""The allocation-free matmul entry point, for callers that cannot allocate device memory at call
time (a host whose memory manager owns the whole device, a serving loop that must not take
cudaMalloc's implicit device synchronisation): its scratch lives in a static device array.

Called through the C ABI and checked against the CPU oracle (fp32 dequantise-then-matmul) within
the tolerance the other GPU tests use (max relative error 2e-3, per-row cosine 0.99999), on two calls
in a row, since every call reuses the same static array; the array's error word must read clean
afterwards. A weight stays usable after its context is closed (the call needs none). Collected last
so that a stop-at-first-failure run has already run every other test; it also passes alone in a
fresh process."""
import ctypes as C

import numpy as np
import pytest

from oracle import s4ref

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _noalloc_errors(lib, clear=1):
    f = C.c_uint32()
    assert lib.s4_noalloc_check_errors(0, C.byref(f), clear) == 0, lib.s4_last_error().decode()
    return f.value


@pytest.mark.parametrize("K,N,M", [(2048, 3072, 64), (6144, 2048, 300), (96, 200, 5), (2048, 8224, 1),
                                   (2048, 12288, 128)])
def test_noalloc_matches_oracle(pkg, ctx, K, N, M):
    lib = pkg.load_library()
    rng = np.random.default_rng(K + N + M)
    packed, scales = s4ref.config_weights(rng, K, N)
    W = ctx.upload(packed, scales, N, K)  # set-up may allocate; the call under test does not
    x = torch.from_numpy(s4ref.config_x(rng, M, K)).cuda()
    _, ref = s4ref.matmul(x.cpu().numpy(), packed, scales)
    stream = torch.cuda.current_stream().cuda_stream
    _noalloc_errors(lib)
    for call in range(2):
        y = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
        rc = lib.s4_matmul_noalloc(W.handle, x.data_ptr(), M, y.data_ptr(), stream)
        assert rc == 0, lib.s4_last_error().decode()
        torch.cuda.synchronize()
        ok, mr, mc = s4ref.check(y.cpu().numpy(), ref)
        assert ok, f"call {call}: max_rel={mr:.3e} min_cos={mc:.7f}"
    assert _noalloc_errors(lib) == 0


def test_noalloc_after_context_closed(pkg):
    """The weight records its device and SM count: a call after s4_destroy of its context reads
    nothing the context owned."""
    lib = pkg.load_library()
    K, N, M = 2048, 3072, 48
    rng = np.random.default_rng(7)
    packed, scales = s4ref.config_weights(rng, K, N)
    c = pkg.Context(0)
    W = c.upload(packed, scales, N, K)
    c.close()
    x = torch.from_numpy(s4ref.config_x(rng, M, K)).cuda()
    _, ref = s4ref.matmul(x.cpu().numpy(), packed, scales)
    for call in range(2):
        y = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
        assert lib.s4_matmul_noalloc(W.handle, x.data_ptr(), M, y.data_ptr(), None) == 0, lib.s4_last_error().decode()
        torch.cuda.synchronize()
        ok, mr, mc = s4ref.check(y.cpu().numpy(), ref)
        assert ok, f"call {call}: max_rel={mr:.3e} min_cos={mc:.7f}"
    assert _noalloc_errors(lib) == 0
    W.free()


def test_noalloc_rejects_sizes_beyond_its_scratch(pkg, ctx):
    lib = pkg.load_library()
    N, K = 16385 * 128, 32  # 16385 n-blocks: one more tile counter than the static scratch holds
    packed = np.full((N, 1, 16), 0x88, dtype=np.uint8)
    scales = np.zeros((N, 1), dtype=np.float16)
    W = ctx.upload(packed, scales, N, K)
    x = torch.zeros((1, K), dtype=torch.float16, device="cuda")
    y = torch.empty((1, N), dtype=torch.float16, device="cuda")
    rc = lib.s4_matmul_noalloc(W.handle, x.data_ptr(), 1, y.data_ptr(), None)
    assert rc == pkg.s4mm.ERR_INVALID
    assert b"static scratch" in lib.s4_last_error()
    assert lib.s4_matmul_noalloc(W.handle, x.data_ptr(), 0, y.data_ptr(), None) == 0  # M == 0: no-op
    f = C.c_uint32()
    assert lib.s4_noalloc_check_errors(0, None, 0) == pkg.s4mm.ERR_INVALID
    assert lib.s4_noalloc_check_errors(-1, C.byref(f), 0) == pkg.s4mm.ERR_INVALID
