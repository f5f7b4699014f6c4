"""A bounded device wait that runs out reports through the error word and leaves the context usable.

The cross-GPU barrier (s4_peer_barrier) waits up to one second for every rank's flag. Here it runs on
one GPU as rank 0 of 2, and "rank 1's" flag array is a second zeroed buffer in this GPU's own memory
that nothing ever signals, so the wait must expire: the kernel sets kErrWaitTimeout in the context's
error word and returns (no trap, no hang), s4_check_errors reports it, s4_clear_errors resets it, and
the next matmul on the same context is correct. Failure detection of the reference's host side
(engine.js:109, 373: GPU errors collected after the forward and rethrown) maps to this error word."""
import time

import numpy as np
import pytest

from oracle import s4ref

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

K_ERR_WAIT_TIMEOUT = 1  # kErrWaitTimeout in csrc/common.cuh


def test_peer_barrier_wait_expires_and_context_recovers(pkg):
    c = pkg.Context(0)
    try:
        assert c.check_errors() == 0
        mine = c.buffer_alloc(64)      # rank 0's flag array (zeroed)
        silent = c.buffer_alloc(64)    # the absent rank's flag array: nobody writes rank 1's slot of `mine`
        t0 = time.time()
        c.peer_barrier([mine, silent], rank=0, epoch=1)
        err = c.check_errors()         # synchronises: returns once the kernel gave up
        dt = time.time() - t0
        assert err & K_ERR_WAIT_TIMEOUT, f"expected the wait-timeout bit, got 0x{err:x}"
        assert 0.5 < dt < 30.0, f"the bounded wait took {dt:.2f} s"
        c.clear_errors()
        assert c.check_errors() == 0
        # the context is usable after the expired wait
        rng = np.random.default_rng(3)
        Kd, N, M = 2048, 3072, 8
        packed, scales = s4ref.config_weights(rng, Kd, N)
        W = c.upload(packed, scales, N, Kd)
        x = torch.from_numpy(s4ref.config_x(rng, M, Kd)).cuda()
        y = c.matmul(x, W)
        torch.cuda.synchronize()
        _, ref = s4ref.matmul(x.cpu().numpy(), packed, scales)
        ok, mr, mc = s4ref.check(y.cpu().numpy(), ref)
        assert ok, f"max_rel={mr:.2e} min_cos={mc:.7f}"
        assert c.check_errors() == 0
        W.free()
        c.buffer_free(mine)
        c.buffer_free(silent)
    finally:
        c.close()


def test_norm_peer_wait_expires_and_context_recovers(pkg):
    """The waiting half of the split barrier, run out: rank 0 of 2 signals (its own slot and the
    absent rank's array get the epoch), then an ADD_NORM that waits for both ranks finds rank 1's slot
    of its own array never written. Thread 0 gives up after one second, sets kErrWaitTimeout, and the
    kernel finishes (it normalises what it has); the context then runs the same call correctly."""
    c = pkg.Context(0)
    try:
        mine = c.buffer_alloc(64)
        silent = c.buffer_alloc(64)
        M, D = 64, 2048
        x = (torch.randn((M, D), device="cuda") * 2).contiguous()
        y = torch.randn((M, D), device="cuda").half()
        c.peer_signal([mine, silent], 0)
        t0 = time.time()
        c.add_rmsnorm(x.clone(), y, wait_flags=mine, nranks=2)
        err = c.check_errors()
        dt = time.time() - t0
        assert err & K_ERR_WAIT_TIMEOUT, f"expected the wait-timeout bit, got 0x{err:x}"
        assert 0.5 < dt < 30.0, f"the bounded wait took {dt:.2f} s"
        c.clear_errors()
        x1 = x.clone()
        h = c.add_rmsnorm(x1, y, wait_flags=mine, nranks=1)  # rank 0 alone: its own signal is there
        torch.cuda.synchronize()
        assert c.check_errors() == 0
        xr, hr = s4ref.add_rmsnorm(x.cpu().numpy(), y.cpu().numpy())
        np.testing.assert_array_equal(x1.cpu().numpy(), xr)
        np.testing.assert_allclose(h.cpu().numpy().astype(np.float32), hr.astype(np.float32), rtol=1e-3, atol=1e-3)
        c.buffer_free(mine)
        c.buffer_free(silent)
    finally:
        c.close()
