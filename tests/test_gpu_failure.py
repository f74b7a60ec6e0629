"""Failure detection without a GPU fault: the tensor-parallel all-reduce's device-side wait for a peer is bounded in
time. Run on one GPU against a peer that never arrives (elements nothing writes), the wait gives up after its limit, the
call reports WL_ETIMEDOUT, and the device stays usable for the next call."""
import ctypes as C
import time

import numpy as np
import pytest

from gpu_util import dev, empty, host, ptr, rel_l2, weights

pytestmark = pytest.mark.gpu


def test_allreduce_wait_for_a_missing_peer_times_out(wl, oracle):
    t0 = time.perf_counter()
    st = wl.lib().wl_selftest_allreduce_timeout(0, 50)
    took = time.perf_counter() - t0
    assert st == wl.WL_ETIMEDOUT, (st, wl.lib().wl_last_error())
    assert b"peer did not arrive" in wl.lib().wl_last_error()
    assert took < 5.0
    # the context is intact: a matvec right after runs and is right
    O = oracle
    t = O.TYPE_OF["q4_K"]
    rows, cols = 64, 512
    w = weights(O, "q4_K", rows, cols)
    x = np.random.default_rng(0).standard_normal((1, cols)).astype(np.float32)
    dw, dx, dy = dev(w), dev(x.reshape(-1)), empty(rows)      # held: a freed temporary's memory would be reused
    wl.check(wl.lib().wl_matvec(t, ptr(dw), rows, cols, ptr(dx), 1, ptr(dy), None))
    wl.check(wl.lib().wl_kernel_status(0))
    want = x.astype(np.float64) @ O.decode(t, w, rows * cols).reshape(rows, cols).astype(np.float64).T
    assert rel_l2(host(dy), want[0]) <= 1e-4
