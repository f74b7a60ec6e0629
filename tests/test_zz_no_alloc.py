"""wl_matvec_static: the tensor-core Q4_K matvec with its scratch in a static device array (no allocation in the call).

It runs the same kernels as wl_matvec, so both entry points must agree within the matvec tolerance (1e-4 relative
L2) on two calls in a row that share the static scratch, at a small shape, with more than 8 columns (the scratch is
reused across 8-column chunks) and at the largest accepted width. Shapes beyond the limit and formats without the
tensor-core path are rejected before any device work. The file name sorts last, so it also runs after every other
GPU test in one session.
"""
import ctypes as C

import numpy as np
import pytest

from gpu_util import empty, host, ptr, rel_l2, torch_cuda

pytestmark = pytest.mark.gpu

Q4_K, Q6_K = 12, 14
TOL = 1e-4


def _q4k(wl, rows, cols, tid):
    w = empty(rows * cols // 256 * 144, "uint8")
    wl.check(wl.lib().wl_synth_tensor(Q4_K, 77, tid, rows, cols, C.c_float(0.02), C.c_float(0.0), ptr(w), None))
    return w


def _x(ncols, cols, seed):
    torch = torch_cuda()
    g = torch.Generator(device="cpu").manual_seed(seed)
    return torch.randn(ncols * cols, generator=g, dtype=torch.float32).cuda()


def _both(wl, w, rows, cols, x, ncols):
    ref = empty(ncols * rows)
    wl.check(wl.lib().wl_matvec(Q4_K, ptr(w), rows, cols, ptr(x), ncols, ptr(ref), None))
    return host(ref)


@pytest.mark.parametrize("rows,cols,n1,n2", [(300, 4096, 3, 8), (257, 2048, 11, 1), (64, 32768, 8, 2)])
def test_static_scratch_matches_wl_matvec_on_two_calls_in_a_row(wl, rows, cols, n1, n2):
    L = wl.lib()
    w = _q4k(wl, rows, cols, 0x900 + cols // 256)
    x1, x2 = _x(n1, cols, 1), _x(n2, cols, 2)
    y1, y2 = empty(n1 * rows), empty(n2 * rows)
    # back to back on one stream: the second call reuses the scratch the first one used
    wl.check(L.wl_matvec_static(Q4_K, ptr(w), rows, cols, ptr(x1), n1, ptr(y1), None))
    wl.check(L.wl_matvec_static(Q4_K, ptr(w), rows, cols, ptr(x2), n2, ptr(y2), None))
    got1, got2 = host(y1), host(y2)
    want1, want2 = _both(wl, w, rows, cols, x1, n1), _both(wl, w, rows, cols, x2, n2)
    assert np.isfinite(got1).all() and np.isfinite(got2).all()
    assert rel_l2(got1, want1) <= TOL, rel_l2(got1, want1)
    assert rel_l2(got2, want2) <= TOL, rel_l2(got2, want2)


def test_static_scratch_rejects_what_it_cannot_hold(wl):
    L = wl.lib()
    cols = 32768 + 256
    w = empty(4 * cols // 256 * 144, "uint8")
    x = empty(cols)
    y = empty(4)
    with pytest.raises(wl.ArgumentError, match="static scratch limit"):
        wl.check(L.wl_matvec_static(Q4_K, ptr(w), 4, cols, ptr(x), 1, ptr(y), None))
    w6 = empty(4 * 1024 // 256 * 210, "uint8")
    with pytest.raises(wl.NotSupportedError, match="use wl_matvec"):
        wl.check(L.wl_matvec_static(Q6_K, ptr(w6), 4, 1024, ptr(x), 1, ptr(y), None))
