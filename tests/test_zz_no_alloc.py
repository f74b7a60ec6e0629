"""wl_matvec_static: the tensor-core Q4_K matvec with its scratch in a static device array (no allocation in the call),
for callers whose device memory is all planned and owned by their own allocator.

It runs the tensor-core kernel on the GGUF rows through a TMA tensor map, where wl_matvec repacks the rows into tiles
first, so both entry points must agree within the matvec tolerance (1e-4 relative L2) on two calls in a row that
share the static scratch, at a small shape, with more than 8 columns (the scratch is reused across 8-column chunks)
and at the largest accepted width. In a fresh process, calls after the first leave the device's free memory as it
was, while wl_matvec on the same shape grows its scratch. Shapes beyond the limit and formats without the tensor-core
path are rejected before any device work. The file name sorts last, so it also runs after every other GPU test in one
session.
"""
import ctypes as C
import os
import subprocess
import sys

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


_NO_ALLOC_CHILD = r"""
import ctypes as C, sys
import torch
sys.path.insert(0, sys.argv[1])
from windlass_b200 import _lib
L = _lib.lib()
rows, cols = 64, 32768
w = torch.empty(rows * cols // 256 * 144, dtype=torch.uint8, device="cuda")
x = torch.randn(16 * cols, device="cuda")
y = torch.empty(16 * rows, device="cuda")
_lib.check(L.wl_synth_tensor(12, 77, 0x9A0, rows, cols, C.c_float(0.02), C.c_float(0.0), C.c_void_p(w.data_ptr()), None))
def static(n):
    _lib.check(L.wl_matvec_static(12, C.c_void_p(w.data_ptr()), rows, cols, C.c_void_p(x.data_ptr()), n,
                                  C.c_void_p(y.data_ptr()), None))
for n in (1, 3, 8, 16):            # the first call looks up the static array and sets the kernel attributes
    static(n)
torch.cuda.synchronize()
free0 = torch.cuda.mem_get_info()[0]
for n in (16, 8, 3, 1, 16):
    static(n)
torch.cuda.synchronize()
free1 = torch.cuda.mem_get_info()[0]
_lib.check(L.wl_matvec(12, C.c_void_p(w.data_ptr()), rows, cols, C.c_void_p(x.data_ptr()), 8, C.c_void_p(y.data_ptr()),
                       None))
torch.cuda.synchronize()
free2 = torch.cuda.mem_get_info()[0]
print(free0, free1, free2)
"""


def test_static_calls_allocate_no_device_memory(wl, tmp_path):
    """A fresh process (kernels loaded eagerly, so that no lazy module load is counted): after the first calls, more
    wl_matvec_static calls at the largest width leave the free device memory unchanged, to the byte; wl_matvec on the
    same shape then allocates its scratch (about 2.2 MB), which the same measurement sees."""
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, CUDA_MODULE_LOADING="EAGER")
    r = subprocess.run([sys.executable, "-c", _NO_ALLOC_CHILD, root], capture_output=True, text=True, env=env,
                       timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    free0, free1, free2 = (int(v) for v in r.stdout.split()[-3:])
    assert free1 == free0, f"wl_matvec_static changed the free device memory by {free0 - free1} bytes"
    assert free2 < free1, "the measurement did not see wl_matvec's scratch allocation"
