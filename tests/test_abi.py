"""The C-ABI library loads, exports what include/windlass.h declares, and reports host-side errors with the
reference's exception kinds, without a GPU (no compute call is made)."""
import ctypes as C
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_library_exports_every_declared_function(wl):
    names = wl.declared_functions()
    assert "wl_forward" in names and "wl_forward_batch" in names and "wl_matvec" in names
    out = subprocess.run(["nm", "-D", "--defined-only", wl.LIB_PATH], capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = [n for n in names if n not in exported]
    assert not missing, f"declared but not exported: {missing}"
    lib = wl.lib()
    for n in names:
        assert getattr(lib, n) is not None


def test_library_is_built_for_sm100a(wl):
    out = subprocess.run(["cuobjdump", "--list-elf", wl.LIB_PATH], capture_output=True, text=True)
    if out.returncode != 0:
        pytest.skip("cuobjdump unavailable")
    assert "sm_100a" in out.stdout


def test_options_and_version(wl):
    o = wl.options()
    assert o.size == C.sizeof(wl.Options) and o.max_batch == 64 and o.resident == -1
    assert b"sm_100a" in wl.lib().wl_version()


def _open(wl, path):
    h = C.c_void_p()
    o = wl.options()
    return wl.lib().wl_open(path.encode(), C.byref(o), C.byref(h)), h


def test_open_missing_file_is_io_error(wl, tmp_path):
    st, h = _open(wl, str(tmp_path / "nope.gguf"))
    assert st == wl.WL_EIO and not h.value
    assert b"Cannot open" in wl.lib().wl_last_error()


def test_open_garbage_is_format_error(wl, tmp_path):
    p = tmp_path / "bad.gguf"
    p.write_bytes(b"not a gguf file at all, just text" * 4)
    st, _ = _open(wl, str(p))
    assert st == wl.WL_EFORMAT
    assert b"is not a GGUF file" in wl.lib().wl_last_error()


def test_truncated_file_is_format_error(wl, oracle, tmp_path):
    p = oracle.write_tiny(str(tmp_path / "t.gguf"), type=oracle.Q8_0)
    data = open(p, "rb").read()
    q = tmp_path / "trunc.gguf"
    q.write_bytes(data[: len(data) // 2])
    st, _ = _open(wl, str(q))
    assert st == wl.WL_EFORMAT
    assert b"extends past the end" in wl.lib().wl_last_error()


def test_unsupported_architecture(wl, oracle, tmp_path):
    """ModelConfig.From refuses architectures outside its list (src/ModelConfig.cs:40-42)."""
    O = oracle
    g = O.lib().or_gguf_mem_new
    g.restype = C.c_void_p
    h = g()
    O.lib().or_gguf_mem_set_string.argtypes = [C.c_void_p, C.c_char_p, C.c_char_p]
    O.lib().or_gguf_mem_set_string(h, b"general.architecture", b"gpt2")
    O.lib().or_gguf_save(h, str(tmp_path / "gpt2.gguf").encode())
    O.lib().or_gguf_close(h)
    st, _ = _open(wl, str(tmp_path / "gpt2.gguf"))
    assert st == wl.WL_EUNSUPPORTED
    assert b"not supported" in wl.lib().wl_last_error()


def test_null_arguments_are_argument_errors(wl):
    L = wl.lib()
    assert L.wl_forward(None, None, None, 1, 0, 0, None, None, wl.PROGRESS(), None) == wl.WL_EINVAL
    assert L.wl_matvec(12, None, 8, 256, None, 1, None, None) == wl.WL_EINVAL
    assert L.wl_matvec(12, None, 8, 100, None, 1, None, None) == wl.WL_EINVAL    # cols not whole blocks
    assert L.wl_dequant(15, None, 256, None, None) == wl.WL_EUNSUPPORTED       # Q8_K has no decoder
    assert L.wl_synth_tensor(23, 0, 0, 1, 256, 0.02, 0.0, None, None) == wl.WL_EUNSUPPORTED
    assert L.wl_close(None) == wl.WL_OK


def test_no_cpu_fallback_in_the_product():
    """The product never includes, imports or loads the oracle."""
    import re
    bad = re.compile(r'#include\s+"[^"]*oracle|^\s*(from|import)\s+oracle|liboracle|\bor_[a-z_]+\(', re.M)
    for d, _, files in os.walk(os.path.join(ROOT, "windlass_b200")):
        for f in files:
            if f.endswith((".py", ".cpp", ".cu", ".h", ".cuh")):
                src = open(os.path.join(d, f), encoding="utf-8").read()
                assert not bad.search(src), f"{f} reaches the oracle"


def test_streamed_layers_refuse_the_cuda_core_prefill(wl):
    """resident = 0 keeps only the tensor-core layout of streamed weights, so prefill_path 1 is refused up front."""
    from windlass_b200.transformer import config0_spec
    h = C.c_void_p()
    o = wl.options(resident=0, prefill_path=1)
    spec = config0_spec()
    st = wl.lib().wl_open_synthetic(C.byref(spec), C.byref(o), C.byref(h))
    assert st == wl.WL_EUNSUPPORTED and b"prefill_path 1" in wl.lib().wl_last_error()


def test_stream_file_needs_a_streamed_file_model(wl, oracle, tmp_path):
    """stream_file = 1 reads the layers from the model's GGUF file: refused with resident weights, for a synthetic model
    (no file) and for a value other than 0 or 1, before any device work."""
    from windlass_b200.transformer import config0_spec
    h = C.c_void_p()
    spec = config0_spec()
    st = wl.lib().wl_open_synthetic(C.byref(spec), C.byref(wl.options(resident=0, stream_file=1)), C.byref(h))
    assert st == wl.WL_EINVAL and b"synthetic model" in wl.lib().wl_last_error()
    path = oracle.write_synth(str(tmp_path / "c0.gguf"), spec)
    st = wl.lib().wl_open(path.encode(), C.byref(wl.options(resident=1, stream_file=1)), C.byref(h))
    assert st == wl.WL_EINVAL and b"resident = 0" in wl.lib().wl_last_error()
    st = wl.lib().wl_open(path.encode(), C.byref(wl.options(resident=0, stream_file=2)), C.byref(h))
    assert st == wl.WL_EINVAL and b"0 or 1" in wl.lib().wl_last_error()
