"""ctypes binding of libwindlass_cuda.so (include/windlass.h).

The library is the product: this module only loads it and maps statuses to exceptions. There is no fallback: if
the shared library is missing or cannot be loaded, `lib()` raises.
"""
import ctypes as C
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libwindlass_cuda.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "windlass.h")

WL_OK, WL_EINVAL, WL_EUNSUPPORTED, WL_EIO, WL_EFORMAT, WL_ENOMEM, WL_ECUDA, WL_ENCCL, WL_ETIMEDOUT, WL_CANCELLED = range(10)

TYPES = {"f32": 0, "f16": 1, "q4_0": 2, "q4_1": 3, "q5_0": 6, "q5_1": 7, "q8_0": 8, "q2_K": 10, "q3_K": 11,
         "q4_K": 12, "q5_K": 13, "q6_K": 14, "iq2_xxs": 16, "iq2_xs": 17, "iq3_xxs": 18, "iq1_s": 19, "iq4_nl": 20,
         "iq3_s": 21, "iq2_s": 22, "iq4_xs": 23, "iq1_m": 29, "bf16": 30}


class WindlassError(RuntimeError):
    def __init__(self, status, message):
        super().__init__(f"[{status}] {message}")
        self.status = status


class ArgumentError(WindlassError, ValueError):        # ArgumentException
    pass


class NotSupportedError(WindlassError, NotImplementedError):   # NotSupportedException
    pass


class InvalidDataError(WindlassError, ValueError):     # InvalidDataException
    pass


class OperationCanceledError(WindlassError):           # OperationCanceledException
    pass


_EXC = {WL_EINVAL: ArgumentError, WL_EUNSUPPORTED: NotSupportedError, WL_EFORMAT: InvalidDataError,
        WL_CANCELLED: OperationCanceledError}


class Options(C.Structure):
    _fields_ = [("size", C.c_int32), ("device", C.c_int32), ("max_context", C.c_int32), ("max_batch", C.c_int32),
                ("resident", C.c_int32), ("prefill_path", C.c_int32), ("use_graphs", C.c_int32),
                ("tp_size", C.c_int32), ("tp_rank", C.c_int32), ("tp_nccl_only", C.c_int32),
                ("stream_file", C.c_int32), ("reserved", C.c_int32 * 5),
                ("tp_id", C.c_uint8 * 128)]


class Info(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("layers", "embd", "heads", "kv_heads", "head_dim", "vocab", "context_length",
                                          "max_context", "expert_count", "expert_used", "expert_ff", "moe")] + \
               [("weight_bytes", C.c_int64), ("device_bytes", C.c_int64), ("arch", C.c_char * 32),
                ("tp_size", C.c_int32), ("tp_rank", C.c_int32), ("tp_fused", C.c_int32)]


class Stats(C.Structure):
    _fields_ = [("bytes_h2d", C.c_int64), ("expert_runs", C.c_int64), ("forward_calls", C.c_int64),
                ("batch_calls", C.c_int64), ("tokens", C.c_int64), ("last_forward_ms", C.c_double),
                ("kernel_launches", C.c_int64)]


class ProfileEntry(C.Structure):
    _fields_ = [("launches", C.c_int64), ("ms", C.c_double), ("bytes", C.c_double)]


class SynthSpec(C.Structure):
    _fields_ = [("arch", C.c_char * 16)] + \
               [(n, C.c_int32) for n in ("layers", "embd", "heads", "kv_heads", "head_dim", "ff", "vocab",
                                          "context_length", "experts", "experts_used", "expert_ff")] + \
               [(n, C.c_float) for n in ("rope_base", "rms_eps", "sigma")] + \
               [(n, C.c_int32) for n in ("type_attn", "type_attn_v", "type_ffn", "type_ffn_down", "type_embd",
                                          "type_output")] + \
               [("seed", C.c_uint64)]


PROGRESS = C.CFUNCTYPE(None, C.c_int32, C.c_int32, C.c_void_p)

_lib = None


def declared_functions():
    """Names of the functions include/windlass.h declares."""
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(wl_[a-z_0-9]+)\s*\(", src)) - {"wl_progress_fn"})


def lib():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise OSError(f"{LIB_PATH} is missing: build it with `python -m windlass_b200.build` (there is no CPU fallback)")
    L = C.CDLL(LIB_PATH)
    P, I32, I64, U64, F = C.c_void_p, C.c_int32, C.c_int64, C.c_uint64, C.c_float
    sig = {
        "wl_options_init": (None, [C.POINTER(Options)]), "wl_last_error": (C.c_char_p, []),
        "wl_version": (C.c_char_p, []), "wl_tp_unique_id": (I32, [P, I32]),
        "wl_open": (I32, [C.c_char_p, C.POINTER(Options), C.POINTER(P)]),
        "wl_open_synthetic": (I32, [C.POINTER(SynthSpec), C.POINTER(Options), C.POINTER(P)]),
        "wl_close": (I32, [P]), "wl_info_get": (I32, [P, C.POINTER(Info)]), "wl_stats_get": (I32, [P, C.POINTER(Stats)]),
        "wl_seq_new": (I32, [P, C.POINTER(P)]), "wl_seq_free": (I32, [P]), "wl_seq_truncate": (I32, [P, I32]),
        "wl_seq_length": (I32, [P, C.POINTER(I32)]), "wl_truncate": (I32, [P, I32]),
        "wl_length": (I32, [P, C.POINTER(I32)]),
        "wl_forward": (I32, [P, P, P, I32, I32, I32, P, P, PROGRESS, P]),
        "wl_forward_batch": (I32, [P, P, P, I32, P, P, PROGRESS, P]),
        "wl_forward_argmax": (I32, [P, P, P, I32, I32, I32, P, P, PROGRESS, P]),
        "wl_forward_batch_argmax": (I32, [P, P, P, I32, P, P, PROGRESS, P]),
        "wl_forward_mixed": (I32, [P, P, P, I32, P, P, P, P, PROGRESS, P]),
        "wl_forward_sample": (I32, [P, P, P, I32, I32, C.c_double, C.c_double, C.c_double, P, P, PROGRESS, P]),
        "wl_forward_batch_sample": (I32, [P, P, P, I32, P, P, P, P, P, PROGRESS, P]),
        "wl_sample": (I32, [P, I32, C.c_double, C.c_double, C.c_double, P, P]),
        "wl_generate_greedy": (I32, [P, P, I32, I32, P, I32, I32, P, C.POINTER(I32), P]),
        "wl_argmax": (I32, [P, I32, I32, P, P]), "wl_route": (I32, [P, I32, I32, I32, I32, P, P, P]), "wl_kernel_status": (I32, [I32]),
        "wl_dequant": (I32, [I32, P, I64, P, P]),
        "wl_matvec": (I32, [I32, P, I32, I32, P, I32, P, P]),
        "wl_matvec_static": (I32, [I32, P, I32, I32, P, I32, P, P]),
        "wl_tiles_size": (I32, [I32, I32, I32, C.POINTER(I64)]),
        "wl_make_tiles": (I32, [I32, P, I32, I32, P, P]),
        "wl_matvec_tiles": (I32, [I32, P, I32, I32, P, I32, P, P]),
        "wl_bench_matvec_tiles": (I32, [I32, P, I32, I32, I32, P, I32, P, I32, C.POINTER(C.c_double), P]),
        "wl_matmul": (I32, [I32, P, I32, I32, P, I32, P, I32, P]),
        "wl_gemm_tiles": (I32, [I32, P, I32, I32, P, I32, P, P]),
        "wl_selftest_allreduce_timeout": (I32, [I32, I32]),
        "wl_synth_tensor": (I32, [I32, U64, C.c_uint32, I64, I64, F, F, P, P]),
        "wl_bench_decode": (I32, [P, P, I32, I32, C.POINTER(C.c_double)]),
        "wl_bench_matvecs": (I32, [P, I32, I32, C.POINTER(C.c_double), C.POINTER(C.c_double)]),
        "wl_profile": (I32, [P, I32]), "wl_profile_get": (I32, [P, I32, C.POINTER(ProfileEntry)]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def check(status):
    if status != WL_OK:
        msg = lib().wl_last_error()
        raise _EXC.get(status, WindlassError)(status, msg.decode() if msg else "")
    return status


def options(**kw):
    o = Options()
    lib().wl_options_init(C.byref(o))
    for k, v in kw.items():
        if k == "tp_id":
            if v is not None:
                C.memmove(o.tp_id, bytes(v), 128)
        else:
            setattr(o, k, v)
    return o


def tp_unique_id():
    """A fresh tensor-parallel group id (128 bytes; wl_tp_unique_id): one rank makes it, every rank opens with it."""
    buf = (C.c_uint8 * 128)()
    check(lib().wl_tp_unique_id(buf, 128))
    return bytes(buf)
