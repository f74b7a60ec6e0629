"""ctypes binding of the CPU oracle (liboracle.so). Test infrastructure: only tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg import this module, and only to check or to time the reference's CPU arithmetic."""
import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

# ggml_type numbers (Gguf.cs:19-25)
F32, F16, Q4_0, Q4_1, Q5_0, Q5_1, Q8_0 = 0, 1, 2, 3, 6, 7, 8
Q2_K, Q3_K, Q4_K, Q5_K, Q6_K = 10, 11, 12, 13, 14
IQ2_XXS, IQ2_XS, IQ3_XXS, IQ1_S, IQ4_NL, IQ3_S, IQ2_S, IQ4_XS, IQ1_M, BF16 = 16, 17, 18, 19, 20, 21, 22, 23, 29, 30
NAMES = {F32: "f32", F16: "f16", BF16: "bf16", Q4_0: "q4_0", Q4_1: "q4_1", Q5_0: "q5_0", Q5_1: "q5_1", Q8_0: "q8_0",
         Q2_K: "q2_K", Q3_K: "q3_K", Q4_K: "q4_K", Q5_K: "q5_K", Q6_K: "q6_K", IQ2_XXS: "iq2_xxs", IQ2_XS: "iq2_xs",
         IQ3_XXS: "iq3_xxs", IQ1_S: "iq1_s", IQ4_NL: "iq4_nl", IQ3_S: "iq3_s", IQ2_S: "iq2_s", IQ4_XS: "iq4_xs",
         IQ1_M: "iq1_m"}
TYPE_OF = {v: k for k, v in NAMES.items()}


def build():
    """Compiles liboracle.so from the C sources beside this file (make)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


class OrConfig(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("layers", "embd", "heads", "kv_heads", "head_dim", "vocab", "context_length",
                                        "rope_dims")] + \
               [(n, C.c_float) for n in ("rms_eps", "rope_base", "rope_freq_scale")] + \
               [(n, C.c_int) for n in ("rope_neox", "qk_norm", "qk_norm_full", "post_norms", "tied")] + \
               [(n, C.c_float) for n in ("embedding_scale", "residual_scale", "attention_scale", "logit_scale")] + \
               [(n, C.c_int) for n in ("expert_count", "expert_used", "expert_ff", "shared_expert_ff",
                                        "expert_weights_norm")] + \
               [("arch", C.c_char * 32)]


class SynthSpec(C.Structure):
    """or_synth_spec: the benchmark configurations as synthetic decoders (tensor ids shared with the CUDA library)."""
    _fields_ = [("arch", C.c_char * 16)] + \
               [(n, C.c_int) for n in ("layers", "embd", "heads", "kv_heads", "head_dim", "ff", "vocab",
                                        "context_length", "experts", "experts_used", "expert_ff")] + \
               [(n, C.c_float) for n in ("rope_base", "rms_eps", "sigma")] + \
               [(n, C.c_int) for n in ("type_attn", "type_attn_v", "type_ffn", "type_ffn_down", "type_embd",
                                        "type_output")] + \
               [("seed", C.c_uint64)]


def synth_spec_from(spec):
    """Copies a windlass_b200 SynthSpec (same field names) into the oracle's structure."""
    s = SynthSpec()
    for name, _ in SynthSpec._fields_:
        setattr(s, name, getattr(spec, name))
    return s


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        P, I, I64, U64, F, S = C.c_void_p, C.c_int, C.c_int64, C.c_uint64, C.c_float, C.c_char_p
        sig = {
            "or_half_to_float": (F, [C.c_uint16]), "or_float_to_half": (C.c_uint16, [F]),
            "or_layout": (I, [I, C.POINTER(I), C.POINTER(I)]), "or_can_decode": (I, [I]), "or_can_dot": (I, [I]),
            "or_decode_row": (I, [I, P, I64, P]), "or_dot_row": (F, [I, P, P, I]),
            "or_block": (None, [P, I, I, P, I, I, I, P, I]),
            "or_matmul": (I, [I, P, I, I, I64, P, I, P, I, I]),
            "or_rng_init": (None, [P, U64]), "or_rng_next": (U64, [P]), "or_rng_normal": (F, [P]),
            "or_rng_uniform": (C.c_double, [P]), "or_rng_byte": (C.c_uint8, [P]),
            "or_matrix": (I, [P, I, I, I, F, P]),
            "or_write_tiny": (I, [S, S, I, I, I, I, I, I, I, U64]),
            "or_write_tiny_moe": (I, [S, S, I, I, I, I, I, I, I, I, I, I, I, I, C.c_uint32, I, U64]),
            "or_write_tiny_arch": (I, [S, S, I, I, I, I, I, I, I, F, F, F, F, I, I, U64]),
            "or_synth_tensor": (I, [I, U64, C.c_uint32, I64, I64, F, F, P, I]),
            "or_quantize_block": (None, [I, P, P]),
            "or_model_open": (P, [S, I, I, C.c_char_p, I]), "or_model_close": (None, [P]),
            "or_model_config": (I, [P, C.POINTER(OrConfig)]),
            "or_seq_new": (P, [P]), "or_seq_free": (None, [P]), "or_seq_length": (I, [P]),
            "or_seq_truncate": (None, [P, I]),
            "or_forward": (I, [P, P, P, I, I, I, P, C.c_char_p, I]),
            "or_forward_batch": (I, [P, P, P, I, P, C.c_char_p, I]),
            "or_expert_runs": (I64, [P]),
            "or_route": (None, [P, I, I, I, P, P, P]),
            "or_rmsnorm_rows": (None, [P, I, I, P, F, P]),
            "or_argmax": (I, [P, I]),
            "or_sample": (I, [P, I, C.c_double, C.c_double, C.c_double, P]),
            "or_layer": (I, [P, I, P, I, I, P, C.c_char_p, I]),
            "or_default_threads": (I, []),
            "or_synth_gguf": (P, [C.POINTER(SynthSpec), I, I]),
            "or_gguf_save": (I, [P, S]), "or_gguf_close": (None, [P]),
            "or_model_open_gguf": (P, [P, I, I, C.c_char_p, I]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _ptr(a):
    return a.ctypes.data_as(C.c_void_p)


def layout(t):
    b, s = C.c_int(), C.c_int()
    if not lib().or_layout(t, C.byref(b), C.byref(s)):
        raise ValueError(f"unknown type {t}")
    return b.value, s.value


def row_bytes(t, cols):
    b, s = layout(t)
    return cols // b * s


def half_to_float(h):
    return lib().or_half_to_float(h)


def float_to_half(f):
    return lib().or_float_to_half(f)


def decode(t, data, n):
    data = np.ascontiguousarray(np.frombuffer(bytes(data), dtype=np.uint8) if not isinstance(data, np.ndarray) else data)
    out = np.empty(n, dtype=np.float32)
    if lib().or_decode_row(t, _ptr(data), n, _ptr(out)) != 0:
        raise ValueError(f"cannot decode type {t}")
    return out


def dot_row(t, row, x):
    row = np.ascontiguousarray(row, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    return lib().or_dot_row(t, _ptr(row), _ptr(x), x.size)


def matmul(t, w, rows, cols, x, each_token=False, threads=0):
    """Transformer.MatMul / MatMulEach: y[T][rows] for x[T][cols]."""
    w = np.ascontiguousarray(w, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, cols)
    T = x.shape[0]
    y = np.empty((T, rows), dtype=np.float32)
    if lib().or_matmul(t, _ptr(w), rows, cols, row_bytes(t, cols), _ptr(x), T, _ptr(y), int(each_token), threads):
        raise ValueError("matmul failed")
    return y


class Rng:
    """xorshift64* of tests/TinyModels.cs:89-97."""

    def __init__(self, seed):
        self._s = (C.c_uint64 * 1)()
        lib().or_rng_init(self._s, seed)

    def next(self):
        return lib().or_rng_next(self._s)

    def byte(self):
        return lib().or_rng_byte(self._s)

    def uniform(self):
        return lib().or_rng_uniform(self._s)

    def normal(self):
        return lib().or_rng_normal(self._s)

    def normals(self, n):
        return np.array([self.normal() for _ in range(n)], dtype=np.float32)


def matrix(rng, t, rows, cols, rms):
    """TinyModels.Matrix: random block bytes with fitted fp16 scales."""
    out = np.empty(rows * cols // layout(t)[0] * layout(t)[1], dtype=np.uint8)
    if lib().or_matrix(rng._s, t, rows, cols, rms, _ptr(out)):
        raise ValueError("matrix failed")
    return out


def write_tiny(path, arch="llama", type=Q8_0, tied=False, spm=False, rope_freqs=False, layers=2, embd=256, heads=4,
               kv_heads=2, ff=512, seed=1):
    flags = (1 if tied else 0) | (2 if spm else 0) | (4 if rope_freqs else 0)
    if lib().or_write_tiny(path.encode(), arch.encode(), type, flags, layers, embd, heads, kv_heads, ff, seed):
        raise IOError(f"cannot write {path}")
    return path


def write_tiny_moe(path, layout="llama", type=Q8_0, tied=False, layers=2, embd=256, heads=4, kv_heads=2, experts=4,
                   used=2, expert_ff=256, shared_ff=256, dense_ff=256, norm_key=-1, dense_layers=(), dense_twin=False,
                   seed=1):
    mask = 0
    for l in dense_layers:
        mask |= 1 << l
    if lib().or_write_tiny_moe(path.encode(), layout.encode(), type, int(tied), layers, embd, heads, kv_heads, experts,
                               used, expert_ff, shared_ff, dense_ff, norm_key, mask, int(dense_twin), seed):
        raise IOError(f"cannot write {path}")
    return path


def write_tiny_arch(path, arch="granite", type=Q8_0, tied=False, layers=2, embd=256, heads=4, kv_heads=2, ff=512,
                    embedding_scale=0.0, residual_scale=0.0, attention_scale=0.0, logit_scale=0.0, omit_post_ffw=False,
                    short_qnorm=False, seed=1):
    """TinyArchs.Build (tests/TinyArchs.cs): a tiny Granite or OLMo 2 model, or the Llama twin of a Granite one."""
    if lib().or_write_tiny_arch(path.encode(), arch.encode(), type, int(tied), layers, embd, heads, kv_heads, ff,
                                embedding_scale, residual_scale, attention_scale, logit_scale, int(omit_post_ffw),
                                int(short_qnorm), seed):
        raise IOError(f"cannot write {path}")
    return path


def synth_tensor(t, seed, tid, rows, cols, sigma, offset=0.0, threads=0):
    b, s = layout(t)
    out = np.empty(rows * cols // b * s, dtype=np.uint8)
    if lib().or_synth_tensor(t, seed, tid, rows, cols, sigma, offset, _ptr(out), threads):
        raise ValueError("synth_tensor: unsupported type or shape")
    return out


def quantize_block(t, x):
    b, s = layout(t)
    x = np.ascontiguousarray(x, dtype=np.float32)
    assert x.size == b
    out = np.zeros(s, dtype=np.uint8)
    lib().or_quantize_block(t, _ptr(x), _ptr(out))
    return out


def route(logits, k, renorm):
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    sel = np.zeros(k, dtype=np.int32)
    w = np.zeros(k, dtype=np.float32)
    cnt = np.zeros(logits.size, dtype=np.int32)
    lib().or_route(_ptr(logits), logits.size, k, int(renorm), _ptr(sel), _ptr(w), _ptr(cnt))
    return sel, w, cnt


def argmax(logits):
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    return lib().or_argmax(_ptr(logits), logits.size)


def sample(logits, temperature, top_p, draw):
    """Sampler.Sample (Engine.cs:361-380) with the uniform draw passed in: (id, margin), margin the relative distance
    of the draw (and the nucleus limit) from the nearest boundary between two ids around the choice."""
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    m = C.c_double(0.0)
    i = lib().or_sample(_ptr(logits), logits.size, float(temperature), float(top_p), float(draw), C.byref(m))
    return i, m.value


def write_synth(path, spec, threads=0):
    """Writes the synthetic decoder of `spec` (windlass_b200 SynthSpec or SynthSpec) as a GGUF file."""
    s = synth_spec_from(spec)
    g = lib().or_synth_gguf(C.byref(s), 0, threads)
    if not g:
        raise ValueError("unsupported synthetic spec")
    rc = lib().or_gguf_save(g, path.encode())
    lib().or_gguf_close(g)
    if rc:
        raise IOError(f"cannot write {path}")
    return path


class Model:
    """Transformer restated on the CPU: Forward, ForwardBatch, NewSequence, Truncate, Length, ExpertRuns.

    Model(path) opens a GGUF file; Model(synth=spec, build_layers=n) builds the synthetic decoder of `spec` in
    memory (only its first n layers when n > 0)."""

    def __init__(self, path=None, max_context=512, threads=0, synth=None, build_layers=0):
        err = C.create_string_buffer(512)
        if synth is not None:
            s = synth_spec_from(synth)
            g = lib().or_synth_gguf(C.byref(s), build_layers, threads)
            if not g:
                raise ValueError("unsupported synthetic spec")
            self._m = lib().or_model_open_gguf(g, max_context, threads, err, 512)
        else:
            self._m = lib().or_model_open(path.encode(), max_context, threads, err, 512)
        if not self._m:
            raise ValueError(err.value.decode())
        c = OrConfig()
        lib().or_model_config(self._m, C.byref(c))
        self.config = c
        self.vocab = c.vocab

    def close(self):
        if self._m:
            lib().or_model_close(self._m)
            self._m = None

    def __del__(self):
        self.close()

    def new_sequence(self):
        return Sequence(self)

    def forward(self, tokens, pos0=0, all_logits=False, seq=None):
        tokens = np.ascontiguousarray(tokens, dtype=np.int32)
        T = tokens.size
        out = np.empty((T if all_logits else 1) * self.vocab, dtype=np.float32)
        err = C.create_string_buffer(512)
        if lib().or_forward(self._m, seq._s if seq else None, _ptr(tokens), T, pos0, int(all_logits), _ptr(out), err, 512):
            raise ValueError(err.value.decode())
        return out.reshape(-1, self.vocab) if all_logits else out

    def forward_batch(self, seqs, tokens):
        tokens = np.ascontiguousarray(tokens, dtype=np.int32)
        N = tokens.size
        arr = (C.c_void_p * N)(*[s._s for s in seqs])
        out = np.empty(N * self.vocab, dtype=np.float32)
        err = C.create_string_buffer(512)
        if lib().or_forward_batch(self._m, arr, _ptr(tokens), N, _ptr(out), err, 512):
            raise ValueError(err.value.decode())
        return out.reshape(N, self.vocab)

    def layer(self, l, x, pos0=0, seq=None):
        x = np.ascontiguousarray(x, dtype=np.float32)
        err = C.create_string_buffer(512)
        T = x.size // self.config.embd
        if lib().or_layer(self._m, l, _ptr(x), T, pos0, seq._s if seq else None, err, 512):
            raise ValueError(err.value.decode())
        return x

    @property
    def expert_runs(self):
        return lib().or_expert_runs(self._m)


class Sequence:
    def __init__(self, model):
        self._model = model
        self._s = lib().or_seq_new(model._m)

    @property
    def length(self):
        return lib().or_seq_length(self._s)

    def truncate(self, n):
        lib().or_seq_truncate(self._s, n)

    def __del__(self):
        if self._s and self._model._m:
            lib().or_seq_free(self._s)
        self._s = None
