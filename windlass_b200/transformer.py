"""Host-side mirror of the reference's Transformer surface (src/Transformer.cs) over libwindlass_cuda.

    CudaTransformer(path)              LayeredBackend.Load -> new Transformer      (src/Engine.cs:55-91)
      .forward(tokens, pos0, all_logits, cancel, on_stage, seq)  Transformer.Forward  (src/Transformer.cs:77-109)
      .forward_batch(seqs, tokens, cancel, on_stage)             Transformer.ForwardBatch (src/Transformer.cs:132-170)
      .forward_argmax / .forward_batch_argmax                     the same, with Sampler.Sample at temperature 0
                                                                  (src/Engine.cs:356-360) done on the device
      .generate_greedy(token, max_new, stop_ids)                  the greedy decode loop (src/Engine.cs:187-203),
                                                                  token ids chained on the device
      .truncate(n), .length                                       Transformer.Truncate / Length (:57, :28)
      .new_sequence() -> Sequence (.length, .truncate(n))         Transformer.NewSequence (:60), Sequence (src/Batch.cs)
      .expert_runs, .bytes_read                                   Transformer.ExpertRuns (:27), LayerStream.BytesRead

Argument errors raise ArgumentError (ArgumentException), unsupported models NotSupportedError
(NotSupportedException), malformed files InvalidDataError (InvalidDataException), a set cancel flag
OperationCanceledError; logits come back as numpy float32 arrays shaped like the reference's return values.
"""
import ctypes as C

import numpy as np

from . import _lib
from ._lib import check, lib


class CancelFlag:
    """The CancellationToken of Forward: set() makes the next stage boundary raise OperationCanceledError."""

    def __init__(self):
        self._v = C.c_int32(0)

    def set(self):
        self._v.value = 1

    @property
    def ptr(self):
        return C.cast(C.byref(self._v), C.c_void_p)


class Sequence:
    """One request's KV cache on the device (src/Batch.cs:13-36)."""

    def __init__(self, model):
        self._model = model
        h = C.c_void_p()
        check(lib().wl_seq_new(model._h, C.byref(h)))
        self._h = h

    @property
    def length(self):
        n = C.c_int32()
        check(lib().wl_seq_length(self._h, C.byref(n)))
        return n.value

    def truncate(self, n):
        check(lib().wl_seq_truncate(self._h, n))

    def close(self):
        if self._h:
            check(lib().wl_seq_free(self._h))
            self._h = None

    def __del__(self):
        try:
            if self._h and self._model._h:
                lib().wl_seq_free(self._h)
        except Exception:
            pass
        self._h = None


class CudaTransformer:
    def __init__(self, path=None, synthetic=None, device=0, max_context=0, max_batch=64, prefill_path=0, resident=-1,
                 use_graphs=1, tp_size=1, tp_rank=0, tp_id=None, tp_nccl_only=0, stream_file=0):
        """tp_size > 1: this process is rank tp_rank of a tensor-parallel group whose ranks all open the same model
        with the same tp_id (windlass_b200.tp) and then make the same calls; each call returns the full logits.
        tp_nccl_only=1 keeps every all-reduce on NCCL instead of the fused peer-memory path. resident=0 streams the
        layers; with stream_file=1 (a GGUF path, one GPU) each stage is read from the file at every use."""
        opt = _lib.options(device=device, max_context=max_context, max_batch=max_batch, prefill_path=prefill_path,
                           resident=resident, use_graphs=use_graphs, tp_size=tp_size, tp_rank=tp_rank, tp_id=tp_id,
                           tp_nccl_only=tp_nccl_only, stream_file=stream_file)
        h = C.c_void_p()
        if synthetic is not None:
            check(lib().wl_open_synthetic(C.byref(synthetic), C.byref(opt), C.byref(h)))
        else:
            check(lib().wl_open(str(path).encode(), C.byref(opt), C.byref(h)))
        self._h = h
        info = _lib.Info()
        check(lib().wl_info_get(self._h, C.byref(info)))
        self.info = info
        self.vocab = info.vocab
        self.max_context = info.max_context

    def close(self):
        if self._h:
            check(lib().wl_close(self._h))
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def new_sequence(self):
        return Sequence(self)

    @property
    def length(self):
        n = C.c_int32()
        check(lib().wl_length(self._h, C.byref(n)))
        return n.value

    def truncate(self, n):
        check(lib().wl_truncate(self._h, n))

    def stats(self):
        s = _lib.Stats()
        check(lib().wl_stats_get(self._h, C.byref(s)))
        return s

    @property
    def expert_runs(self):
        return self.stats().expert_runs

    @property
    def bytes_read(self):
        return self.stats().bytes_h2d

    def forward(self, tokens, pos0=0, all_logits=False, cancel=None, on_stage=None, seq=None, out=None):
        tokens = np.ascontiguousarray(tokens, dtype=np.int32)
        T = int(tokens.size)
        rows = T if all_logits else 1
        if out is None:
            out = np.empty(rows * self.vocab, dtype=np.float32)
        cb = _lib.PROGRESS(lambda d, t, u: on_stage(d, t)) if on_stage else _lib.PROGRESS()
        check(lib().wl_forward(self._h, seq._h if seq is not None else None, tokens.ctypes.data_as(C.c_void_p), T, pos0,
                               int(all_logits), out.ctypes.data_as(C.c_void_p), cancel.ptr if cancel else None, cb,
                               None))
        return out.reshape(T, self.vocab) if all_logits else out

    def forward_argmax(self, tokens, pos0=0, all_rows=False, cancel=None, on_stage=None, seq=None, out=None):
        """forward() with the greedy choice made on the device (Sampler.Sample at temperature 0,
        src/Engine.cs:356-360): the last row's argmax as an int, or every row's as an int32 array (all_rows, the
        guess-ahead check of src/Engine.cs:207-216)."""
        tokens = np.ascontiguousarray(tokens, dtype=np.int32)
        T = int(tokens.size)
        if out is None:
            out = np.empty(T if all_rows else 1, dtype=np.int32)
        cb = _lib.PROGRESS(lambda d, t, u: on_stage(d, t)) if on_stage else _lib.PROGRESS()
        check(lib().wl_forward_argmax(self._h, seq._h if seq is not None else None, tokens.ctypes.data_as(C.c_void_p),
                                      T, pos0, int(all_rows), out.ctypes.data_as(C.c_void_p),
                                      cancel.ptr if cancel else None, cb, None))
        return out if all_rows else int(out[0])

    def forward_batch_argmax(self, seqs, tokens, cancel=None, on_stage=None, out=None):
        """forward_batch() returning each row's argmax (int32 array of N)."""
        tokens = np.ascontiguousarray(tokens, dtype=np.int32)
        N = int(tokens.size)
        arr = (C.c_void_p * max(N, 1))(*[s._h for s in seqs])
        if out is None:
            out = np.empty(max(N, 1), dtype=np.int32)
        cb = _lib.PROGRESS(lambda d, t, u: on_stage(d, t)) if on_stage else _lib.PROGRESS()
        check(lib().wl_forward_batch_argmax(self._h, arr, tokens.ctypes.data_as(C.c_void_p), N,
                                            out.ctypes.data_as(C.c_void_p), cancel.ptr if cancel else None, cb, None))
        return out[:N]

    def forward_sample(self, tokens, temperature, top_p, draw, pos0=0, cancel=None, on_stage=None, seq=None):
        """forward() with Sampler.Sample (src/Engine.cs:361-380) made on the device: the last row's sampled id.
        draw is the caller's uniform double in [0, 1) (rng.NextDouble(), drawn only at temperature > 0)."""
        tokens = np.ascontiguousarray(tokens, dtype=np.int32)
        out = np.empty(1, dtype=np.int32)
        cb = _lib.PROGRESS(lambda d, t, u: on_stage(d, t)) if on_stage else _lib.PROGRESS()
        check(lib().wl_forward_sample(self._h, seq._h if seq is not None else None, tokens.ctypes.data_as(C.c_void_p),
                                      int(tokens.size), pos0, float(temperature), float(top_p), float(draw),
                                      out.ctypes.data_as(C.c_void_p), cancel.ptr if cancel else None, cb, None))
        return int(out[0])

    def forward_batch_sample(self, seqs, tokens, temperature, top_p, draws, cancel=None, on_stage=None):
        """forward_batch() returning each row sampled on the device with its own temperature, top_p and draw
        (arrays of N, or scalars for every row): an int32 array of N ids."""
        tokens = np.ascontiguousarray(tokens, dtype=np.int32)
        N = int(tokens.size)
        arr = (C.c_void_p * max(N, 1))(*[s._h for s in seqs])
        t, p, d = (np.ascontiguousarray(np.broadcast_to(np.asarray(v, dtype=np.float64), (max(N, 1),)))
                   for v in (temperature, top_p, draws))
        out = np.empty(max(N, 1), dtype=np.int32)
        cb = _lib.PROGRESS(lambda d_, t_, u: on_stage(d_, t_)) if on_stage else _lib.PROGRESS()
        check(lib().wl_forward_batch_sample(self._h, arr, tokens.ctypes.data_as(C.c_void_p), N,
                                            t.ctypes.data_as(C.c_void_p), p.ctypes.data_as(C.c_void_p),
                                            d.ctypes.data_as(C.c_void_p), out.ctypes.data_as(C.c_void_p),
                                            cancel.ptr if cancel else None, cb, None))
        return out[:N]

    def forward_mixed(self, seqs, token_lists, cancel=None, on_stage=None, argmax=False):
        """One pass over several sequences' new tokens (a decode step that prompts join): sequence i takes
        token_lists[i]; returns each sequence's last-row logits ([N][vocab]), or its greedy id (argmax=True)."""
        N = len(seqs)
        counts = np.array([len(t) for t in token_lists], dtype=np.int32)
        toks = np.ascontiguousarray(np.concatenate([np.asarray(t, dtype=np.int32) for t in token_lists]) if N else
                                    np.zeros(0, dtype=np.int32), dtype=np.int32)
        arr = (C.c_void_p * max(N, 1))(*[s._h for s in seqs])
        cb = _lib.PROGRESS(lambda d, t, u: on_stage(d, t)) if on_stage else _lib.PROGRESS()
        if argmax:
            ids = np.empty(max(N, 1), dtype=np.int32)
            check(lib().wl_forward_mixed(self._h, arr, counts.ctypes.data_as(C.c_void_p), N,
                                         toks.ctypes.data_as(C.c_void_p), None, ids.ctypes.data_as(C.c_void_p),
                                         cancel.ptr if cancel else None, cb, None))
            return ids[:N]
        out = np.empty(max(N, 1) * self.vocab, dtype=np.float32)
        check(lib().wl_forward_mixed(self._h, arr, counts.ctypes.data_as(C.c_void_p), N, toks.ctypes.data_as(C.c_void_p),
                                     out.ctypes.data_as(C.c_void_p), None, cancel.ptr if cancel else None, cb, None))
        return out[: N * self.vocab].reshape(N, self.vocab)

    def generate_greedy(self, token, max_new, stop_ids=(), chunk=0, cancel=None, seq=None):
        """Greedy decode chained on the device (the loop of src/Engine.cs:187-203 at temperature 0): forwards
        `token`, then each produced id, at the sequence's next positions; returns the produced ids (int32 array), which
        end at the first stop id or after max_new. The sequence grows by their count."""
        out = np.empty(max(int(max_new), 1), dtype=np.int32)
        stop = np.ascontiguousarray(list(stop_ids), dtype=np.int32)
        n = C.c_int32()
        check(lib().wl_generate_greedy(self._h, seq._h if seq is not None else None, int(token), int(max_new),
                                       stop.ctypes.data_as(C.c_void_p) if stop.size else None, int(stop.size),
                                       int(chunk), out.ctypes.data_as(C.c_void_p), C.byref(n),
                                       cancel.ptr if cancel else None))
        return out[:n.value].copy()

    def bench_decode(self, seqs, steps):
        """Device milliseconds of `steps` device-resident decode steps of `seqs` (no host copies)."""
        arr = (C.c_void_p * len(seqs))(*[s._h for s in seqs])
        ms = C.c_double()
        check(lib().wl_bench_decode(self._h, arr, len(seqs), steps, C.byref(ms)))
        return ms.value

    def bench_matvecs(self, T, steps):
        """(device ms, bytes per step) of the step's Q4_K matvec launches replayed alone (wl_bench_matvecs)."""
        ms, by = C.c_double(), C.c_double()
        check(lib().wl_bench_matvecs(self._h, int(T), int(steps), C.byref(ms), C.byref(by)))
        return ms.value, by.value

    def profile(self, on):
        check(lib().wl_profile(self._h, int(on)))

    def profile_get(self, type_id):
        e = _lib.ProfileEntry()
        check(lib().wl_profile_get(self._h, type_id, C.byref(e)))
        return e

    def forward_batch(self, seqs, tokens, cancel=None, on_stage=None, out=None):
        tokens = np.ascontiguousarray(tokens, dtype=np.int32)
        N = int(tokens.size)
        arr = (C.c_void_p * max(N, 1))(*[s._h for s in seqs])
        if out is None:
            out = np.empty(N * self.vocab, dtype=np.float32)
        cb = _lib.PROGRESS(lambda d, t, u: on_stage(d, t)) if on_stage else _lib.PROGRESS()
        check(lib().wl_forward_batch(self._h, arr, tokens.ctypes.data_as(C.c_void_p), N,
                                     out.ctypes.data_as(C.c_void_p), cancel.ptr if cancel else None, cb, None))
        return out.reshape(N, self.vocab)


def synth_spec(arch="llama", layers=4, embd=512, heads=8, kv_heads=8, head_dim=0, ff=1408, vocab=4096,
               context_length=4096, experts=0, experts_used=0, expert_ff=0, rope_base=10000.0, rms_eps=1e-5,
               sigma=0.02, type_attn=12, type_attn_v=12, type_ffn=12, type_ffn_down=12, type_embd=14, type_output=14,
               seed=0):
    s = _lib.SynthSpec()
    s.arch = arch.encode()
    for k, v in dict(layers=layers, embd=embd, heads=heads, kv_heads=kv_heads, head_dim=head_dim, ff=ff, vocab=vocab,
                     context_length=context_length, experts=experts, experts_used=experts_used, expert_ff=expert_ff,
                     rope_base=rope_base, rms_eps=rms_eps, sigma=sigma, type_attn=type_attn, type_attn_v=type_attn_v,
                     type_ffn=type_ffn, type_ffn_down=type_ffn_down, type_embd=type_embd, type_output=type_output,
                     seed=seed).items():
        setattr(s, k, v)
    return s


# The benchmark configurations, as synthetic specs.
def config0_spec():
    """tiny llama, 4 layers, d512, 8/8 heads, hd64, FFN 1408 (ffn_down Q8_0: 1408 is not a multiple of
    256), vocab 4096, eps 1e-5, theta 1e4, attn/FFN Q4_K, token_embd/output Q6_K, seed 0."""
    return synth_spec("llama", 4, 512, 8, 8, 64, 1408, 4096, 4096, rope_base=10000.0, type_ffn_down=8, seed=0)


def llama8b_spec(seed=0):
    """Llama-3-8B shape, Q4_K_M mix (Q4_K attn/FFN, Q6_K attn_v/output)."""
    return synth_spec("llama", 32, 4096, 32, 8, 128, 14336, 128256, 8192, rope_base=500000.0, type_attn_v=14,
                      type_embd=12, seed=seed)


def llama70b_spec(seed=0, layers=80):
    """Llama-3.3-70B shape, Q4_K_M mix (Q4_K attn/FFN, Q6_K attn_v/output)."""
    return synth_spec("llama", layers, 8192, 64, 8, 128, 28672, 128256, 8192, rope_base=500000.0, type_attn_v=14,
                      type_embd=12, seed=seed)


def qwen3moe_spec(seed=0, layers=48):
    """Qwen3-MoE shape, 128 experts top-8, expert FFN 768, QK-norm, Q4_K experts, Q6_K output."""
    return synth_spec("qwen3moe", layers, 2048, 32, 4, 128, 0, 151936, 8192, experts=128, experts_used=8,
                      expert_ff=768, rope_base=1000000.0, rms_eps=1e-6, type_attn_v=14, type_embd=12, seed=seed)
