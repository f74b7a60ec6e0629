"""Writes a synthetic dense llama-shaped model as a GGUF file (version 3), for the file-backed streaming benchmark.

The tensors are the ones wl_open_synthetic builds for the same spec (wl_synth_tensor with the same tensor ids: layer
tensors (layer + 1) << 8 | slot, the embedding, final norm and head 1..3; norm vectors around 1.0), generated on the
GPU and written in GGUF's layout (little endian; dims innermost first; data aligned to 32 bytes), so opening the file
gives the synthetic model's weights. The metadata keys are the ones ModelConfig reads (src/ModelConfig.cs:38-155).
"""
import ctypes as C
import struct

from windlass_b200 import _lib

_BLOCK = {0: (1, 4), 8: (32, 34), 12: (256, 144), 14: (256, 210)}      # F32, Q8_0, Q4_K, Q6_K
_SLOT = {"attn_norm": 1, "attn_q": 2, "attn_k": 3, "attn_v": 4, "attn_output": 5, "ffn_norm": 6, "ffn_gate": 7,
         "ffn_up": 8, "ffn_down": 9}
ALIGN = 32


def _s(b):
    return struct.pack("<Q", len(b)) + b


def _kv(key, value):
    if isinstance(value, str):
        return _s(key.encode()) + struct.pack("<I", 8) + _s(value.encode())
    if isinstance(value, float):
        return _s(key.encode()) + struct.pack("<I", 6) + struct.pack("<f", value)
    return _s(key.encode()) + struct.pack("<I", 4) + struct.pack("<I", value)


def _row_bytes(t, cols):
    b, s = _BLOCK[t]
    if cols % b:
        raise ValueError(f"{cols} columns are not whole blocks of type {t}")
    return cols // b * s


def tensors_of(spec):
    """(name, type, rows, cols, tensor id, vector) for every tensor of a dense llama spec, in file order."""
    E, H, KV, hd = spec.embd, spec.heads, spec.kv_heads, spec.head_dim or spec.embd // spec.heads
    QD, KD, F = H * hd, KV * hd, spec.ff
    out = [("token_embd.weight", spec.type_embd, spec.vocab, E, 1, False)]
    for layer in range(spec.layers):
        b = (layer + 1) << 8
        n = f"blk.{layer}."
        out += [(n + "attn_norm.weight", 0, 1, E, b | _SLOT["attn_norm"], True),
                (n + "attn_q.weight", spec.type_attn, QD, E, b | _SLOT["attn_q"], False),
                (n + "attn_k.weight", spec.type_attn, KD, E, b | _SLOT["attn_k"], False),
                (n + "attn_v.weight", spec.type_attn_v, KD, E, b | _SLOT["attn_v"], False),
                (n + "attn_output.weight", spec.type_attn, E, QD, b | _SLOT["attn_output"], False),
                (n + "ffn_norm.weight", 0, 1, E, b | _SLOT["ffn_norm"], True),
                (n + "ffn_gate.weight", spec.type_ffn, F, E, b | _SLOT["ffn_gate"], False),
                (n + "ffn_up.weight", spec.type_ffn, F, E, b | _SLOT["ffn_up"], False),
                (n + "ffn_down.weight", spec.type_ffn_down, E, F, b | _SLOT["ffn_down"], False)]
    out += [("output_norm.weight", 0, 1, E, 2, True), ("output.weight", spec.type_output, spec.vocab, E, 3, False)]
    return out


def write(path, spec):
    """Writes the GGUF file; returns its size in bytes. Needs a CUDA device (the generator runs there)."""
    import torch
    if spec.arch.decode() != "llama" or spec.experts:
        raise ValueError("the writer covers dense llama specs")
    L = _lib.lib()
    hd = spec.head_dim or spec.embd // spec.heads
    kvs = [("general.architecture", "llama"), ("general.alignment", ALIGN), ("llama.block_count", spec.layers),
           ("llama.embedding_length", spec.embd), ("llama.attention.head_count", spec.heads),
           ("llama.attention.head_count_kv", spec.kv_heads), ("llama.attention.key_length", hd),
           ("llama.rope.dimension_count", hd), ("llama.feed_forward_length", spec.ff),
           ("llama.context_length", spec.context_length or 4096), ("llama.rope.freq_base", float(spec.rope_base)),
           ("llama.attention.layer_norm_rms_epsilon", float(spec.rms_eps or 1e-5))]
    ts = tensors_of(spec)
    infos, off = [], 0
    for name, t, rows, cols, _, vec in ts:
        dims = [cols] if vec else [cols, rows]
        infos.append(_s(name.encode()) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims) +
                     struct.pack("<I", t) + struct.pack("<Q", off))
        off += (rows * _row_bytes(t, cols) + ALIGN - 1) // ALIGN * ALIGN
    head = b"GGUF" + struct.pack("<IQQ", 3, len(ts), len(kvs)) + b"".join(_kv(k, v) for k, v in kvs) + b"".join(infos)
    sigma = spec.sigma if spec.sigma > 0 else 0.02
    stream = torch.cuda.current_stream()
    with open(path, "wb") as f:
        f.write(head)
        f.write(b"\0" * ((-len(head)) % ALIGN))
        for name, t, rows, cols, tid, vec in ts:
            n = rows * _row_bytes(t, cols)
            buf = torch.empty(n, dtype=torch.uint8, device="cuda")
            _lib.check(L.wl_synth_tensor(t, spec.seed, tid, rows, cols, C.c_float(sigma), C.c_float(1.0 if vec else 0.0),
                                         C.c_void_p(buf.data_ptr()), C.c_void_p(stream.cuda_stream)))
            f.write(buf.cpu().numpy().tobytes())
            f.write(b"\0" * ((-n) % ALIGN))
        size = f.tell()
    return size
