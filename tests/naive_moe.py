"""An independent double-precision forward pass of the tiny MoE test models (the Naive model of the reference's
tests/MoeTests.cs:336-528), used to pin the oracle's mixture-of-experts path, which the llama.cpp fixtures do not
cover. Nothing here shares code with the oracle's forward pass: it reads the GGUF tensors through the oracle's file
reader and decodes them with the oracle's dequantizers (which the llama.cpp fixtures and gguf-py pin), then runs
every step in numpy float64, rounding only K and V to fp16 as the cache does.
"""
import ctypes as C

import numpy as np


class Naive:
    def __init__(self, oracle, path, layout, experts, used, norm_key=-1, tied=False, dense_layers=()):
        self.O = oracle
        L = oracle.lib()
        L.or_gguf_open.restype = C.c_void_p
        L.or_gguf_open.argtypes = [C.c_char_p, C.c_char_p, C.c_int]
        L.or_gguf_find.restype = C.c_int
        L.or_gguf_find.argtypes = [C.c_void_p, C.c_char_p]
        L.or_gguf_tensor_info.restype = C.c_int
        L.or_gguf_tensor_info.argtypes = [C.c_void_p, C.c_int, C.POINTER(C.c_int), C.POINTER(C.c_int64),
                                          C.POINTER(C.c_int), C.POINTER(C.c_int64), C.POINTER(C.c_void_p)]
        L.or_gguf_get_int.restype = C.c_int64
        L.or_gguf_get_int.argtypes = [C.c_void_p, C.c_char_p, C.c_int64]
        L.or_gguf_close.argtypes = [C.c_void_p]
        err = C.create_string_buffer(256)
        self.g = L.or_gguf_open(path.encode(), err, 256)
        if not self.g:
            raise IOError(err.value.decode())
        self.L = L
        self.layout, self.experts, self.used = layout, experts, used
        self.tied, self.dense_layers = tied, set(dense_layers)
        self.qwen = layout in ("qwen2moe", "qwen3moe")
        self.renorm = (norm_key == 1) if norm_key >= 0 else layout != "qwen2moe"
        self.cache = {}
        a = layout + "."
        self.layers = int(L.or_gguf_get_int(self.g, (a + "block_count").encode(), 0))
        self.embd = int(L.or_gguf_get_int(self.g, (a + "embedding_length").encode(), 0))
        self.heads = int(L.or_gguf_get_int(self.g, (a + "attention.head_count").encode(), 0))
        self.kv_heads = int(L.or_gguf_get_int(self.g, (a + "attention.head_count_kv").encode(), 0))
        self.expert_ff = int(L.or_gguf_get_int(self.g, (a + "expert_feed_forward_length").encode(), 0))

    def close(self):
        if self.g:
            self.L.or_gguf_close(self.g)
            self.g = None

    def W(self, name):
        """Every element of a tensor decoded to float, rows after rows (experts stacked), as a [rows][cols] array."""
        if name in self.cache:
            return self.cache[name]
        i = self.L.or_gguf_find(self.g, name.encode())
        if i < 0:
            raise KeyError(name)
        t, nd, size, data = C.c_int(), C.c_int(), C.c_int64(), C.c_void_p()
        dims = (C.c_int64 * 4)()
        self.L.or_gguf_tensor_info(self.g, i, C.byref(t), dims, C.byref(nd), C.byref(size), C.byref(data))
        cols = int(dims[0])
        rows = 1
        for k in range(1, nd.value):
            rows *= int(dims[k])
        raw = np.frombuffer(C.string_at(data.value, size.value), dtype=np.uint8)
        w = self.O.decode(t.value, raw, rows * cols).astype(np.float64).reshape(rows, cols)
        self.cache[name] = w
        return w

    @staticmethod
    def rms(x, w):
        scale = 1.0 / np.sqrt(float(np.sum(x * x)) / x.size + 1e-5)
        return x * scale * w.reshape(-1)

    @staticmethod
    def silu(a):
        return a / (1.0 + np.exp(-a))

    def swiglu(self, gate, up, down, h):
        return down @ (self.silu(gate @ h) * (up @ h))

    @staticmethod
    def fp16(v):
        return np.asarray(v, dtype=np.float32).astype(np.float16).astype(np.float64)

    def rope(self, v, pos, n, base):
        i = np.arange(n // 2)
        ang = pos * np.power(base, -2.0 * i / n)
        c, s = np.cos(ang), np.sin(ang)
        a, b = (i, i + n // 2) if self.qwen else (2 * i, 2 * i + 1)
        x0, x1 = v[a].copy(), v[b].copy()
        v[a] = x0 * c - x1 * s
        v[b] = x0 * s + x1 * c

    def moe(self, p, h):
        N, X, E = self.experts, self.expert_ff, self.embd
        logit = self.W(p + "ffn_gate_inp.weight") @ h
        prob = np.exp(logit - logit.max())
        prob /= prob.sum()
        order = sorted(range(N), key=lambda e: (-prob[e], e))[: self.used]
        chosen = sum(prob[e] for e in order)
        gate, up, down = self.W(p + "ffn_gate_exps.weight"), self.W(p + "ffn_up_exps.weight"), self.W(p + "ffn_down_exps.weight")
        y = np.zeros(E)
        for e in order:
            wgt = prob[e] / chosen if self.renorm else prob[e]
            y += wgt * self.swiglu(gate[e * X:(e + 1) * X], up[e * X:(e + 1) * X], down[e * E:(e + 1) * E], h)
        if self.layout == "qwen2moe":
            sg = 1.0 / (1.0 + np.exp(-float((self.W(p + "ffn_gate_inp_shexp.weight") @ h)[0])))
            y += sg * self.swiglu(self.W(p + "ffn_gate_shexp.weight"), self.W(p + "ffn_up_shexp.weight"),
                                  self.W(p + "ffn_down_shexp.weight"), h)
        return y

    def forward(self, toks):
        E, H, KV = self.embd, self.heads, self.kv_heads
        HD = E // H
        base = 1000000.0 if self.qwen else 500000.0
        embd = self.W("token_embd.weight")
        head = embd if self.tied else self.W("output.weight")
        K = [[] for _ in range(self.layers)]
        V = [[] for _ in range(self.layers)]
        out = []
        for t, tok in enumerate(toks):
            x = embd[tok].copy()
            for l in range(self.layers):
                p = f"blk.{l}."
                h = self.rms(x, self.W(p + "attn_norm.weight"))
                q, k, v = self.W(p + "attn_q.weight") @ h, self.W(p + "attn_k.weight") @ h, self.W(p + "attn_v.weight") @ h
                if self.layout == "qwen2moe":
                    q = q + self.W(p + "attn_q.bias").reshape(-1)
                    k = k + self.W(p + "attn_k.bias").reshape(-1)
                    v = v + self.W(p + "attn_v.bias").reshape(-1)
                if self.layout == "qwen3moe":
                    wq, wk = self.W(p + "attn_q_norm.weight"), self.W(p + "attn_k_norm.weight")
                    for hh in range(H):
                        q[hh * HD:(hh + 1) * HD] = self.rms(q[hh * HD:(hh + 1) * HD], wq)
                    for hh in range(KV):
                        k[hh * HD:(hh + 1) * HD] = self.rms(k[hh * HD:(hh + 1) * HD], wk)
                for hh in range(H):
                    seg = q[hh * HD:(hh + 1) * HD]
                    self.rope(seg, t, HD, base)
                    q[hh * HD:(hh + 1) * HD] = seg
                for hh in range(KV):
                    seg = k[hh * HD:(hh + 1) * HD]
                    self.rope(seg, t, HD, base)
                    k[hh * HD:(hh + 1) * HD] = seg
                K[l].append(self.fp16(k))
                V[l].append(self.fp16(v))
                Kl, Vl = np.stack(K[l]), np.stack(V[l])
                att = np.zeros(H * HD)
                for hh in range(H):
                    kvh = hh // (H // KV)
                    sc = Kl[:, kvh * HD:(kvh + 1) * HD] @ q[hh * HD:(hh + 1) * HD] / np.sqrt(HD)
                    e = np.exp(sc - sc.max())
                    att[hh * HD:(hh + 1) * HD] = (e / e.sum()) @ Vl[:, kvh * HD:(kvh + 1) * HD]
                x = x + self.W(p + "attn_output.weight") @ att
                h2 = self.rms(x, self.W(p + "ffn_norm.weight"))
                if l in self.dense_layers:
                    f = self.swiglu(self.W(p + "ffn_gate.weight"), self.W(p + "ffn_up.weight"), self.W(p + "ffn_down.weight"), h2)
                else:
                    f = self.moe(p, h2)
                x = x + f
            out.append(head @ self.rms(x, self.W("output_norm.weight")))
        return np.stack(out)
