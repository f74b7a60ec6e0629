"""An independent double-precision forward pass of the tiny Granite and OLMo 2 test models (the Ref class of the
reference's tests/ArchTests.cs:181-251, which writes out llama.cpp's llm_build_granite and llm_build_olmo2), used to
pin the oracle's Granite scales and OLMo 2 post-norms, which the llama.cpp fixtures do not cover:

    granite: x = embd * embedding_scale; per layer x += attn(norm(x)) * residual_scale, x += ffn(norm(x)) *
             residual_scale; scores use attention.scale when set; logits = head(norm(x)) / logit_scale.
    olmo2:   per layer q = norm_full(Wq x), k = norm_full(Wk x) (no pre-norm), NEOX RoPE, attention;
             x += norm(Wo att); x += norm(ffn(x)).

It shares no code with the oracle's forward pass: tensors are decoded by the oracle's dequantizers (pinned by the
llama.cpp fixtures and gguf-py) through naive_moe.Naive's reader, and every step runs in numpy float64, rounding only
K and V to fp16 as the cache does.
"""
import numpy as np

from naive_moe import Naive


class NaiveArch:
    def __init__(self, oracle, path, arch, layers=2, embd=256, heads=4, kv_heads=2, ff=512, tied=False,
                 embedding_scale=0.0, residual_scale=0.0, attention_scale=0.0, logit_scale=0.0):
        self.n = Naive(oracle, path, arch, 0, 0, tied=tied)
        self.arch, self.L, self.E, self.H, self.KV, self.F = arch, layers, embd, heads, kv_heads, ff
        self.tied = tied
        self.es = embedding_scale or 1.0
        self.rs = residual_scale or 1.0
        self.HD = embd // heads
        self.kq = attention_scale or 1.0 / np.sqrt(self.HD)
        self.div = logit_scale or 1.0

    def close(self):
        self.n.close()

    @staticmethod
    def rope(v, off, n, pos, base, neox):
        i = np.arange(n // 2)
        ang = pos * np.power(base, -2.0 * i / n)
        c, s = np.cos(ang), np.sin(ang)
        a, b = (off + i, off + i + n // 2) if neox else (off + 2 * i, off + 2 * i + 1)
        x0, x1 = v[a].copy(), v[b].copy()
        v[a] = x0 * c - x1 * s
        v[b] = x0 * s + x1 * c

    def forward(self, toks):
        n, W = self.n, self.n.W
        olmo = self.arch == "olmo2"
        E, H, KV, HD = self.E, self.H, self.KV, self.HD
        embd = W("token_embd.weight")
        head = embd if self.tied else W("output.weight")
        K = [[] for _ in range(self.L)]
        V = [[] for _ in range(self.L)]
        out = []
        for t, tok in enumerate(toks):
            x = embd[tok] * self.es
            for l in range(self.L):
                p = f"blk.{l}."
                h = x if olmo else n.rms(x, W(p + "attn_norm.weight"))
                q, k, v = W(p + "attn_q.weight") @ h, W(p + "attn_k.weight") @ h, W(p + "attn_v.weight") @ h
                if olmo:
                    q = n.rms(q, W(p + "attn_q_norm.weight"))
                    k = n.rms(k, W(p + "attn_k_norm.weight"))
                for hh in range(H):
                    self.rope(q, hh * HD, HD, t, 500000.0, olmo)
                for hh in range(KV):
                    self.rope(k, hh * HD, HD, t, 500000.0, olmo)
                K[l].append(n.fp16(k))
                V[l].append(n.fp16(v))
                Kl, Vl = np.stack(K[l]), np.stack(V[l])
                att = np.zeros(H * HD)
                for hh in range(H):
                    kvh = hh // (H // KV)
                    sc = Kl[:, kvh * HD:(kvh + 1) * HD] @ q[hh * HD:(hh + 1) * HD] * self.kq
                    e = np.exp(sc - sc.max())
                    att[hh * HD:(hh + 1) * HD] = (e / e.sum()) @ Vl[:, kvh * HD:(kvh + 1) * HD]
                o = W(p + "attn_output.weight") @ att
                if olmo:
                    o = n.rms(o, W(p + "post_attention_norm.weight"))
                x = x + o * self.rs
                h2 = x if olmo else n.rms(x, W(p + "ffn_norm.weight"))
                f = n.swiglu(W(p + "ffn_gate.weight"), W(p + "ffn_up.weight"), W(p + "ffn_down.weight"), h2)
                if olmo:
                    f = n.rms(f, W(p + "post_ffw_norm.weight"))
                x = x + f * self.rs
            out.append(head @ n.rms(x, W("output_norm.weight")) / self.div)
        return np.stack(out)
