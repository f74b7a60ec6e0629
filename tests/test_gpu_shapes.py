"""Parity with the CPU oracle at the shapes the benchmark runs, through the C ABI.

The fixture-model tests (test_gpu_model.py) use head_dim 64, hidden sizes up to 2048 and short prompts. The
benchmark's kernels are other instantiations: head_dim 128 attention over about a thousand cached positions split
into ranges and merged (k_attn_part<128, 8>, k_attn_combine<16>), the residual + RmsNorm + activation prep at 8192
and 4096 values a row, the two-matrix q+k and gate+up launches at 8192 x 8192 / 28672 x 8192, the Q6_K head over
128256 and 151936 rows, and the Qwen3-MoE per-head QK-norm + RoPE at head_dim 128 with 128 experts top-8. Here each
is compared with the oracle (the reference's Transformer restated in C) on models of the benchmark's own shapes with
fewer layers:

- configs[3] (Llama-3.3-70B shape, one layer): a 1099-token prompt, then greedy decode steps at positions 1099..,
  every step's logits within 1e-3 of their standard deviation with the same top token;
- configs[2] (Llama-3-8B shape, two layers): a 512-token prompt and 32 greedy tokens identical to the oracle's
  (the configs[0] check of the reference's own harness, at the 8B shape);
- configs[4] (Qwen3-MoE shape, two layers): decode at batch 1 and ForwardBatch at batch 8, logits within 1e-3 of
  their standard deviation (the reference's MatchesReference allows 3e-3, tests/MoeTests.cs:82-114) with the same
  top token.

By default a prompt's rows run through the tcgen05 GEMM, whose logits carry the bf16 hi/lo error (2^-16 a product)
and are held to the stated bf16 prefill tolerance, 2e-2 max-abs with the same top token. Decode steps run through
the integer tensor-core matvec (within 1e-4 relative L2 of the reference's fp32 dot). For the decode-step checks the
prompt runs on that matvec too (prefill_path 2), so that the KV cache the steps attend over is at fp32 level, as
the oracle's is; otherwise near-ties among 128256 random logits would flip on the GEMM's rounding, not on an error.
"""
import numpy as np
import pytest

from windlass_b200.transformer import CudaTransformer, llama70b_spec, llama8b_spec, qwen3moe_spec

pytestmark = pytest.mark.gpu


def close(got, want, what, rel=1e-3):
    got = np.asarray(got, dtype=np.float32).reshape(np.shape(want))
    want = np.asarray(want, dtype=np.float32)
    rows_g = got.reshape(-1, want.shape[-1])
    rows_w = want.reshape(-1, want.shape[-1])
    for i, (g, w) in enumerate(zip(rows_g, rows_w)):
        std = float(w.std())
        md = float(np.abs(g - w).max())
        assert md <= rel * std, f"{what} row {i}: max |diff| {md:.3e} vs std {std:.3e}"
        assert int(np.argmax(g)) == int(np.argmax(w)), f"{what} row {i}: top token differs"


def gemm_prompt_close(got, want, what):
    """The stated tolerance of bf16 tensor-core prefill logits: 2e-2 max-abs, the same top token."""
    md = float(np.abs(np.asarray(got) - np.asarray(want)).max())
    assert md <= 2e-2, f"{what}: max |diff| {md:.3e}"
    assert int(np.argmax(got)) == int(np.argmax(want)), f"{what}: top token differs"


def test_70b_shape_layer_decode_over_a_long_prompt(wl, oracle):
    """configs[3] shape: d 8192, 64 query / 8 KV heads of 128, FFN 28672, Q4_K with Q6_K attn_v and head, vocab
    128256. The decode steps attend over 1100-1103 cached positions, which k_attn_part<128, 8> splits into 16 ranges
    per KV head and k_attn_combine<16> merges."""
    O = oracle
    spec = llama70b_spec(layers=1)
    P = 1099
    prompt = np.random.default_rng(70).integers(0, spec.vocab, P).astype(np.int32)
    om = O.Model(synth=spec, build_layers=1, max_context=P + 8)
    want = om.forward(prompt)
    with CudaTransformer(synthetic=spec, max_context=P + 8) as m:
        gemm_prompt_close(m.forward(prompt), want, "70B-shape prompt on the tcgen05 GEMM, last row")
    with CudaTransformer(synthetic=spec, max_context=P + 8, prefill_path=2) as m:
        close(m.forward(prompt), want, "70B-shape prompt on the integer matvec, last row")
        for i in range(4):
            t = int(np.argmax(want))
            got = m.forward([t], pos0=P + i)
            want = om.forward([t], pos0=P + i)
            close(got, want, f"70B-shape decode at position {P + i}")


def test_8b_shape_greedy_tokens_identical(wl, oracle):
    """configs[2] shape (d 4096, 32/8 heads of 128, FFN 14336, vocab 128256), two layers: a 512-token prompt and
    32 greedy tokens, each side choosing its own next token; the sequences are identical."""
    O = oracle
    spec = llama8b_spec()
    spec.layers = 2
    P, N = 512, 32
    prompt = np.random.default_rng(8).integers(0, spec.vocab, P).astype(np.int32)
    om = O.Model(synth=spec, build_layers=2, max_context=P + N + 4)
    lw = om.forward(prompt)
    with CudaTransformer(synthetic=spec, max_context=P + N + 4) as m:
        gemm_prompt_close(m.forward(prompt), lw, "8B-shape prompt on the tcgen05 GEMM, last row")
    with CudaTransformer(synthetic=spec, max_context=P + N + 4, prefill_path=2) as m:
        lg = m.forward(prompt)
        close(lg, lw, "8B-shape prompt on the integer matvec, last row")
        want, got = [], []
        for i in range(N):
            tw, tg = int(np.argmax(lw)), int(np.argmax(lg))
            want.append(tw)
            got.append(tg)
            lw = om.forward([tw], pos0=P + i)
            lg = m.forward([tg], pos0=P + i)
        assert got == want


def test_qwen3moe_shape_decode_b1_and_b8(wl, oracle):
    """configs[4] shape (d 2048, 32/4 heads of 128 with QK-norm, 128 experts top-8 of FFN 768, vocab 151936), two
    layers: decode steps at batch 1, then ForwardBatch steps of 8 sequences with prompts of different lengths."""
    O = oracle
    spec = qwen3moe_spec(layers=2)
    rng = np.random.default_rng(48)
    om = O.Model(synth=spec, build_layers=2, max_context=96)
    prompt = rng.integers(0, spec.vocab, 40).astype(np.int32)
    lw = om.forward(prompt)
    with CudaTransformer(synthetic=spec, max_context=96) as m:
        gemm_prompt_close(m.forward(prompt), lw, "MoE-shape prompt on the tcgen05 GEMM, last row")
    with CudaTransformer(synthetic=spec, max_context=96, prefill_path=2) as m:
        lg = m.forward(prompt)
        close(lg, lw, "MoE-shape prompt on the integer matvec, last row")
        for i in range(3):
            t = int(np.argmax(lw))
            lw, lg = om.forward([t], pos0=40 + i), m.forward([t], pos0=40 + i)
            close(lg, lw, f"MoE-shape decode at position {40 + i}")
        prompts = [rng.integers(0, spec.vocab, n).astype(np.int32) for n in (3, 9, 1, 17, 30, 5, 12, 24)]
        sw = [om.new_sequence() for _ in prompts]
        sg = [m.new_sequence() for _ in prompts]
        for a, b, p in zip(sw, sg, prompts):
            om.forward(p, seq=a)
            m.forward(p, seq=b)
        toks = rng.integers(0, spec.vocab, 8).astype(np.int32)
        for step in range(2):
            bw = om.forward_batch(sw, toks)
            bg = m.forward_batch(sg, toks)
            close(bg, bw, f"MoE-shape ForwardBatch b8 step {step}")
            toks = bw.argmax(axis=1).astype(np.int32)


def test_70b_shape_batch_rows_bit_identical_to_single_runs(wl):
    """ForwardBatch rows equal single-sequence Forward bit for bit (tests/BatchTests.cs:29-94) at the 70B layer's
    shapes, where the decode matvec's launch shape is chosen from the matrix's row tiles: batches of 8, 3 and 2
    sequences (the persistent paired-tile form, the three-MMA form and the packed two-column form of the integer
    matvec against the single column; the single-sequence steps also do RoPE and the KV append inside the attention
    kernel, the batches in k_rope_append)."""
    spec = llama70b_spec(layers=1)
    rng = np.random.default_rng(707)
    prompts = [rng.integers(0, spec.vocab, n).astype(np.int32) for n in (37, 5, 120, 64, 1, 77, 200, 19)]
    with CudaTransformer(synthetic=spec, max_context=256) as m, CudaTransformer(synthetic=spec, max_context=256) as solo:
        seqs = [m.new_sequence() for _ in prompts]
        ref = [solo.new_sequence() for _ in prompts]
        for s, r, p in zip(seqs, ref, prompts):
            m.forward(p, seq=s)
            solo.forward(p, seq=r)
        toks = rng.integers(0, spec.vocab, 8).astype(np.int32)
        for n in (8, 3, 2):
            rows = m.forward_batch(seqs[:n], toks[:n])
            for i in range(n):
                want = solo.forward([int(toks[i])], pos0=ref[i].length, seq=ref[i])
                assert np.array_equal(rows[i].view(np.uint32), want.view(np.uint32)), (n, i)
            toks = rows.argmax(axis=1).astype(np.int32).tolist() + list(toks[n:])
            toks = np.array(toks, dtype=np.int32)
