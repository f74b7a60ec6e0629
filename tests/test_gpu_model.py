"""Model-level parity of the CUDA forward pass with the CPU oracle (the reference's Transformer restated), through
the C ABI, mirroring the reference's engine tests:

- logits of the 18 StandardSpecs fixture models and the I-quant models match the oracle (tests/Tests.cs:250-278);
- greedy decode of 32 tokens after a 32-token prompt gives the oracle's token sequence, from the GGUF
  file and from the on-device synthetic generator alike;
- token-by-token decoding and Truncate match a full pass (tests/Tests.cs:323-346);
- ForwardBatch rows are bit-identical to single runs (tests/BatchTests.cs:29-94);
- MoE layouts match the oracle and only the chosen experts run (tests/MoeTests.cs:82-181);
- cancel, progress and argument errors behave like Transformer.Forward (src/Transformer.cs:83-109).
"""
import numpy as np
import pytest

from windlass_b200 import _lib
from windlass_b200.transformer import CudaTransformer, CancelFlag, config0_spec

pytestmark = pytest.mark.gpu

PROBE = [1, 10, 50, 100, 200, 257, 290, 5, 7, 99, 33, 72]


def standard_specs(O):
    specs = [("llama", t, {}) for t in (O.F32, O.F16, O.BF16, O.Q4_0, O.Q4_1, O.Q5_0, O.Q5_1, O.Q8_0, O.Q2_K, O.Q3_K,
                                         O.Q4_K, O.Q5_K, O.Q6_K)]
    specs += [("qwen2", O.Q8_0, {}), ("qwen3", O.Q4_K, {}), ("qwen2", O.Q6_K, {"tied": True}),
              ("llama", O.Q8_0, {"spm": True}), ("llama", O.F16, {"rope_freqs": True})]
    specs += [("llama", t, {}) for t in (O.IQ4_NL, O.IQ4_XS, O.IQ3_XXS, O.IQ3_S, O.IQ2_XXS, O.IQ2_XS, O.IQ2_S,
                                          O.IQ1_S, O.IQ1_M)]
    return specs


def compare(got, want, what, rel=1e-3):
    got = np.asarray(got).reshape(want.shape)
    std = float(want.std())
    md = float(np.abs(got - want).max())
    assert md <= rel * std, f"{what}: max |diff| {md:.3e} vs std {std:.3e}"
    if want.ndim == 2:
        assert (got.argmax(axis=1) == want.argmax(axis=1)).all(), f"{what}: argmax differs"


def test_fixture_models_match_oracle(wl, oracle, tmp_path):
    O = oracle
    for arch, t, kw in standard_specs(O):
        p = O.write_tiny(str(tmp_path / f"{arch}-{t}-{len(kw)}.gguf"), arch=arch, type=t, **kw)
        want = O.Model(p).forward(PROBE, all_logits=True)
        with CudaTransformer(p, max_context=512) as m:
            got = m.forward(PROBE, all_logits=True)
            compare(got, want, f"{arch}-{O.NAMES[t]}{kw}")
            last = m.forward(PROBE[:5], all_logits=False)
            compare(last, O.Model(p).forward(PROBE[:5]), f"{arch}-{O.NAMES[t]} last row")


def greedy(model_forward, prompt, steps):
    logits = model_forward(prompt, 0)
    toks = []
    for i in range(steps):
        nt = int(np.argmax(logits))          # Sampler greedy: first index of the largest logit (src/Engine.cs:356-360)
        toks.append(nt)
        logits = model_forward([nt], len(prompt) + i)
    return toks


def test_config0_greedy_tokens_identical(wl, oracle, tmp_path):
    """32 uniform random prompt ids, greedy decode 32 tokens, batch 1; token sequences identical."""
    O = oracle
    spec = config0_spec()
    p = O.write_synth(str(tmp_path / "config0.gguf"), spec)
    prompt = np.random.default_rng(0).integers(0, 4096, 32).astype(np.int32)
    om = O.Model(p, max_context=128)
    want = greedy(lambda t, p0: om.forward(t, pos0=p0), prompt, 32)
    with CudaTransformer(p, max_context=128) as m:
        got = greedy(lambda t, p0: m.forward(t, pos0=p0), prompt, 32)
    assert got == want
    with CudaTransformer(synthetic=spec, max_context=128) as ms, CudaTransformer(p, max_context=128) as mf:
        a = ms.forward(prompt, all_logits=True)
        b = mf.forward(prompt, all_logits=True)
        assert np.array_equal(a, b), "the on-device generator and the GGUF file give different weights"
        compare(a, O.Model(p, max_context=128).forward(prompt, all_logits=True), "config0 prefill")


@pytest.mark.parametrize("prefill_path,tol", [(2, 1e-3), (0, 2e-2)])
def test_kv_cache_stepwise_and_truncate(wl, oracle, tmp_path, prefill_path, tol):
    """tests/Tests.cs:323-346: a 12-token pass equals 4 + 8 single-token passes, and Truncate then a 6-token pass, within
    1e-3 of each other, when the prompt rows run on the fp32-level integer tensor-core matvec (prefill_path 2). With
    the default prefill path the prompt's Q4_K/Q6_K rows run on the bf16 tcgen05 GEMM, whose stated logit tolerance is
    2e-2 max-abs."""
    O = oracle
    for arch, t, kw in (("llama", O.Q8_0, {"rope_freqs": True}), ("qwen2", O.Q6_K, {"tied": True}),
                        ("llama", O.IQ4_XS, {})):
        p = O.write_tiny(str(tmp_path / f"kv-{arch}-{t}.gguf"), arch=arch, type=t, **kw)
        with CudaTransformer(p, prefill_path=prefill_path) as m:
            full = m.forward(PROBE)
            step = m.forward(PROBE[:4])
            for i in range(4, len(PROBE)):
                step = m.forward([PROBE[i]], pos0=i)
            assert np.abs(full - step).max() < tol, (arch, t, float(np.abs(full - step).max()))
            assert m.length == len(PROBE)
            m.truncate(6)
            assert m.length == 6
            again = m.forward(PROBE[6:], pos0=6)
            assert np.abs(full - again).max() < tol, (arch, t, float(np.abs(full - again).max()))


def test_batch_rows_bit_identical_to_single_runs(wl, oracle, tmp_path):
    O = oracle
    p = O.write_tiny(str(tmp_path / "batch.gguf"), arch="qwen3", type=O.Q4_K)
    prompts = [[1, 10, 50], [100, 200, 257, 290, 5], [7], [99, 33, 72, 1, 10, 50, 100, 200, 257, 290]]
    with CudaTransformer(p) as m, CudaTransformer(p) as solo:
        seqs = [m.new_sequence() for _ in prompts]
        ref = [solo.new_sequence() for _ in prompts]
        for s, r, pr in zip(seqs, ref, prompts):
            m.forward(pr, seq=s)
            solo.forward(pr, seq=r)
        toks = [5, 7, 9, 11]
        for step in range(3):
            rows = m.forward_batch(seqs, toks)
            for i in range(len(prompts)):
                want = solo.forward([toks[i]], pos0=ref[i].length, seq=ref[i])
                assert np.array_equal(rows[i].view(np.uint32), want.view(np.uint32)), (step, i)
            toks = [int(np.argmax(r)) for r in rows]
        # a sequence leaves the batch and the others continue unchanged
        rows = m.forward_batch(seqs[1:3], toks[1:3])
        for i in (1, 2):
            want = solo.forward([toks[i]], pos0=ref[i].length, seq=ref[i])
            assert np.array_equal(rows[i - 1], want)
        assert [s.length for s in seqs] == [len(prompts[0]) + 3, len(prompts[1]) + 4, len(prompts[2]) + 4,
                                            len(prompts[3]) + 3]
        with pytest.raises(_lib.ArgumentError):
            m.forward_batch([seqs[0], seqs[0]], [1, 2])


MOE_SPECS = [
    dict(layout="llama", type=0, experts=4, used=2),
    dict(layout="mixtral", type=8, experts=8, used=2),
    dict(layout="llama", type=6, experts=4, used=3, norm_key=0),
    dict(layout="qwen2moe", type=12, experts=8, used=2),
    dict(layout="qwen2moe", type=14, experts=4, used=2, norm_key=1, tied=True),
    dict(layout="qwen3moe", type=12, experts=8, used=3, layers=3, dense_layers=(1,)),
    dict(layout="qwen3moe", type=11, experts=4, used=2, norm_key=0),
    dict(layout="qwen3moe", type=1, experts=4, used=4),
]


@pytest.mark.parametrize("spec", MOE_SPECS, ids=lambda s: f"{s['layout']}-t{s['type']}-e{s['experts']}k{s['used']}")
def test_moe_models_match_oracle(wl, oracle, tmp_path, spec):
    O = oracle
    p = O.write_tiny_moe(str(tmp_path / "moe.gguf"), **spec)
    want = O.Model(p).forward(PROBE, all_logits=True)
    with CudaTransformer(p) as m:
        compare(m.forward(PROBE, all_logits=True), want, str(spec))


def test_only_chosen_experts_run(wl, oracle, tmp_path):
    O = oracle
    p = O.write_tiny_moe(str(tmp_path / "moe8.gguf"), layout="qwen3moe", type=O.Q4_K, experts=8, used=2, layers=2)
    with CudaTransformer(p) as m:
        m.forward([10])
        assert m.expert_runs == 2 * 2
    with CudaTransformer(p) as m:
        m.forward(PROBE)
        assert 4 <= m.expert_runs <= 16


def test_cancel_progress_and_argument_errors(wl, oracle, tmp_path):
    O = oracle
    p = O.write_tiny(str(tmp_path / "err.gguf"), type=O.Q8_0)
    with CudaTransformer(p, max_context=64) as m:
        seen = []
        m.forward(PROBE, on_stage=lambda d, t: seen.append((d, t)))
        assert seen == [(i, 3) for i in range(1, 4)]
        flag = CancelFlag()
        flag.set()
        with pytest.raises(_lib.OperationCanceledError):
            m.forward([1, 2, 3], pos0=4, cancel=flag)
        assert m.length == 4                        # the sequence keeps positions before pos0
        with pytest.raises(_lib.ArgumentError, match="pos0 is past"):
            m.forward([1], pos0=9)
        with pytest.raises(_lib.ArgumentError, match="positions; the context is 64"):
            m.forward(list(range(61)), pos0=4)
        with pytest.raises(_lib.ArgumentError, match="outside the vocabulary"):
            m.forward([m.vocab])
        with pytest.raises(_lib.ArgumentError, match="No tokens"):
            m.forward([])


def test_graph_replays_equal_eager_steps(wl):
    """Decode steps replayed from captured CUDA graphs (the default, wl_options.use_graphs = 1) return bit for bit the
    logits of the same steps launched one kernel at a time, for Forward and ForwardBatch."""
    from windlass_b200.transformer import synth_spec
    spec = synth_spec("llama", 2, 2048, 32, 8, 64, 4096, 8192, rope_base=500000.0, type_attn_v=14, type_embd=12, seed=7)
    prompt = np.random.default_rng(1).integers(0, spec.vocab, 20).astype(np.int32)
    with CudaTransformer(synthetic=spec, max_context=128, use_graphs=1) as g, \
            CudaTransformer(synthetic=spec, max_context=128, use_graphs=0) as e:
        lg, le = g.forward(prompt), e.forward(prompt)
        assert np.array_equal(lg, le)
        launches0 = g.stats().kernel_launches
        for i in range(6):
            t = int(np.argmax(le))
            lg, le = g.forward([t], pos0=len(prompt) + i), e.forward([t], pos0=len(prompt) + i)
            assert np.array_equal(lg, le), f"graph step {i} differs from the eager step"
        assert g.stats().kernel_launches > launches0
        sg = [g.new_sequence() for _ in range(3)]
        se = [e.new_sequence() for _ in range(3)]
        for k in range(3):
            g.forward(prompt[: 5 + k], seq=sg[k])
            e.forward(prompt[: 5 + k], seq=se[k])
        for step in range(3):
            bg = g.forward_batch(sg, [3 + step, 4, 5])
            be = e.forward_batch(se, [3 + step, 4, 5])
            assert np.array_equal(bg, be), f"graph batch step {step} differs from the eager step"


@pytest.mark.parametrize("case", ["config0", "gqa-file", "gqa-read-file", "moe-read-file", "moe"])
def test_streamed_layers_match_resident(wl, oracle, tmp_path, case):
    """StreamingIsExact (tests/Tests.cs:305-321): weights streamed through two device slots (wl_options.resident = 0,
    LayerStream), from pinned host memory or read from the GGUF file at every use (stream_file = 1, the
    "read-file" cases), give bit-identical logits to resident weights for prompts, decode steps and ForwardBatch, and
    every pass copies at least every layer's bytes."""
    from windlass_b200.transformer import synth_spec
    read_file = case.endswith("read-file")
    if case == "config0":
        spec, src = config0_spec(), None
    elif case.startswith("gqa"):
        spec = synth_spec("llama", 3, 2048, 32, 8, 64, 4096, 8192, rope_base=500000.0, type_attn_v=14, type_embd=12,
                          seed=5)
        src = oracle.write_synth(str(tmp_path / "gqa.gguf"), spec)
    else:
        spec = synth_spec("qwen3moe", 2, 512, 8, 4, 64, 0, 4096, experts=8, experts_used=2, expert_ff=256,
                          rope_base=1000000.0, type_attn_v=14, type_embd=12, seed=3)
        src = oracle.write_synth(str(tmp_path / "moe.gguf"), spec) if read_file else None

    def open_model(resident):
        if src:
            return CudaTransformer(src, max_context=128, resident=resident, stream_file=int(read_file and resident == 0))
        return CudaTransformer(synthetic=spec, max_context=128, resident=resident)

    prompt = np.random.default_rng(2).integers(0, spec.vocab, 24).astype(np.int32)
    with open_model(0) as st, open_model(1) as rs:
        a, b = st.forward(prompt, all_logits=True), rs.forward(prompt, all_logits=True)
        assert np.array_equal(a, b), "streamed prompt logits differ from resident ones"
        layer_bytes = st.info.weight_bytes
        for i in range(4):
            t = int(np.argmax(b[-1] if i == 0 else lb))
            h0 = st.bytes_read
            la, lb = st.forward([t], pos0=len(prompt) + i), rs.forward([t], pos0=len(prompt) + i)
            assert np.array_equal(la, lb), f"streamed decode step {i} differs"
            assert st.bytes_read - h0 >= 0.5 * layer_bytes, "a streamed pass must copy the layers' weights"
        sa, sb = [st.new_sequence() for _ in range(2)], [rs.new_sequence() for _ in range(2)]
        for k in range(2):
            st.forward(prompt[: 6 + k], seq=sa[k])
            rs.forward(prompt[: 6 + k], seq=sb[k])
        assert np.array_equal(st.forward_batch(sa, [7, 9]), rs.forward_batch(sb, [7, 9]))


def test_repeated_prompts_are_deterministic(wl):
    """The same prompt run again and again on one model (the tcgen05 GEMM prefill, kernels overlapping through
    programmatic dependent launch) gives the same bits every time, and stays within the stated tolerance of bf16
    tensor-core prefill logits (2e-2 max-abs) of the fp32-level integer-matvec prefill, with the same argmax rows
    (each matrix product is within 1e-4 relative L2: test_gpu_kernels; two layers and the head compound it)."""
    from windlass_b200.transformer import synth_spec
    spec = synth_spec("llama", 2, 2048, 32, 8, 64, 4096, 8192, rope_base=500000.0, type_attn_v=14, type_embd=12, seed=7)
    prompt = np.random.default_rng(1).integers(0, spec.vocab, 20).astype(np.int32)
    with CudaTransformer(synthetic=spec, max_context=128) as m, \
            CudaTransformer(synthetic=spec, max_context=128, prefill_path=2) as ref:
        want = ref.forward(prompt, all_logits=True)
        outs = [m.forward(prompt, all_logits=True).copy() for _ in range(4)]
        for i, o in enumerate(outs):
            assert np.array_equal(o, outs[0]), f"prefill {i} differs from the first"
        rel = float(np.linalg.norm(outs[0] - want) / np.linalg.norm(want))
        assert rel <= 1e-3, rel
        assert float(np.abs(outs[0] - want).max()) <= 2e-2
        assert (outs[0].argmax(axis=1) == want.argmax(axis=1)).all()


def test_moe_decode_steps_on_the_device(wl):
    """Decode steps of a mixture-of-experts model keep the router's choice on the device (one grouped matvec launch
    per projection over every token-expert pair, CUDA graphs allowed). Each step's logits are bit for bit those of
    the same positions in a prompt run through the host-grouped path (prefill_path 2: every column as if alone), for
    single steps and ForwardBatch, and ExpertRuns counts the distinct experts each step runs."""
    from windlass_b200.transformer import synth_spec
    spec = synth_spec("qwen3moe", 2, 512, 8, 4, 64, 0, 4096, experts=16, experts_used=4, expert_ff=256,
                      rope_base=1000000.0, type_attn_v=14, type_embd=12, seed=11)
    toks = np.random.default_rng(4).integers(0, spec.vocab, 12).astype(np.int32)
    with CudaTransformer(synthetic=spec, max_context=64, prefill_path=2) as host_path, \
            CudaTransformer(synthetic=spec, max_context=64) as dev_path:
        want = host_path.forward(toks, all_logits=True)
        for i, t in enumerate(toks):
            before = dev_path.expert_runs
            got = dev_path.forward([int(t)], pos0=i)
            assert np.array_equal(got, want[i]), f"decode step {i} differs from the host-grouped path"
            assert dev_path.expert_runs - before == 2 * 4          # 2 layers x 4 distinct experts for one token
        s = [dev_path.new_sequence() for _ in range(3)]
        for k in range(3):
            dev_path.forward(toks[: 4 + k], seq=s[k])
        batch = dev_path.forward_batch(s, [toks[4], toks[5], toks[6]])
        ref = host_path.new_sequence()
        for k in range(3):
            ref.truncate(0)
            row = host_path.forward(np.append(toks[: 4 + k], toks[4 + k]).astype(np.int32), seq=ref, all_logits=True)[-1]
            assert np.array_equal(batch[k], row), f"batch row {k} differs"
