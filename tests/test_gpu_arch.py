"""The CUDA forward pass on the Granite and OLMo 2 fixture models (tests/TinyArchs.cs, restated in the oracle's
generator), through the C ABI, mirroring the reference's tests/ArchTests.cs:

- the six ArchTests.Specs models match the oracle (whose own Granite and OLMo 2 paths are pinned to an independent
  float64 model by test_oracle_arch.py) within 1e-3 of the standard deviation, with the same top token at every
  position (MatchesReference allows 3e-3);
- a Granite file with no scale keys gives bit for bit the Llama twin's logits (GraniteWithoutScalesIsLlama);
- each Granite scale changes the logits, and the logit scale divides them exactly (EachScaleMatters);
- streamed and resident weights give identical logits, and token-by-token decoding matches a full pass within 1e-3
  (StreamingAndKvCache);
- OLMo 2 files without post_ffw_norm or with a per-head attn_q_norm are refused with the reference's messages
  (ConfigAndRefusals).
"""
import numpy as np
import pytest

from test_oracle_arch import PROBE, SPECS, spec_id, write
from windlass_b200 import _lib
from windlass_b200.transformer import CudaTransformer

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("s", SPECS, ids=spec_id)
def test_arch_models_match_oracle(wl, oracle, tmp_path, s):
    p = write(oracle, tmp_path, s)
    want = oracle.Model(p).forward(PROBE, all_logits=True)
    for path in (0, 2):         # the default prompt path (tcgen05 GEMM for Q4_K) and the fp32-level matvec
        with CudaTransformer(p, max_context=512, prefill_path=path) as m:
            got = m.forward(PROBE, all_logits=True)
        std = float(want.std())
        md = float(np.abs(got - want).max())
        tol = 2e-2 if path == 0 and s["type"] == 12 else 1e-3 * std
        assert md <= tol, f"prefill path {path}: max |diff| {md:.3e} vs std {std:.3e}"
        assert (got.argmax(axis=1) == want.argmax(axis=1)).all()


def test_granite_without_scales_is_llama(wl, oracle, tmp_path):
    g = oracle.write_tiny_arch(str(tmp_path / "g.gguf"), "granite", oracle.Q4_K)
    l = oracle.write_tiny_arch(str(tmp_path / "l.gguf"), "llama", oracle.Q4_K)
    with CudaTransformer(g) as mg, CudaTransformer(l) as ml:
        a, b = mg.forward(PROBE, all_logits=True), ml.forward(PROBE, all_logits=True)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
        for i in range(3):
            t = int(np.argmax(a[-1] if i == 0 else da))
            da, db = mg.forward([t], pos0=len(PROBE) + i), ml.forward([t], pos0=len(PROBE) + i)
            assert np.array_equal(da.view(np.uint32), db.view(np.uint32))


def test_each_granite_scale_matters(wl, oracle, tmp_path):
    O = oracle
    with CudaTransformer(O.write_tiny_arch(str(tmp_path / "p.gguf"), "granite", O.Q8_0)) as m:
        plain = m.forward(PROBE)
    one = [dict(embedding_scale=3.0), dict(residual_scale=0.3), dict(attention_scale=0.5), dict(logit_scale=4.0)]
    got = []
    for i, kw in enumerate(one):
        with CudaTransformer(O.write_tiny_arch(str(tmp_path / f"s{i}.gguf"), "granite", O.Q8_0, **kw)) as m:
            got.append(m.forward(PROBE))
        assert float(np.abs(got[-1] - plain).max()) > 1e-3, f"{kw} has no effect on the logits"
    assert np.array_equal(got[3], plain * np.float32(1.0 / 4.0)), "logit_scale divides the logits exactly"


@pytest.mark.parametrize("i", [1, 4])
def test_streamed_resident_and_token_by_token(wl, oracle, tmp_path, i):
    p = write(oracle, tmp_path, SPECS[i])
    with CudaTransformer(p, resident=0) as st, CudaTransformer(p, resident=1) as rs:
        a, b = st.forward(PROBE, all_logits=True), rs.forward(PROBE, all_logits=True)
        assert np.array_equal(a, b), "streamed logits differ from resident ones"
    with CudaTransformer(p, prefill_path=2) as m:
        full = m.forward(PROBE)
        step = m.forward(PROBE[:4])
        for j in range(4, len(PROBE)):
            step = m.forward([PROBE[j]], pos0=j)
        assert float(np.abs(full - step).max()) < 1e-3


def test_olmo2_refusals(wl, oracle, tmp_path):
    with pytest.raises(_lib.NotSupportedError, match="post_ffw_norm"):
        CudaTransformer(oracle.write_tiny_arch(str(tmp_path / "nopost.gguf"), "olmo2", omit_post_ffw=True))
    with pytest.raises(_lib.NotSupportedError, match="whole Q and K"):
        CudaTransformer(oracle.write_tiny_arch(str(tmp_path / "shortq.gguf"), "olmo2", short_qnorm=True))
