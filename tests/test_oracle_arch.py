"""The oracle's Granite and OLMo 2 paths against the reference's own checks (tests/ArchTests.cs), on the CPU:

- MatchesReference (:66-98): the six tiny models of TinyArchs (tests/TinyArchs.cs, restated in the oracle's
  generator) against an independent float64 forward pass (tests/naive_arch.py, the reference's Ref), within 3e-3 of
  the standard deviation with the same top token at every position;
- GraniteWithoutScalesIsLlama (:100-105): a Granite file with no scale keys gives exactly the Llama twin's logits;
- EachScaleMatters (:107-126): each scale changes the logits, and the logit scale divides them exactly;
- token-by-token decoding matches a full pass within 1e-3 (StreamingAndKvCache, :128-150);
- ConfigAndRefusals (:152-165): the scales are read, and OLMo 2 files without post_ffw_norm or with a per-head
  attn_q_norm are refused with the reference's messages.
"""
import numpy as np
import pytest

from naive_arch import NaiveArch

PROBE = [1, 10, 50, 100, 200, 257, 290, 5, 7, 99, 33, 72]

# ArchTests.Specs (tests/ArchTests.cs:56-64)
SPECS = [
    dict(arch="granite", type=0, embedding_scale=12.0, residual_scale=0.22, attention_scale=0.0156, logit_scale=8.0),
    dict(arch="granite", type=12, tied=True, embedding_scale=12.0, residual_scale=0.22, attention_scale=0.0156,
         logit_scale=8.0),
    dict(arch="granite", type=8, residual_scale=0.5),
    dict(arch="olmo2", type=0),
    dict(arch="olmo2", type=8, layers=3),
    dict(arch="olmo2", type=14, tied=True),
]


def spec_id(s):
    return "-".join(f"{k}={v}" for k, v in s.items())


def write(O, tmp_path, s):
    kw = dict(s)
    arch = kw.pop("arch")
    return O.write_tiny_arch(str(tmp_path / (spec_id(s).replace("=", "") + ".gguf")), arch, **kw)


def naive(O, path, s):
    kw = {k: v for k, v in s.items() if k not in ("type",)}
    return NaiveArch(O, path, **kw)


@pytest.mark.parametrize("s", SPECS, ids=spec_id)
def test_arch_models_match_float64_reference(oracle, tmp_path, s):
    O = oracle
    p = write(O, tmp_path, s)
    got = O.Model(p).forward(PROBE, all_logits=True)
    ref = naive(O, p, s)
    want = ref.forward(PROBE)
    ref.close()
    std = float(want[-1].std())
    md = float(np.abs(got - want).max())
    assert md <= 3e-3 * std, f"max diff {md} vs std {std}"
    assert (got.argmax(axis=1) == want.argmax(axis=1)).all()


def test_granite_without_scales_is_llama(oracle, tmp_path):
    O = oracle
    g = O.write_tiny_arch(str(tmp_path / "g.gguf"), "granite", O.Q4_K)
    l = O.write_tiny_arch(str(tmp_path / "l.gguf"), "llama", O.Q4_K)
    a = O.Model(g).forward(PROBE, all_logits=True)
    b = O.Model(l).forward(PROBE, all_logits=True)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_each_granite_scale_matters(oracle, tmp_path):
    O = oracle
    plain = O.Model(O.write_tiny_arch(str(tmp_path / "p.gguf"), "granite", O.Q8_0)).forward(PROBE)
    one = [dict(embedding_scale=3.0), dict(residual_scale=0.3), dict(attention_scale=0.5), dict(logit_scale=4.0)]
    for i, kw in enumerate(one):
        got = O.Model(O.write_tiny_arch(str(tmp_path / f"s{i}.gguf"), "granite", O.Q8_0, **kw)).forward(PROBE)
        assert float(np.abs(got - plain).max()) > 1e-3, f"{kw} has no effect on the logits"
    scaled = O.Model(str(tmp_path / "s3.gguf")).forward(PROBE)
    assert np.array_equal(scaled, plain * np.float32(1.0 / 4.0)), "logit_scale divides the logits exactly"


@pytest.mark.parametrize("i", [1, 4])
def test_token_by_token_matches_full_pass(oracle, tmp_path, i):
    O = oracle
    p = write(O, tmp_path, SPECS[i])
    full = O.Model(p).forward(PROBE)
    m = O.Model(p)
    step = m.forward(PROBE[:4])
    for j in range(4, len(PROBE)):
        step = m.forward([PROBE[j]], pos0=j)
    assert float(np.abs(full - step).max()) < 1e-3


def test_config_and_refusals(oracle, tmp_path):
    O = oracle
    g = O.Model(write(O, tmp_path, SPECS[0])).config
    assert (g.embedding_scale, g.residual_scale, g.attention_scale, g.logit_scale) == \
        (12.0, np.float32(0.22), np.float32(0.0156), 8.0)
    assert not g.rope_neox and not g.post_norms and not g.qk_norm
    n = O.Model(write(O, tmp_path, SPECS[3])).config
    assert n.post_norms and n.qk_norm and n.qk_norm_full and n.rope_neox and n.embedding_scale == 0.0
    plain = O.Model(O.write_tiny_arch(str(tmp_path / "llama.gguf"), "llama")).config
    assert plain.residual_scale == 0.0 and not plain.post_norms
    with pytest.raises(ValueError, match="post_ffw_norm"):
        O.Model(O.write_tiny_arch(str(tmp_path / "nopost.gguf"), "olmo2", omit_post_ffw=True))
    with pytest.raises(ValueError, match="whole Q and K"):
        O.Model(O.write_tiny_arch(str(tmp_path / "shortq.gguf"), "olmo2", short_qnorm=True))
