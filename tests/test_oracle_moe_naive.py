"""MatchesReference (tests/MoeTests.cs:82-110) on the oracle: the oracle's forward pass of the eight reference MoE
test models (each layout, several weight types, both renormalisation settings, a tied head, a dense layer among MoE
layers) against an independent double-precision model (tests/naive_moe.py): every logit within 3e-3 of the last
row's standard deviation and the top token equal at every position. The CUDA path is compared with the oracle on the
same models in tests/test_gpu_model.py."""
import numpy as np
import pytest

from tests.naive_moe import Naive

PROBE = [1, 10, 50, 100, 200, 257, 290, 5, 7, 99, 33, 72]


def specs(O):
    return [
        dict(layout="llama", type=O.F32, experts=4, used=2),
        dict(layout="mixtral", type=O.Q8_0, experts=8, used=2),
        dict(layout="llama", type=O.Q5_0, experts=4, used=3, norm_key=0),
        dict(layout="qwen2moe", type=O.Q4_K, experts=8, used=2),
        dict(layout="qwen2moe", type=O.Q6_K, experts=4, used=2, norm_key=1, tied=True),
        dict(layout="qwen3moe", type=O.Q4_K, experts=8, used=3, layers=3, dense_layers=(1,)),
        dict(layout="qwen3moe", type=O.Q3_K, experts=4, used=2, norm_key=0),
        dict(layout="qwen3moe", type=O.F16, experts=4, used=4),
    ]


@pytest.mark.parametrize("i", range(8))
def test_oracle_moe_matches_the_naive_double_model(oracle, tmp_path, i):
    O = oracle
    s = specs(O)[i]
    path = O.write_tiny_moe(str(tmp_path / f"moe{i}.gguf"), **s)
    got = O.Model(path, max_context=64).forward(PROBE, all_logits=True)
    nv = Naive(O, path, s["layout"], s["experts"], s["used"], s.get("norm_key", -1), s.get("tied", False),
               s.get("dense_layers", ()))
    try:
        want = nv.forward(PROBE)
    finally:
        nv.close()
    T, V = want.shape
    got = np.asarray(got, dtype=np.float64).reshape(T, V)
    std = float(want[-1].std())
    md = float(np.abs(got - want).max())
    agree = int((got.argmax(axis=1) == want.argmax(axis=1)).sum())
    assert md <= 3e-3 * std and agree == T, f"{s}: max diff {md:.5f} (std {std:.3f}), top token {agree}/{T}"
