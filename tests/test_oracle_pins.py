"""Pins the CPU oracle to the reference's own golden vectors and known answers (no GPU).

- llama.cpp logits and argmax for the 18 StandardSpecs tiny models (tests/fixtures/llama-cpp-reference.txt, via
  tests/golden/llamacpp_reference.json), with the reference's tolerance (tests/Tests.cs:250-278).
- I-quant table hashes (tests/IQuantTests.cs:251-318) and the hand-built IQ4_NL / IQ2_XXS blocks (:320-370).
- An independent dequantizer (gguf-py 0.19.0) on the same bytes, bit-exact, for Q8_0, Q6_K, Q4_K, IQ4_XS, IQ2_XXS.
- Fused dot == decode-then-dot (tests/Tests.cs:280-303), routing hand cases (tests/MoeTests.cs:116-149),
  batch rows == single runs (tests/BatchTests.cs:29-94), KV stepwise == full pass (tests/Tests.cs:323-346).
"""
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PROBE = [1, 10, 50, 100, 200, 257, 290, 5, 7, 99, 33, 72]


def standard_specs(O):
    specs = [("llama", t, {}) for t in (O.F32, O.F16, O.BF16, O.Q4_0, O.Q4_1, O.Q5_0, O.Q5_1, O.Q8_0, O.Q2_K, O.Q3_K,
                                         O.Q4_K, O.Q5_K, O.Q6_K)]
    specs += [("qwen2", O.Q8_0, {}), ("qwen3", O.Q4_K, {}), ("qwen2", O.Q6_K, {"tied": True}),
              ("llama", O.Q8_0, {"spm": True}), ("llama", O.F16, {"rope_freqs": True})]
    return specs


def spec_key(O, arch, t, kw):
    return arch + "-" + O.NAMES[t] + ("-tied" if kw.get("tied") else "") + ("-spm" if kw.get("spm") else "") + \
        ("-ropefreqs" if kw.get("rope_freqs") else "")


def test_oracle_matches_llamacpp_fixture(oracle, golden, tmp_path):
    O = oracle
    problems = []
    for arch, t, kw in standard_specs(O):
        key = spec_key(O, arch, t, kw)
        p = str(tmp_path / (key + ".gguf"))
        O.write_tiny(p, arch=arch, type=t, **kw)
        logits = O.Model(p).forward(PROBE, all_logits=True)
        ref = golden["models"][key]
        last = np.array(ref["last"])
        assert logits.shape == (len(PROBE), last.size), key
        std = last.std()
        md = np.abs(logits[-1] - last).max()
        agree = sum(int(np.argmax(logits[i])) == ref["argmax"][i] for i in range(len(PROBE)))
        tol = 0.02 if t in (O.F32, O.F16) else 0.2
        if md / std > tol or agree < len(PROBE) - 1:
            problems.append(f"{key}: max diff {md:.4f} (std {std:.3f}), top token agrees at {agree}/12")
    assert not problems, "\n".join(problems)


def _array(name):
    src = open(os.path.join(ROOT, "windlass_b200", "csrc", "iq_tables.h")).read()
    m = re.search(name + r"\[\d+\] = \{(.*?)\};", src, re.S)
    return [int(v.strip().rstrip("ULu"), 0) for v in m.group(1).split(",") if v.strip()]


def _fnv(vals, width):
    h = 14695981039346656037
    for v in vals:
        for j in range(width):
            h ^= (v >> (8 * j)) & 0xFF
            h = (h * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return h


@pytest.mark.parametrize("name,width,expect", [
    ("WL_IQ2XXS_GRID", 8, 0xbb4ee025b5ac6e8e), ("WL_IQ2XS_GRID", 8, 0xc9b1ee61e79909bd),
    ("WL_IQ2S_GRID", 8, 0x123edd38a3b62b90), ("WL_IQ3XXS_GRID", 4, 0xdfa5dc83d6a155d5),
    ("WL_IQ3S_GRID", 4, 0xfa37020c25b44829), ("WL_IQ1S_GRID", 8, 0x6703ed863501ae2e)])
def test_iq_table_hashes(name, width, expect):
    assert _fnv(_array(name), width) == expect


def test_iq_sign_and_value_tables():
    ks = _array("WL_KSIGNS_IQ2XS")
    for i, v in enumerate(ks):
        assert v == i | ((bin(i).count("1") & 1) << 7)
    assert _array("WL_KVALUES_IQ4NL") == [-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113]


def test_iq_hand_blocks(oracle):
    O = oracle
    kv = [-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113]
    nl = bytearray(18)
    nl[0], nl[1] = 0x00, 0x40
    for j in range(16):
        nl[2 + j] = j | ((15 - j) << 4)
    y = O.decode(O.IQ4_NL, bytes(nl), 32)
    assert list(y[:16]) == [2.0 * kv[j] for j in range(16)]
    assert list(y[16:]) == [2.0 * kv[15 - j] for j in range(16)]
    xxs = bytearray(66)
    xxs[0], xxs[1] = 0x00, 0x3C
    xxs[2:6] = bytes([0, 1, 2, 3])
    aux1 = (3 << 28) | (0 << 0) | (1 << 7) | (2 << 14) | (127 << 21)
    xxs[6:10] = aux1.to_bytes(4, "little")
    y = O.decode(O.IQ2_XXS, bytes(xxs), 256)
    want = [0.875 * 8] * 8
    want += [0.875 * (43 if j == 0 else 8) * (-1 if j in (0, 7) else 1) for j in range(8)]
    want += [0.875 * (25 if j < 2 else 8) * (-1 if j in (1, 7) else 1) for j in range(8)]
    want += [-0.875 * (43 if j == 1 else 8) for j in range(8)]
    np.testing.assert_allclose(y[:32], want, atol=1e-6)
    np.testing.assert_allclose(y[32:], 1.0, atol=1e-6)


def random_blocks(O, t, blocks, seed):
    """RandomBlocks of tests/IQuantTests.cs: random payload with a chosen fp16 scale in each block."""
    rng = O.Rng(seed)
    bs, bb = O.layout(t)
    data = bytearray(rng.byte() for _ in range(blocks * bb))
    dbits = [0x3A00, 0x3E00, 0x3800, 0xB400, 0x3C00]
    for k in range(blocks):
        if t == O.IQ1_M:
            for i in range(4):
                hi = data[k * bb + 48 + 2 * i + 1]
                data[k * bb + 48 + 2 * i + 1] = (hi & 0x0F) | (((dbits[k % 5] >> (4 * i)) & 15) << 4)
        else:
            data[k * bb] = dbits[k % 5] & 0xFF
            data[k * bb + 1] = dbits[k % 5] >> 8
    return np.frombuffer(bytes(data), dtype=np.uint8).copy()


@pytest.mark.parametrize("tname", ["q8_0", "q6_K", "q4_K", "iq4_xs", "iq2_xxs", "q5_K", "q4_0", "q2_K", "q3_K"])
def test_decoders_match_gguf_py(oracle, tname):
    gq = pytest.importorskip("gguf.quants")
    from gguf import GGMLQuantizationType as G
    O = oracle
    t = O.TYPE_OF[tname]
    bs, bb = O.layout(t)
    rng = O.Rng(11)
    cols = 2 * max(bs, 256)
    data = O.matrix(rng, t, 3, cols, 0.5) if t not in (O.IQ4_XS, O.IQ2_XXS) else random_blocks(O, t, 3 * cols // bs, 11)
    mine = O.decode(t, data, 3 * cols)
    theirs = gq.dequantize(data, G[tname.upper()]).reshape(-1).astype(np.float32)
    assert np.array_equal(mine.view(np.uint32), theirs.view(np.uint32)), f"{tname}: oracle and gguf-py disagree"


def test_fused_dot_matches_decode(oracle):
    """FusedDotMatchesDecode (tests/Tests.cs:280-303)."""
    O = oracle
    for t in (O.F32, O.F16, O.BF16, O.Q4_0, O.Q8_0, O.Q4_K, O.Q5_K, O.Q6_K):
        assert O.lib().or_can_dot(t)
        data = O.matrix(O.Rng(3), t, 3, 512, 0.5)
        x = O.Rng(9).normals(512)
        rb = len(data) // 3
        for r in range(3):
            row = data[r * rb:(r + 1) * rb]
            dec = O.decode(t, row, 512).astype(np.float64)
            want = float(np.dot(dec, x.astype(np.float64)))
            mag = float(np.abs(dec * x).sum())
            got = O.dot_row(t, row, x)
            assert abs(got - want) <= 1e-5 * mag + 1e-6, (O.NAMES[t], r, got, want)


def test_routing_math(oracle):
    """RoutingMath (tests/MoeTests.cs:116-149)."""
    O = oracle
    lg = np.array([1, 3, 2, 0], dtype=np.float32)
    z = np.exp(1) + np.exp(3) + np.exp(2) + 1
    p1, p2 = np.exp(3) / z, np.exp(2) / z
    sel, w, cnt = O.route(lg, 2, False)
    assert list(sel) == [1, 2] and abs(w[0] - p1) < 1e-6 and abs(w[1] - p2) < 1e-6 and list(cnt) == [0, 1, 1, 0]
    sel, w, cnt = O.route(lg, 2, True)
    assert abs(w[0] - p1 / (p1 + p2)) < 1e-6 and abs(w[0] + w[1] - 1) < 1e-6
    sel, w, _ = O.route(np.full(4, 2, dtype=np.float32), 2, False)
    assert list(sel) == [0, 1] and abs(w[0] - 0.25) < 1e-6
    sel, w, _ = O.route(np.full(4, 2, dtype=np.float32), 2, True)
    assert abs(w[0] - 0.5) < 1e-6 and abs(w[1] - 0.5) < 1e-6
    sel, w, _ = O.route(lg, 4, True)
    assert list(sel) == [1, 2, 0, 3] and abs(w.sum() - 1) < 1e-6


def test_oracle_batch_rows_equal_single_runs(oracle, tmp_path):
    """BatchForwardMatchesSingle (tests/BatchTests.cs:29-94) on the oracle itself."""
    O = oracle
    p = O.write_tiny(str(tmp_path / "q4k.gguf"), arch="qwen3", type=O.Q4_K)
    m = O.Model(p)
    a, b = m.new_sequence(), m.new_sequence()
    m.forward([1, 10, 50], seq=a)
    m.forward([100, 200], seq=b)
    batch = m.forward_batch([a, b], [7, 99])
    ref = O.Model(p)
    a2, b2 = ref.new_sequence(), ref.new_sequence()
    ref.forward([1, 10, 50], seq=a2)
    ref.forward([100, 200], seq=b2)
    assert np.array_equal(batch[0], ref.forward([7], pos0=3, seq=a2))
    assert np.array_equal(batch[1], ref.forward([99], pos0=2, seq=b2))


def test_oracle_kv_cache_matches_full_pass(oracle, tmp_path):
    """KvCacheMatchesFullPass (tests/Tests.cs:323-346)."""
    O = oracle
    p = O.write_tiny(str(tmp_path / "q8.gguf"), arch="llama", type=O.Q8_0, rope_freqs=True)
    full = O.Model(p).forward(PROBE)
    m = O.Model(p)
    step = m.forward(PROBE[:4])
    for i in range(4, len(PROBE)):
        step = m.forward([PROBE[i]], pos0=i)
    assert np.abs(full - step).max() < 1e-3
    again = m.forward(PROBE[6:], pos0=6)          # Truncate(6) then Forward from position 6
    assert np.abs(full - again).max() < 1e-3


def test_synthetic_quantizers_round_trip(oracle):
    """The round-to-nearest quantizers keep N(0, 0.02) weights close (relative RMS error per format)."""
    O = oracle
    rng = np.random.default_rng(0)
    x = (rng.standard_normal(256 * 64) * 0.02).astype(np.float32)
    for t, bound in ((O.Q8_0, 0.01), (O.Q6_K, 0.03), (O.Q4_K, 0.12)):
        bs, bb = O.layout(t)
        out = np.concatenate([O.quantize_block(t, x[i:i + bs]) for i in range(0, x.size, bs)])
        y = O.decode(t, out, x.size)
        rel = np.sqrt(np.mean((y - x) ** 2)) / np.sqrt(np.mean(x ** 2))
        assert rel < bound, (O.NAMES[t], rel)
