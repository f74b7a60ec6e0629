"""Sampling on the device (Sampler.Sample, src/Engine.cs:361-380, with the generator's draw passed in) against the
oracle's or_sample, through the C ABI:

- wl_sample on random rows of the benchmark vocabularies (32000, 128256, 151936) and ragged small ones, over
  temperatures (0 and below: greedy) and top_p (>= 1: index order; < 1: the nucleus), many draws each. The device
  sums in a tree order where the reference adds one term at a time, so the choice is held equal wherever the draw lies
  more than 1e-9 of sum(p) from a boundary between two ids (the oracle reports that distance); within it either side
  of the boundary is accepted. Rows of equal logits check the order among equal probabilities (ascending ids).
- wl_forward_sample / wl_forward_batch_sample give or_sample of the logits wl_forward / wl_forward_batch return, and
  the greedy id at temperature 0; a draw outside [0, 1) is an argument error.
"""
import ctypes as C

import numpy as np
import pytest

from windlass_b200 import _lib
from windlass_b200.transformer import CudaTransformer, config0_spec

pytestmark = pytest.mark.gpu

SAFE = 1e-9


def device_sample(x, temperature, top_p, draw):
    import torch
    _lib.check(_lib.lib().wl_sample(C.c_void_p(x.data_ptr()), x.numel(), float(temperature), float(top_p),
                                    float(draw), C.c_void_p(OUT.data_ptr()), None))
    return int(OUT.cpu()[0])


OUT = None


@pytest.fixture(scope="module", autouse=True)
def out_word(wl):
    import torch
    global OUT
    OUT = torch.full((1,), -7, dtype=torch.int32, device="cuda")
    yield
    OUT = None


def check_row(oracle, v, t, p, draws):
    import torch
    x = torch.from_numpy(np.ascontiguousarray(v, dtype=np.float32)).cuda()
    near = 0
    for d in draws:
        want, margin = oracle.sample(v, t, p, d)
        got = device_sample(x, t, p, d)
        if margin > SAFE:
            assert got == want, f"V={v.size} t={t} top_p={p} draw={d}: {got} vs {want} (margin {margin:.2e})"
        else:
            near += 1
    return near


@pytest.mark.parametrize("V", [1, 3, 255, 4097, 32000, 128256, 151936])
def test_sample_kernel_matches_oracle(wl, oracle, V):
    rng = np.random.default_rng(V)
    near = total = 0
    for t in (0.0, -1.0, 0.25, 0.8, 1.0, 1.7):
        for p in (1.0, 0.95, 0.5, 0.05):
            v = (rng.standard_normal(V) * 3).astype(np.float32)
            draws = [float(d) for d in rng.random(6)] + [0.0]
            near += check_row(oracle, v, t, p, draws)
            total += len(draws)
    assert near <= total // 50


def test_sample_kernel_equal_probabilities(wl, oracle):
    rng = np.random.default_rng(11)
    for V in (4, 1000, 128256):
        v = np.zeros(V, dtype=np.float32)
        v[rng.integers(0, V, 3)] = 1.5                              # three equal leaders, the rest tied below
        draws = [float(d) for d in rng.random(8)]
        for t, p in ((1.0, 1.0), (1.0, 0.3), (0.5, 0.9), (1.0, 0.999)):
            check_row(oracle, v, t, p, draws)
        q = rng.integers(-3, 3, V).astype(np.float32)               # many ties at every level
        for t, p in ((1.0, 1.0), (0.7, 0.6), (2.0, 0.2)):
            check_row(oracle, q, t, p, draws)


def test_sample_kernel_underflow_and_extremes(wl, oracle):
    rng = np.random.default_rng(5)
    v = (rng.standard_normal(128256) * 50).astype(np.float32)
    # a tiny temperature leaves one id with a nonzero probability
    check_row(oracle, v, 1e-4, 1.0, [0.0, 0.5, 0.999999])
    check_row(oracle, v, 1e-4, 0.5, [0.0, 0.5, 0.999999])
    # a huge temperature makes the row nearly uniform
    check_row(oracle, v, 1e6, 1.0, [float(d) for d in rng.random(5)])
    check_row(oracle, v, 1e6, 0.9, [float(d) for d in rng.random(5)])


def test_sample_kernel_rejects_bad_arguments(wl):
    import torch
    x = torch.zeros(8, device="cuda")
    with pytest.raises(_lib.ArgumentError):
        _lib.check(_lib.lib().wl_sample(None, 8, 1.0, 1.0, 0.5, C.c_void_p(OUT.data_ptr()), None))
    with pytest.raises(_lib.ArgumentError):
        _lib.check(_lib.lib().wl_sample(C.c_void_p(x.data_ptr()), 0, 1.0, 1.0, 0.5, C.c_void_p(OUT.data_ptr()), None))
    for d in (1.0, -0.1, float("nan")):
        with pytest.raises(_lib.ArgumentError):
            _lib.check(_lib.lib().wl_sample(C.c_void_p(x.data_ptr()), 8, 1.0, 1.0, d, C.c_void_p(OUT.data_ptr()), None))
    # at temperature 0 the draw is not read
    _lib.check(_lib.lib().wl_sample(C.c_void_p(x.data_ptr()), 8, 0.0, 1.0, 7.0, C.c_void_p(OUT.data_ptr()), None))
    assert int(OUT.cpu()[0]) == 0


@pytest.fixture(scope="module")
def config0_file(oracle, tmp_path_factory):
    p = str(tmp_path_factory.mktemp("sample") / "config0.gguf")
    oracle.write_synth(p, config0_spec())
    return p


def test_forward_sample_is_sample_of_forward(wl, oracle, config0_file):
    rng = np.random.default_rng(21)
    prompt = rng.integers(0, 4096, 16).astype(np.int32)
    with CudaTransformer(config0_file, max_context=256) as m:
        a, b = m.new_sequence(), m.new_sequence()
        tok = None
        for i in range(6):
            toks = prompt if i == 0 else [tok]
            lg = m.forward(toks, seq=a, pos0=a.length)
            t, p, d = (0.8, 0.9, float(rng.random())) if i % 2 else (1.2, 1.0, float(rng.random()))
            want, margin = oracle.sample(lg, t, p, d)
            got = m.forward_sample(toks, t, p, d, seq=b, pos0=b.length)
            if margin > SAFE:
                assert got == want, (i, got, want)
            assert b.length == a.length
            tok = want
        # temperature 0 is the greedy id, whatever the draw
        lg = m.forward([tok], seq=a, pos0=a.length)
        assert m.forward_sample([tok], 0.0, 0.5, 3.0, seq=b, pos0=b.length) == oracle.argmax(lg)
        with pytest.raises(_lib.ArgumentError):
            m.forward_sample([tok], 1.0, 1.0, 1.0, seq=b, pos0=b.length)
        # ForwardBatch: each row with its own options
        seqs = [m.new_sequence() for _ in range(4)]
        for j, s in enumerate(seqs):
            m.forward(prompt[: 3 + j], seq=s)
        toks = np.array([7, 70, 700, 3000], dtype=np.int32)
        lb = m.forward_batch(seqs, toks)
        for s in seqs:
            s.truncate(s.length - 1)
        temps, tops = np.array([0.0, 0.6, 1.0, 1.5]), np.array([1.0, 0.8, 1.0, 0.3])
        draws = rng.random(4)
        ib = m.forward_batch_sample(seqs, toks, temps, tops, draws)
        for r in range(4):
            want, margin = oracle.sample(lb[r], temps[r], tops[r], draws[r])
            if margin > SAFE:
                assert int(ib[r]) == want, (r, int(ib[r]), want)
        assert [s.length for s in seqs] == [4, 5, 6, 7]
