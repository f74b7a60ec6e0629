"""Greedy selection on the device, against the host rule of the reference's sampler (Sampler.Sample at temperature 0,
src/Engine.cs:356-360, and Argmax, :329-334: best = 0; if x[i] > x[best] then best = i), through the C ABI:

- wl_argmax on crafted rows: ties, NaN at index 0 and elsewhere, -0 and +0, all -inf, ragged and large vocabularies,
  many rows at once; compared with the oracle's or_argmax (the same loop in C);
- wl_forward_argmax / wl_forward_batch_argmax give the argmax of the logits wl_forward / wl_forward_batch return;
- wl_generate_greedy (the decode loop of src/Engine.cs:187-203 with the id chained on the device) gives the tokens
  of a host loop of forward + argmax, and leaves the sequence where that loop does, across chunk boundaries, with
  stop ids, cancel and after further forwards; on configs[0] it gives the oracle's greedy tokens;
- wl_forward_mixed (prompts joining a decode step) gives each sequence's own pass.
"""
import ctypes as C

import numpy as np
import pytest

from windlass_b200 import _lib
from windlass_b200.transformer import CancelFlag, CudaTransformer, config0_spec

pytestmark = pytest.mark.gpu


def device_argmax(rows):
    import torch
    x = torch.from_numpy(np.ascontiguousarray(rows, dtype=np.float32)).cuda()
    R, V = x.shape
    ids = torch.full((R,), -7, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    _lib.check(_lib.lib().wl_argmax(C.c_void_p(x.data_ptr()), V, R, C.c_void_p(ids.data_ptr()), None))
    return ids.cpu().numpy()


def test_argmax_kernel_matches_host_rule(wl, oracle):
    rng = np.random.default_rng(3)
    cases = []
    for V in (1, 2, 7, 255, 256, 257, 2048, 2049, 4096, 32000, 128256, 151936, 1 << 20):
        cases.append(rng.standard_normal((3, V)).astype(np.float32))
    # ties: the lowest index of the repeated maximum wins
    t = rng.standard_normal((4, 128256)).astype(np.float32)
    t[0, [5, 90000, 128255]] = 9.0
    t[1, [128255, 64000]] = 9.0
    t[2, :] = 1.0
    t[3, [0, 77]] = 50.0
    cases.append(t)
    # NaN: at index 0 the answer is 0; elsewhere it never wins; all NaN gives 0
    n = rng.standard_normal((4, 50000)).astype(np.float32)
    n[0, 0] = np.nan
    n[0, 10] = 1e30
    n[1, [3, 40000]] = np.nan
    n[1, 20000] = 100.0
    n[2, :] = np.nan
    n[3, 1:] = np.nan
    n[3, 0] = -5.0
    cases.append(n)
    # signed zeros compare equal; infinities
    z = np.full((4, 3000), -1.0, dtype=np.float32)
    z[0, 100], z[0, 50] = 0.0, -0.0
    z[1, 7], z[1, 8] = -0.0, 0.0
    z[2, :] = -np.inf
    z[3, 2999] = np.inf
    z[3, 1] = np.inf
    cases.append(z)
    # many rows in one launch
    cases.append(rng.standard_normal((300, 5000)).astype(np.float32))
    for rows in cases:
        got = device_argmax(rows)
        want = np.array([oracle.argmax(r) for r in rows], dtype=np.int32)
        assert (got == want).all(), f"V={rows.shape[1]}: {got[got != want][:5]} vs {want[got != want][:5]}"


def test_argmax_kernel_rejects_bad_arguments(wl):
    with pytest.raises(_lib.ArgumentError):
        _lib.check(_lib.lib().wl_argmax(None, 10, 1, None, None))
    with pytest.raises(_lib.ArgumentError):
        _lib.check(_lib.lib().wl_argmax(C.c_void_p(16), 0, 1, C.c_void_p(16), None))


def host_argmax(v):
    best = 0
    for i in range(1, v.size):          # the reference's loop, for small vocabularies only
        if v[i] > v[best]:
            best = i
    return best


@pytest.fixture(scope="module")
def config0_file(oracle, tmp_path_factory):
    p = str(tmp_path_factory.mktemp("greedy") / "config0.gguf")
    oracle.write_synth(p, config0_spec())
    return p


def test_forward_argmax_is_argmax_of_forward(wl, oracle, config0_file):
    prompt = np.random.default_rng(1).integers(0, 4096, 24).astype(np.int32)
    with CudaTransformer(config0_file, max_context=256) as m:
        logits = m.forward(prompt, all_logits=True)
        ids = m.forward_argmax(prompt, all_rows=True)
        assert m.length == 24
        assert list(ids) == [oracle.argmax(r) for r in logits]
        assert m.forward_argmax(prompt) == oracle.argmax(logits[-1])
        # decode rows, and the graph path (the second T = 1 call of a shape replays a captured graph)
        for i in range(4):
            tok = (int(ids[-1]) + i) % 4096
            lg = m.forward([tok], pos0=24 + i)
            assert m.forward_argmax([tok], pos0=24 + i) == oracle.argmax(lg)
        # ForwardBatch
        seqs = [m.new_sequence() for _ in range(3)]
        for j, s in enumerate(seqs):
            m.forward(prompt[: 5 + j], seq=s)
        toks = np.array([11, 22, 33], dtype=np.int32)
        lb = m.forward_batch(seqs, toks)
        for s in seqs:
            s.truncate(s.length - 1)
        ib = m.forward_batch_argmax(seqs, toks)
        assert list(ib) == [oracle.argmax(r) for r in lb]
        assert [s.length for s in seqs] == [6, 7, 8]


def reference_loop(m, token, max_new, stop, seq=None):
    """LayeredBackend.Generate's greedy loop on host logits (src/Engine.cs:187-203)."""
    out = []
    pos = (seq.length if seq is not None else m.length)
    cur = token
    for _ in range(max_new):
        lg = m.forward([cur], pos0=pos, seq=seq)
        pos += 1
        cur = host_argmax(lg)
        out.append(cur)
        if cur in stop:
            break
    return out


@pytest.mark.parametrize("chunk", [1, 5, 16, 64])
def test_generate_greedy_matches_host_loop(wl, config0_file, chunk):
    prompt = np.random.default_rng(2).integers(0, 4096, 20).astype(np.int32)
    with CudaTransformer(config0_file, max_context=256) as m:
        a, b = m.new_sequence(), m.new_sequence()
        first = int(np.argmax(m.forward(prompt, seq=a)))
        m.forward(prompt, seq=b)
        want = reference_loop(m, first, 40, (), seq=a)
        got = m.generate_greedy(first, 40, chunk=chunk, seq=b)
        assert list(got) == want
        assert b.length == a.length == 60
        # the KV cache the chained steps left is the one the host loop left: the next pass agrees bit for bit
        la = m.forward([7], pos0=60, seq=a)
        lb = m.forward([7], pos0=60, seq=b)
        assert np.array_equal(la, lb)


def test_generate_greedy_stops_at_stop_id(wl, config0_file):
    prompt = np.random.default_rng(4).integers(0, 4096, 12).astype(np.int32)
    with CudaTransformer(config0_file, max_context=256) as m:
        s = m.new_sequence()
        first = int(np.argmax(m.forward(prompt, seq=s)))
        full = list(m.generate_greedy(first, 30, chunk=8, seq=s))
        assert len(full) == 30 and s.length == 42
        absent = next(i for i in range(4096) if i not in full)
        for k in (0, 3, 7, 8, 20):
            s.truncate(12)
            got = list(m.generate_greedy(first, 30, stop_ids=[absent, full[k]], chunk=8, seq=s))
            k0 = full.index(full[k])                 # the first occurrence ends the call
            assert got == full[: k0 + 1]
            assert s.length == 12 + k0 + 1
        s.truncate(12)
        assert list(m.generate_greedy(first, 0, seq=s)) == [] and s.length == 12


def test_generate_greedy_cancel_and_errors(wl, config0_file):
    with CudaTransformer(config0_file, max_context=64) as m:
        m.forward([1, 2, 3])
        c = CancelFlag()
        c.set()
        with pytest.raises(_lib.OperationCanceledError):
            m.generate_greedy(5, 10, cancel=c)
        assert m.length == 3
        with pytest.raises(_lib.ArgumentError):
            m.generate_greedy(4096, 4)                # outside the vocabulary
        with pytest.raises(_lib.ArgumentError):
            m.generate_greedy(5, 62)                  # 3 + 62 positions > 64
        with pytest.raises(_lib.ArgumentError):
            m.generate_greedy(5, 4, chunk=65)
        assert m.length == 3
        assert len(m.generate_greedy(5, 61)) == 61 and m.length == 64


def test_generate_greedy_config0_oracle_tokens(wl, oracle, config0_file):
    """configs[0] (32 prompt ids, 32 greedy tokens, b1): the chained device decode gives the oracle's tokens."""
    prompt = np.random.default_rng(0).integers(0, 4096, 32).astype(np.int32)
    om = oracle.Model(config0_file, max_context=128)
    logits = om.forward(prompt)
    want = []
    for i in range(32):
        t = oracle.argmax(logits)
        want.append(t)
        logits = om.forward([t], pos0=32 + i)
    with CudaTransformer(config0_file, max_context=128) as m:
        first = m.forward_argmax(prompt)
        got = [first] + list(m.generate_greedy(first, 31))
    assert got == want


def test_generate_greedy_moe_device_path(wl, oracle, tmp_path):
    """MoE decode steps (router top-k and grouped expert matvec on the device) chain the same way."""
    p = oracle.write_tiny_moe(str(tmp_path / "moe.gguf"), layout="qwen3moe", type=oracle.Q4_K, experts=8, used=2,
                              layers=2)
    with CudaTransformer(p, max_context=128) as m:
        a, b = m.new_sequence(), m.new_sequence()
        first = int(np.argmax(m.forward([3, 1, 4, 1, 5], seq=a)))
        m.forward([3, 1, 4, 1, 5], seq=b)
        want = reference_loop(m, first, 20, (), seq=a)
        runs = m.expert_runs
        got = m.generate_greedy(first, 20, chunk=7, seq=b)
        assert list(got) == want
        assert m.expert_runs - runs == 20 * 2 * 2          # 20 steps x 2 layers x 2 chosen experts


def test_forward_mixed_rows_equal_each_sequence_alone(wl, oracle, config0_file):
    """wl_forward_mixed (prompts joining a decode step): each sequence's last row equals that sequence's own pass,
    bit for bit up to 8 rows (every row on the per-column matvec), and within the prompt tolerance beyond (rows on
    the tensor-core GEMM); lengths advance by each count; the argmax form returns the rows' greedy ids."""
    from tests.test_gpu_model import compare
    rng = np.random.default_rng(5)
    toks = [rng.integers(0, 4096, n).astype(np.int32) for n in (9, 6, 40)]
    with CudaTransformer(config0_file, max_context=256) as m:
        mixed = [m.new_sequence() for _ in range(3)]
        alone = [m.new_sequence() for _ in range(3)]
        for s, a, t in zip(mixed, alone, toks):
            m.forward(t[:5], seq=s)
            m.forward(t[:5], seq=a)
        # 8 rows: sequence 0 decodes one token, 1 takes a 1-token step, 2 joins with 6 prompt tokens
        for step in range(3):              # the same shape again: the captured graph serves it
            parts = [toks[0][5 + step:6 + step], toks[1][5:6] if step == 0 else np.array([7 + step], np.int32),
                     toks[2][5 + 6 * step: 11 + 6 * step]]
            got = m.forward_mixed(mixed, parts)
            for i in range(3):
                want = m.forward(parts[i], pos0=alone[i].length, seq=alone[i])
                assert np.array_equal(got[i], want), f"step {step}: mixed row {i} differs from its own pass"
            assert [s.length for s in mixed] == [a.length for a in alone]
        # 24 rows: the GEMM path for the step, the matvec for the single-token pass alone
        parts = [toks[0][8:9], np.array([99], np.int32), toks[2][23:40]]
        ids = m.forward_mixed(mixed, parts, argmax=True)
        wants = [m.forward(p, pos0=a.length, seq=a) for p, a in zip(parts, alone)]
        for i, s in enumerate(mixed):
            s.truncate(s.length - len(parts[i]))
        got = m.forward_mixed(mixed, parts)
        compare(got, np.stack(wants), "mixed step on the GEMM", rel=1e-3)
        assert list(ids) == [oracle.argmax(r) for r in got]
        assert [s.length for s in mixed] == [a.length for a in alone]
        # argument errors
        with pytest.raises(_lib.ArgumentError):
            m.forward_mixed([mixed[0], mixed[0]], [[1], [2]])
        with pytest.raises(_lib.ArgumentError):
            m.forward_mixed(mixed[:2], [[1], []])
        with pytest.raises(_lib.ArgumentError):
            m.forward_mixed(mixed[:1], [list(range(300))])


def test_forward_mixed_matches_oracle(wl, oracle, config0_file):
    """Each sequence of a mixed step against the CPU oracle's own pass over that sequence."""
    from tests.test_gpu_model import compare
    rng = np.random.default_rng(6)
    prompts = [rng.integers(0, 4096, n).astype(np.int32) for n in (3, 7, 12)]
    joins = [rng.integers(0, 4096, n).astype(np.int32) for n in (1, 1, 5)]
    with CudaTransformer(config0_file, max_context=128) as m:
        seqs = [m.new_sequence() for _ in range(3)]
        for s, p in zip(seqs, prompts):
            m.forward(p, seq=s)
        got = m.forward_mixed(seqs, joins)
    for i in range(3):
        om = oracle.Model(config0_file, max_context=128)
        om.forward(prompts[i])
        want = om.forward(joins[i], pos0=len(prompts[i]))
        compare(got[i], want, f"mixed sequence {i}")
