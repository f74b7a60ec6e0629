"""Tensor parallelism on several GPUs (one process per GPU under torchrun, NCCL over NVLink) against the CPU oracle:

- the prompt's logits on every rank match the oracle within 1e-3 of their standard deviation, argmax equal;
- configs[0] greedy decode gives the oracle's tokens;
- every rank returns the same logits (the all-reduce and the head's all-gather leave no rank behind);
- ForwardBatch rows equal single runs (bit-identical at 2 ranks, where each all-reduced value is one sum of two);
- the decode-step all-reduces fused into the matvec and the norm over peer memory give what NCCL's give (bit for bit
  at 2 ranks), and are the ones in use;
- a Qwen3-MoE-shaped model with whole experts placed on each GPU (the "moe" case) meets all of the above.

Needs at least 2 GPUs; WL_TP_TEST_GPUS picks how many ranks (default 2).
"""
import os
import signal
import socket
import subprocess
import sys

import numpy as np
import pytest

from tests.test_gpu_model import compare, greedy
from tests.tp_worker import spec_of

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _gpus():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def run_ranks(n, spec, out, steps=16, graphs=1, nccl_only=0, timeout=300):
    """torchrun of tests/tp_worker.py on n GPUs; every rank's saved results."""
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
           "--master-addr", "127.0.0.1", f"--master-port={_free_port()}", os.path.join(ROOT, "tests", "tp_worker.py"),
           "--spec", spec, "--out", str(out), "--steps", str(steps), "--graphs", str(graphs),
           "--nccl-only", str(nccl_only)]
    p = subprocess.Popen(cmd, cwd=ROOT, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True,
                         start_new_session=True)
    try:
        log, _ = p.communicate(timeout=timeout)
    except subprocess.TimeoutExpired:
        os.killpg(p.pid, signal.SIGKILL)         # torchrun and every rank it started
        log, _ = p.communicate()
        pytest.fail(f"tensor-parallel ranks did not finish in {timeout} s:\n{log[-4000:]}")
    assert p.returncode == 0, f"tensor-parallel ranks failed:\n{log[-4000:]}"
    return [dict(np.load(os.path.join(out, f"rank{r}.npz"))) for r in range(n)]


@pytest.mark.parametrize("spec", ["config0", "gqa", "moe"])
def test_tensor_parallel_matches_oracle(wl, oracle, tmp_path, spec):
    n = int(os.environ.get("WL_TP_TEST_GPUS", "2"))
    if _gpus() < n:
        pytest.skip(f"needs {n} GPUs")
    O = oracle
    sp = spec_of(spec)
    if sp.ff % (n * (32 if sp.type_ffn_down == O.Q8_0 else 256)):
        pytest.skip(f"{spec}'s ffn_down columns ({sp.ff}) do not split into whole blocks over {n} GPUs")
    (tmp_path / "fused").mkdir()
    (tmp_path / "nccl").mkdir()
    res = run_ranks(n, spec, tmp_path / "fused")
    assert all(int(r["fused"]) == 1 for r in res), "the GPUs could not map each other's memory (fused all-reduce off)"
    ref = run_ranks(n, spec, tmp_path / "nccl", nccl_only=1)
    assert all(int(r["fused"]) == 0 for r in ref)
    if n == 2:
        # two partials: the fused sum p0 + p1 and NCCL's sum are the same float operation
        for k in ("prefill", "tokens", "decode", "batch", "single"):
            assert np.array_equal(res[0][k], ref[0][k]), f"fused and NCCL all-reduce differ in {k}"
    for r in range(1, n):
        for k in ("prefill", "tokens", "decode", "batch", "chained", "argmax"):
            assert np.array_equal(res[r][k], res[0][k]), f"rank {r} returned other {k} than rank 0"
    got = res[0]
    # device greedy: the chained decode and the per-step device argmax follow the host argmax's token path
    assert list(got["chained"]) == list(got["tokens"][1:]), "device-chained greedy decode differs from the host loop"
    assert list(got["argmax"][:-1]) == list(got["tokens"][1:]), "device argmax differs from the host argmax"
    prompt = got["prompt"]
    path = O.write_synth(str(tmp_path / f"{spec}.gguf"), sp)
    om = O.Model(path, max_context=256)
    compare(got["prefill"], om.forward(prompt, all_logits=True), f"tp{n} {spec} prefill")
    om2 = O.Model(path, max_context=256)
    want_tokens = greedy(lambda t, p0: om2.forward(t, pos0=p0), prompt, len(got["tokens"]))
    if spec == "config0":
        assert list(got["tokens"]) == want_tokens, "configs[0] greedy tokens differ from the oracle"
    # the decode logits along the GPU's own token path
    om3 = O.Model(path, max_context=256)
    om3.forward(prompt)
    for i, t in enumerate(got["tokens"]):
        compare(got["decode"][i], om3.forward([int(t)], pos0=len(prompt) + i), f"tp{n} {spec} decode step {i}")
    if n == 2:
        assert np.array_equal(got["batch"], got["single"]), "ForwardBatch rows differ from single runs"
    else:
        compare(got["batch"], got["single"], f"tp{n} {spec} batch rows")


def test_in_process_group_matches_process_ranks(wl, tmp_path):
    """tp_rank = -1: one wl_model spanning the GPUs inside this process (one host thread per GPU, peers reached by
    pointer) returns bit for bit what the one-process-per-GPU ranks return, fused all-reduce included."""
    from windlass_b200.transformer import CudaTransformer
    n = int(os.environ.get("WL_TP_TEST_GPUS", "2"))
    if _gpus() < n:
        pytest.skip(f"needs {n} GPUs")
    ranks = run_ranks(n, "gqa", tmp_path)
    sp = spec_of("gqa")
    with CudaTransformer(synthetic=sp, max_context=256, tp_size=n, tp_rank=-1) as m:
        assert m.info.tp_size == n and m.info.tp_rank == -1 and m.info.tp_fused == 1
        prompt = ranks[0]["prompt"]
        assert np.array_equal(m.forward(prompt, all_logits=True), ranks[0]["prefill"])
        for i, t in enumerate(ranks[0]["tokens"]):
            assert np.array_equal(m.forward([int(t)], pos0=len(prompt) + i), ranks[0]["decode"][i]), f"step {i}"
        m.truncate(len(prompt))
        toks = ranks[0]["tokens"]
        assert list(m.generate_greedy(int(toks[0]), len(toks) - 1, chunk=5)) == list(ranks[0]["chained"])
        s1, s2 = m.new_sequence(), m.new_sequence()
        m.forward(prompt[:7], seq=s1)
        m.forward(prompt[3:20], seq=s2)
        assert np.array_equal(m.forward_batch([s1, s2], [11, 22]), ranks[0]["batch"])
        stages = []
        m.forward(prompt[:5], seq=s1, on_stage=lambda d, tot: stages.append(d))
        assert stages[-1] == sp.layers + 1
        s1.close()
        s2.close()
