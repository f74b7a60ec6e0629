"""One rank of the tensor-parallel GPU tests, launched by tests/test_gpu_tp.py under torchrun (one process per GPU).

Every rank opens the same synthetic model split over all ranks (wl_options.tp_*), runs a prompt, a greedy decode (by
host argmax, then chained on the device) and a ForwardBatch step with the same arguments, and saves what its calls
returned to <out>/rank<r>.npz.
"""
import argparse
import datetime
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def spec_of(name):
    from windlass_b200.transformer import config0_spec, synth_spec
    if name == "config0":
        return config0_spec()
    if name == "moe":
        # Qwen3-MoE layers at small size: 16 experts top-4 (whole experts per GPU), QK-norm, head_dim 128
        return synth_spec("qwen3moe", 2, 1024, 16, 8, 128, 0, 8192, experts=16, experts_used=4, expert_ff=512,
                          rope_base=1000000.0, rms_eps=1e-6, type_attn_v=14, type_embd=12, seed=5)
    # GQA with Q6_K attn_v and head, the Q4_K_M mix of the 8B/70B shapes at small size
    return synth_spec("llama", 2, 2048, 32, 8, 64, 4096, 8192, rope_base=500000.0, type_attn_v=14, type_embd=12,
                      seed=7)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--spec", default="config0")
    ap.add_argument("--out", required=True)
    ap.add_argument("--prompt", type=int, default=32)
    ap.add_argument("--steps", type=int, default=16)
    ap.add_argument("--graphs", type=int, default=1)
    ap.add_argument("--nccl-only", type=int, default=0)
    args = ap.parse_args()

    import torch
    import torch.distributed as dist
    from windlass_b200 import tp
    rank, world, local = tp.env_ranks()
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=240))
    spec = spec_of(args.spec)
    m = tp.open_group_model(dist, local, synthetic=spec, max_context=256, use_graphs=args.graphs,
                            tp_nccl_only=args.nccl_only)
    assert m.info.tp_size == world and m.info.tp_rank == rank
    prompt = np.random.default_rng(0).integers(0, spec.vocab, args.prompt).astype(np.int32)
    res = {"prompt": prompt, "prefill": m.forward(prompt, all_logits=True).copy(), "fused": m.info.tp_fused}
    toks, dec = [], []
    logits = res["prefill"][-1]
    for i in range(args.steps):
        t = int(np.argmax(logits))
        toks.append(t)
        logits = m.forward([t], pos0=args.prompt + i).copy()
        dec.append(logits)
    res["tokens"] = np.array(toks, dtype=np.int32)
    res["decode"] = np.stack(dec)
    # the same decode with the greedy choice made and chained on the device (every rank takes the same steps)
    m.truncate(args.prompt)
    res["chained"] = m.generate_greedy(toks[0], args.steps - 1, chunk=5)
    res["argmax"] = np.array([m.forward_argmax([t], pos0=args.prompt + i) for i, t in enumerate(toks)], dtype=np.int32)
    # ForwardBatch: two sequences with different prompts, one step, against each run alone
    s1, s2 = m.new_sequence(), m.new_sequence()
    m.forward(prompt[:7], seq=s1)
    m.forward(prompt[3:20], seq=s2)
    res["batch"] = m.forward_batch([s1, s2], [11, 22]).copy()
    a1, a2 = m.new_sequence(), m.new_sequence()
    m.forward(prompt[:7], seq=a1)
    m.forward(prompt[3:20], seq=a2)
    res["single"] = np.stack([m.forward([11], pos0=7, seq=a1), m.forward([22], pos0=17, seq=a2)])
    np.savez(os.path.join(args.out, f"rank{rank}.npz"), **res)
    for s in (s1, s2, a1, a2):
        s.close()
    m.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
