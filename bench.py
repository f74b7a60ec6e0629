"""Benchmark: decode tokens/s of the Llama-3.3-70B-shaped Q4_K_M decoder (HBM-resident), batch 1.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--prompt P] [--impl windlass|reference]

One step is one decode token (batch 1) through every layer and the output head. The weights are the synthetic
N(0, 0.02) decoder of that shape generated on the device (wl_open_synthetic; no checkpoint exists offline), 39.5 GB
per step, which is far larger than the 126 MB L2, so no flush is needed between steps.

- value: K device-resident decode steps (wl_bench_decode: no host copies) timed with CUDA events on the model's
  stream, max over ranks. With N GPUs (torchrun, one process per GPU) the one model is split over the N GPUs by
  tensor parallelism (rows of q/k/v, gate/up and the head; columns of o and down; two NCCL all-reduces per layer
  over NVLink), so the work per step is fixed and N only shortens it (scaling "strong").
- e2e: the same steps through the public call a greedy host makes (wl_forward_argmax / wl_forward_batch_argmax:
  host token ids in, each row's greedy id back, fed to the next step), with the logits-returning wl_forward and the
  device-chained wl_generate_greedy beside it.
- roofline: the dominant kernel (the Q4_K fused dequant-matvec): the step's own Q4_K launches replayed alone as a
  CUDA graph (wl_bench_matvecs), their algorithmic bytes per step over their CUDA-event time per step.
- cpu_baseline: the reference's CPU arithmetic (the C oracle) on the box's cores, one decoder layer of the same
  shape plus a slice of the output head, scaled to a whole token.
--impl reference prints the CPU arm alone (rank 0; other ranks exit 0).
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tok/s @70B-shape Q4_K_M b1/b8; Q4_K matvec HBM GB/s vs ~8 TB/s"
Q4_K, Q6_K = 12, 14
LAYER_BYTES_70B = 483.5e6   # per decoder layer: q, k, o, gate, up, down Q4_K + v Q6_K


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d.get("hbm_gbs", 6650.0), d.get("bf16_tflops", 1590.0), "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms during the timed region."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.rows = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, ValueError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def __exit__(self, *a):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return None
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if len(r) > 5 + i and r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


def cpu_baseline(seconds=12.0, threads=0):
    """The oracle (the reference's CPU arithmetic) on one 70B-shape decoder layer at T=1 and a 16384-row slice of
    the Q6_K output head, timed with all host threads; returns tok/s for a whole token (80 layers + full head)."""
    from oracle import oracle as O
    from windlass_b200.transformer import llama70b_spec
    spec = llama70b_spec()
    spec.vocab = 16384
    m = O.Model(synth=spec, build_layers=1, max_context=64, threads=threads)
    cores = threads or O.lib().or_default_threads()
    x = (0.02 * __import__("numpy").random.default_rng(0).standard_normal(8192)).astype("float32")
    m.forward([1])                                       # warm
    side = m.new_sequence()
    t_layer, t_fwd, reps = [], [], 0
    t_end = time.perf_counter() + seconds
    pos = 1
    while time.perf_counter() < t_end and pos < 60:
        t0 = time.perf_counter()
        m.layer(0, x.copy(), pos0=pos - 1, seq=side)
        t_layer.append(time.perf_counter() - t0)
        t0 = time.perf_counter()
        m.forward([5], pos0=pos)
        t_fwd.append(time.perf_counter() - t0)
        pos += 1
        reps += 1
    tl, tf = min(t_layer), min(t_fwd)
    t_head_slice = max(tf - tl, 0.0)
    t_token = 80 * tl + t_head_slice * (128256 / 16384)
    m.close()
    return {"value": 1.0 / t_token, "unit": "tok/s", "cores": cores, "kind": "port",
            "sample": f"C oracle (reference CPU arithmetic), {cores} threads: one 70B-shape decoder layer at T=1 "
                      f"({tl * 1e3:.1f} ms, best of {reps}) x 80 + a 16384-row slice of the Q6_K output head scaled to "
                      f"128256 rows ({t_head_slice * 1e3:.1f} ms x {128256 / 16384:.2f})",
            "layer_ms": tl * 1e3, "weights_gbs": LAYER_BYTES_70B / tl / 1e9}


def reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    per_step = []
    for i in range(args.warmup + args.steps):
        r = cpu_baseline(seconds=2.0)
        if i >= args.warmup:
            per_step.append(1.0 / r["value"])
    value = args.steps / sum(per_step)
    out = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": args.gpus,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * sum(per_step) / args.steps,
           "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "q4_K/f32", "data": "synthetic",
           "config": {"workload": "decode b1, Llama-3.3-70B-shaped Q4_K_M (configs[3] b), the reference's CPU "
                                  "arithmetic (C oracle) on the host cores; each step's time is extrapolated from one "
                                  "decoder layer at T=1 x 80 plus a 16384-row slice of the output head scaled to "
                                  "128256 rows (the reference's TimeLayer method), not a whole decoded token",
                      "batch": 1, "prompt": args.prompt, "parallelism": "host cores (no GPU)",
                      "l2": "not applicable (CPU)"},
           "cpu_baseline": {"value": value, "unit": "tok/s", "cores": r["cores"], "kind": "port", "sample": r["sample"]},
           "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out))


def sweep_cpu_cell(fmt, t, raw, rows, cols, b, reps=3, max_s=20.0):
    """The reference's CPU arithmetic for one sweep cell, on all host threads: Transformer.MatMul of b columns
    (MatMulEach, one fused row kernel per column, for b <= 8, as a ForwardBatch step runs them; the decoded tile +
    FastMath.Block for b >= 64, as a prompt does; the I-quants have no fused dot and always take the tile path), best
    of `reps` like the reference's TimeLayer probe (src/Program.cs:493-527). Returns seconds."""
    import numpy as np
    from oracle import oracle as O
    x = np.random.default_rng(b).standard_normal((b, cols)).astype(np.float32)
    best = None
    t_end = time.perf_counter() + max_s
    for _ in range(reps):
        t0 = time.perf_counter()
        O.matmul(t, raw, rows, cols, x, each_token=b <= 8)
        dt = time.perf_counter() - t0
        best = dt if best is None else min(best, dt)
        if time.perf_counter() > t_end:
            break
    return best


def sweep_cell(f, R, K, b, ms, nbytes, hbm, bf16, raw0, t, args):
    """One row of the sweep table: the GPU time per call, its rates and fractions, and the CPU cell beside it."""
    alg = nbytes + 4 * b * (R + K)
    cell = {"format": f, "rows": R, "cols": K, "batch": b, "us": ms * 1e3,
            "gbs": alg / (ms / 1e3) / 1e9, "hbm_frac": alg / (ms / 1e3) / 1e9 / hbm,
            "tflops": 2.0 * R * K * b / (ms / 1e3) / 1e12,
            "bf16_frac": 2.0 * R * K * b / (ms / 1e3) / 1e12 / bf16}
    if raw0 is not None and (b <= 64 or R * K <= 8192 * 8192):
        cs_ = sweep_cpu_cell(f, t, raw0, R, K, b)
        cell["cpu_us"] = cs_ * 1e6
        cell["cpu_gbs"] = alg / cs_ / 1e9
        cell["cpu_gflops"] = 2.0 * R * K * b / cs_ / 1e9
    trace(f"{f} {R}x{K} b{b}: {ms * 1e3:.1f} us, {cell['gbs']:.0f} GB/s ({cell['hbm_frac']:.2f}), "
          f"{cell['tflops']:.2f} TFLOP/s" + (f"; CPU {cell['cpu_us'] / 1e3:.1f} ms" if "cpu_us" in cell else ""))
    return cell


def sweep(args):
    """the matvec/matmul sweep (8192 x 8192 by default; --shapes adds the 70B layer's shapes). Per shape,
    format and batch column count: the time of one call over rotating weight copies whose total exceeds L2, on weights
    repacked once into tiles (the model's layout). b <= 8: the decode matvec, launches back to back as in a decode step
    (wl_bench_matvec_tiles); b > 8: the tcgen05 GEMM for Q4_K and Q6_K (wl_gemm_tiles), the integer tensor-core matvec
    8 columns a launch for Q8_0, IQ4_XS and IQ2_XXS (wl_matvec_tiles); those from CUDA events around replays of a CUDA
    graph of `iters` calls. Then the weight
    bandwidth (b <= 8) or TFLOP/s (b >= 64), with the reference's CPU arithmetic (the C oracle, all host threads,
    best of 3) beside each cell. One JSON line with the whole table."""
    import ctypes as C
    import numpy as np
    import torch
    from windlass_b200 import _lib
    L = _lib.lib()
    shapes = [tuple(int(v) for v in sh.split("x")) for sh in args.shapes.split(",")] if args.shapes else \
        [(args.sweep_n, args.sweep_n)]
    fmts = args.formats.split(",")
    batches = [int(b) for b in args.batches.split(",")]
    stream = torch.cuda.current_stream()
    hbm, bf16, _ = measured_peaks()
    rows_out = []
    rng = np.random.default_rng(0)
    cpu_threads = None
    if not args.no_cpu:
        from oracle import oracle as O
        cpu_threads = O.lib().or_default_threads()
    for (R, K) in shapes:
        for f in fmts:
            t = _lib.TYPES[f]
            bs, ts = {"q4_K": (256, 144), "q6_K": (256, 210), "q8_0": (32, 34), "iq4_xs": (256, 136),
                      "iq2_xxs": (256, 66)}[f]
            nbytes = R * K // bs * ts
            copies = max(4, int(np.ceil(4 * 126e6 / nbytes)))
            ws = []
            raw0 = None
            for k in range(copies):
                buf = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
                if f in ("q4_K", "q6_K", "q8_0"):
                    _lib.check(L.wl_synth_tensor(t, 42 + k, 0x7001, R, K, C.c_float(0.02), C.c_float(0.0),
                                                 C.c_void_p(buf.data_ptr()), C.c_void_p(stream.cuda_stream)))
                else:   # the reference's random-payload method: random bytes with a fixed fp16 scale in each block
                    raw = rng.integers(0, 256, nbytes, dtype=np.uint8).reshape(-1, ts)
                    raw[:, 0], raw[:, 1] = 0x00, 0x1C          # fp16 0.0039
                    buf.copy_(torch.from_numpy(raw.reshape(-1)))
                ws.append(buf)
            if not args.no_cpu:
                torch.cuda.synchronize()
                raw0 = ws[0].cpu().numpy()
            tiled = f in ("q4_K", "q6_K", "q8_0", "iq4_xs", "iq2_xxs")
            if tiled:       # the model's layout: weights repacked once into tiles, so no call repacks
                tb = C.c_int64()
                _lib.check(L.wl_tiles_size(t, R, K, C.byref(tb)))
                tws = []
                for w in ws:
                    tw = torch.empty(tb.value, dtype=torch.uint8, device="cuda")
                    _lib.check(L.wl_make_tiles(t, C.c_void_p(w.data_ptr()), R, K, C.c_void_p(tw.data_ptr()),
                                               C.c_void_p(stream.cuda_stream)))
                    tws.append(tw)
                torch.cuda.synchronize()
            for b in batches:
                x = torch.randn(b, K, device="cuda")
                y = torch.empty(b, R, device="cuda")
                if b <= 8 and tiled:
                    # the decode matvec as it runs inside a step: launches back to back over rotating copies, one
                    # CUDA graph (wl_bench_matvec_tiles), activations prepared once
                    arr = (C.c_void_p * len(tws))(*[tw.data_ptr() for tw in tws])
                    dms = C.c_double()
                    n_it = args.iters * 5
                    _lib.check(L.wl_bench_matvec_tiles(t, arr, len(tws), R, K, C.c_void_p(x.data_ptr()), b,
                                                       C.c_void_p(y.data_ptr()), n_it, C.byref(dms),
                                                       C.c_void_p(stream.cuda_stream)))
                    ms = dms.value / n_it
                    rows_out.append(sweep_cell(f, R, K, b, ms, nbytes, hbm, bf16, raw0, t, args))
                    continue

                def run(i, mode):
                    w = ws[i % copies]
                    cs = C.c_void_p(torch.cuda.current_stream().cuda_stream)
                    if mode == "gemm":     # the tcgen05 GEMM on the repacked weights
                        st = L.wl_gemm_tiles(t, C.c_void_p(tws[i % copies].data_ptr()), R, K,
                                             C.c_void_p(x.data_ptr()), b, C.c_void_p(y.data_ptr()), cs)
                    elif mode == "tiles":  # the integer tensor-core matvec, 8 columns a launch, on the repacked weights
                        st = L.wl_matvec_tiles(t, C.c_void_p(tws[i % copies].data_ptr()), R, K,
                                               C.c_void_p(x.data_ptr()), b, C.c_void_p(y.data_ptr()), cs)
                    elif b <= 8:
                        st = L.wl_matvec(t, C.c_void_p(w.data_ptr()), R, K, C.c_void_p(x.data_ptr()), b,
                                         C.c_void_p(y.data_ptr()), cs)
                    else:
                        st = L.wl_matmul(t, C.c_void_p(w.data_ptr()), R, K, C.c_void_p(x.data_ptr()), b,
                                         C.c_void_p(y.data_ptr()), 0, cs)
                    _lib.check(st)

                def timed(mode):
                    for i in range(max(args.warmup, 3)):
                        run(i, mode)
                    torch.cuda.synchronize()
                    # the calls are captured into one CUDA graph so that host launch overhead is not what gets timed
                    graph = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(graph):
                        for i in range(args.iters):
                            run(i, mode)
                    graph.replay()
                    torch.cuda.synchronize()
                    reps = 5
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record(stream)
                    for _ in range(reps):
                        graph.replay()
                    e1.record(stream)
                    torch.cuda.synchronize()
                    del graph
                    return e0.elapsed_time(e1) / (reps * args.iters)

                paths = {}
                if tiled and f in ("q4_K", "q6_K"):
                    # both prompt paths; the library takes the GEMM from gemm_min_rows rows on (81 Q4_K, 57 Q6_K)
                    paths["gemm"] = timed("gemm")
                    paths["tiles"] = timed("tiles")
                    lib_path = "gemm" if b >= {"q4_K": 81, "q6_K": 57}[f] else "tiles"
                else:
                    lib_path = "tiles" if tiled else "raw"
                    paths[lib_path] = timed(lib_path)
                ms = paths[lib_path]
                cell = sweep_cell(f, R, K, b, ms, nbytes, hbm, bf16, raw0, t, args)
                cell["path"] = {"gemm": "tcgen05 GEMM", "tiles": "integer tensor-core matvec, 8 columns a launch",
                                "raw": "wl_matvec / wl_matmul"}[lib_path]
                for k_, v_ in paths.items():
                    cell[k_ + "_us"] = v_ * 1e3
                rows_out.append(cell)
                continue
                rows_out.append(sweep_cell(f, R, K, b, ms, nbytes, hbm, bf16, raw0, t, args))
            del ws
            if tiled:
                del tws
            torch.cuda.empty_cache()
    print(json.dumps({"metric": "Q4_K matvec HBM GB/s (configs[1] sweep)", "unit": "GB/s", "shapes": shapes,
                      "table": rows_out, "peak_hbm_gbs": hbm, "peak_bf16_tflops": bf16,
                      "cpu": {"kind": "port", "cores": cpu_threads, "method": "C oracle Transformer.MatMul, best of 3"}
                      if cpu_threads else None}))


def streamed(args):
    """configs[3] (a): the 70B-shape decoder with its layers streamed from pinned host memory on one GPU
    (wl_options.resident = 0). Per decode step every layer's weights and the head cross PCIe once; the bound is the
    host-to-device copy rate, measured in the same run (a 1 GiB pinned-to-device copy). One JSON line."""
    import numpy as np
    import torch
    from windlass_b200.transformer import CudaTransformer, llama70b_spec
    torch.cuda.set_device(0)
    src = torch.empty(1 << 30, dtype=torch.uint8, pin_memory=True)
    dst = torch.empty(1 << 30, dtype=torch.uint8, device="cuda")
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    dst.copy_(src, non_blocking=True)
    best = 1e30
    for _ in range(3):
        e0.record()
        dst.copy_(src, non_blocking=True)
        e1.record()
        torch.cuda.synchronize()
        best = min(best, e0.elapsed_time(e1))
    h2d_gbs = (1 << 30) / (best / 1e3) / 1e9
    del src, dst
    from windlass_b200.transformer import llama8b_spec
    spec = llama8b_spec() if args.model == "8b" else llama70b_spec(layers=args.layers or 80)
    path = None
    if args.stream_file:
        # the model as a GGUF file (written here from the synthetic generator), every stage read from it at each use
        import tempfile
        from windlass_b200 import gguf_writer
        tmpdir = tempfile.mkdtemp(prefix="wl_stream_")
        path = os.path.join(tmpdir, "model.gguf")
        t0 = time.perf_counter()
        file_bytes = gguf_writer.write(path, spec)
        trace(f"wrote {file_bytes / 1e9:.2f} GB to {path} in {time.perf_counter() - t0:.1f} s")
    t0 = time.perf_counter()
    trace(f"opening the streamed model ({spec.layers} layers)")
    if path:
        m = CudaTransformer(path, max_context=args.prompt + 64, resident=0, stream_file=1)
    else:
        m = CudaTransformer(synthetic=spec, max_context=args.prompt + 64, resident=0)
    load_s = time.perf_counter() - t0
    s = m.new_sequence()
    rng = np.random.default_rng(0)
    t0 = time.perf_counter()
    m.forward(rng.integers(0, spec.vocab, args.prompt).astype(np.int32), seq=s)
    prefill_s = time.perf_counter() - t0
    trace(f"loaded in {load_s:.1f} s, prefill {args.prompt} in {prefill_s:.1f} s")
    m.bench_decode([s], args.warmup)
    b0 = m.bytes_read
    ms = m.bench_decode([s], args.steps)
    moved = m.bytes_read - b0
    achieved = moved / (ms / 1e3) / 1e9
    shape = "8B" if args.model == "8b" else "70B"
    source = "read from the GGUF file at every use (stream_file)" if path else "streamed from pinned host memory"
    print(json.dumps({"metric": f"decode tok/s @{shape}-shape Q4_K_M b1, layers {source}"
                                + ("" if args.model == "8b" else " (configs[3] a)"),
                      "value": args.steps / (ms / 1e3), "unit": "tok/s",
                      "ms_per_step": ms / args.steps, "steps": args.steps, "warmup": args.warmup, "n_gpus": 1,
                      "h2d_bytes_per_step": moved / args.steps,
                      "roofline": {"bound": "storage" if path else "pcie", "achieved": achieved,
                                   "peak": None if path else h2d_gbs, "unit": "GB/s",
                                   "frac": None if path else achieved / h2d_gbs,
                                   "h2d_copy_gbs": h2d_gbs,
                                   "peak_source": "measured in this run: 1 GiB pinned host to device copy"},
                      "prefill_tok_s": args.prompt / prefill_s, "load_s": load_s}))
    s.close()
    m.close()
    if path:
        os.remove(path)
        os.rmdir(os.path.dirname(path))


def trace(msg):
    """Stage markers on stderr (the JSON line stays alone on stdout)."""
    sys.stderr.write(f"[bench {time.strftime('%H:%M:%S')}] {msg}\n")
    sys.stderr.flush()


def main():
    import faulthandler
    faulthandler.enable()
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=32)
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--prompt", type=int, default=1024)
    ap.add_argument("--layers", type=int, default=0, help="decoder layers (0: the configuration's own count)")
    ap.add_argument("--impl", default="windlass", choices=["windlass", "reference"])
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--tp-nccl-only", action="store_true", help="all-reduce with NCCL only (no fused peer-memory path)")
    ap.add_argument("--sweep", action="store_true", help="configs[1] matvec sweep instead of the decode benchmark")
    ap.add_argument("--sweep-n", type=int, default=8192)
    ap.add_argument("--formats", default="q4_K,q6_K,q8_0,iq4_xs,iq2_xxs")
    ap.add_argument("--batches", default="1,4,8,64,512")
    ap.add_argument("--shapes", default="", help="sweep shapes rows x cols, comma-separated (default: n x n)")
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--streamed", action="store_true", help="configs[3] (a): layers streamed from pinned host memory")
    ap.add_argument("--stream-file", action="store_true",
                    help="with --streamed: write the model as a GGUF file and read every stage from it at each use")
    ap.add_argument("--model", default="70b", choices=["70b", "8b", "moe"],
                    help="70b: configs[3] (the headline); 8b: configs[2]; moe: configs[4] (Qwen3-MoE shape)")
    ap.add_argument("--shard-of", type=int, default=0,
                    help="one GPU runs the shapes one rank holds under tensor parallelism over N GPUs (no exchange)")
    ap.add_argument("--profile-range", action="store_true",
                    help="bracket the timed steps with cudaProfilerStart/Stop (for ncu --profile-from-start off)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        return reference_arm(args)
    if args.sweep:
        return sweep(args)
    if args.streamed:
        return streamed(args)

    import datetime

    import numpy as np
    import torch

    from windlass_b200 import tp
    rank, world, local = tp.env_ranks()
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        # host plumbing only (group id, barriers, max over ranks); the model's collectives are its own NCCL group
        import torch.distributed as dist
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))

    def barrier():
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        torch.cuda.synchronize()

    from windlass_b200.transformer import llama70b_spec, llama8b_spec, qwen3moe_spec, synth_spec
    if args.model == "8b":
        spec = llama8b_spec()
        if args.layers:
            spec.layers = args.layers
    elif args.model == "moe":
        spec = qwen3moe_spec(layers=args.layers or 48)
    else:
        spec = llama70b_spec(layers=args.layers or 80)
    args.layers = spec.layers
    names = {"70b": "Llama-3.3-70B-shaped Q4_K_M (configs[3] b)", "8b": "Llama-3-8B-shaped Q4_K_M (configs[2])",
             "moe": "Qwen3-MoE-shaped, 128 experts top-8 (configs[4])"}
    if args.shard_of > 1:
        g = args.shard_of
        spec = synth_spec("llama", args.layers, 8192, 64 // g, 8 // g, 128, 28672 // g, 128256 // g, 8192,
                          rope_base=500000.0, type_attn_v=14, type_embd=12)
    steps, warm, B = args.steps, args.warmup, args.batch
    ctx = args.prompt + warm + 4 * steps + 80       # warm-up, timed, three e2e loops, the profiled pass
    t0 = time.perf_counter()
    trace(f"opening synthetic model, {args.layers} layers, context {ctx}, tensor parallel over {world} GPU(s)")
    m = tp.open_group_model(dist, local, synthetic=spec, max_context=ctx, tp_nccl_only=int(args.tp_nccl_only))
    allreduce = None
    if world > 1:
        allreduce = "fused into the o/down matvec and the next norm over NVLink peer memory" if m.info.tp_fused \
            else "NCCL ncclAllReduce"
    load_s = time.perf_counter() - t0
    rng = np.random.default_rng(0)          # every rank runs the same tokens
    seqs = [m.new_sequence() for _ in range(B)]
    trace(f"model ready in {load_s:.1f} s; prefill {B} x {args.prompt}")
    t0 = time.perf_counter()
    for s in seqs:
        m.forward(rng.integers(0, spec.vocab, args.prompt).astype(np.int32), seq=s)
    torch.cuda.synchronize()
    prefill_s = time.perf_counter() - t0

    trace(f"prefill {prefill_s:.1f} s; warmup {warm} steps")
    m.bench_decode(seqs, warm)
    launches0 = m.stats().kernel_launches
    trace(f"kernel launches before the timed region: {launches0}")
    barrier()
    with ClockSampler(local) as clk:
        if args.profile_range:
            torch.cuda.profiler.start()
        ms = m.bench_decode(seqs, steps)
        barrier()
        if args.profile_range:
            torch.cuda.profiler.stop()
    launches = m.stats().kernel_launches - launches0
    ms_max = tp.max_over_ranks(dist, ms)
    value = steps * B / (ms_max / 1e3)

    trace(f"timed {steps} steps: {ms:.1f} ms")
    # e2e through the host-facing calls, every step's token ids in from host memory and its result back to host
    # memory. The headline is the greedy serving loop's call (wl_forward_argmax / wl_forward_batch_argmax: the id of
    # each row comes back and is the next step's token); beside it the logits-returning Forward (V floats per row
    # back, Sampler on the host) and, at b1, the device-chained greedy decode (wl_generate_greedy, ids read back
    # every 16 steps).
    toks = rng.integers(0, spec.vocab, B).astype(np.int32)
    ids = np.empty(B, dtype=np.int32)
    barrier()
    t0 = time.perf_counter()
    for _ in range(steps):
        if B == 1:
            toks[0] = m.forward_argmax(toks, pos0=seqs[0].length, seq=seqs[0], out=ids)
        else:
            toks = m.forward_batch_argmax(seqs, toks, out=ids).copy()
    barrier()
    e2e_s = time.perf_counter() - t0
    e2e = steps * B / tp.max_over_ranks(dist, e2e_s)
    out = np.empty(B * spec.vocab, dtype=np.float32)
    barrier()
    t0 = time.perf_counter()
    for _ in range(steps):
        if B == 1:
            m.forward(toks, pos0=seqs[0].length, seq=seqs[0], out=out)
        else:
            m.forward_batch(seqs, toks, out=out)
    barrier()
    e2e_logits = steps * B / tp.max_over_ranks(dist, time.perf_counter() - t0)
    e2e_chained = None
    if B == 1:
        barrier()
        t0 = time.perf_counter()
        got = m.generate_greedy(int(toks[0]), steps, chunk=16, seq=seqs[0])
        barrier()
        e2e_chained = len(got) / tp.max_over_ranks(dist, time.perf_counter() - t0)

    trace(f"e2e {e2e_s:.2f} s ({e2e:.1f} tok/s); logits-returning {e2e_logits:.1f} tok/s; chained {e2e_chained}")
    # live roofline of the dominant kernel: the step's own Q4_K matvec launches (same weights, shapes, pairings and
    # order) captured into a graph and replayed alone, timed with CUDA events on the model's stream
    barrier()
    mv_steps = min(steps, 16)
    mv_ms, mv_bytes = m.bench_matvecs(B, mv_steps)
    mv_ms = tp.max_over_ranks(dist, mv_ms)
    kernel_ms_per_step = mv_ms / mv_steps
    trace(f"Q4_K matvec launches alone: {kernel_ms_per_step:.3f} ms per step for {mv_bytes / 1e9:.2f} GB "
          f"(the whole step {ms_max / steps:.3f} ms)")
    hbm, _, peak_kind = measured_peaks()
    achieved = mv_bytes / (kernel_ms_per_step / 1e3) / 1e9
    traffic = None
    tfile = os.path.join(ROOT, "profiles", "q4k_matvec_traffic.txt")
    if os.path.exists(tfile):
        for line in open(tfile):
            if line.startswith("dram_bytes_per_byte_algorithmic"):
                traffic = float(line.split()[1]) * mv_bytes
    roofline = {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                "traffic": traffic, "traffic_scope": "per step (the step's Q4_K launches), from the DRAM bytes per "
                "algorithmic byte of an ncu capture of the step's launches (profiles/q4k_matvec_traffic.txt)",
                "kernel": "k_mmv_q4k (tensor-core Q4_K matvec)", "peak_source": peak_kind,
                "kernel_ms_per_step": kernel_ms_per_step, "bytes_per_step": mv_bytes,
                "timing": "the step's Q4_K matvec launches replayed alone as a CUDA graph (wl_bench_matvecs), "
                          "CUDA events; per GPU under tensor parallelism"}

    trace("kernel timing done")
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu and args.model == "70b" and not args.shard_of:
        cpu = cpu_baseline()
    trace("cpu baseline done")
    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": steps, "warmup": warm,
                "ms_per_step": ms_max / steps, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": "q4_K/q6_K weights, f32 compute", "data": "synthetic",
                "config": {"workload": (f"decode b{B}, one TP{args.shard_of} rank's shard of the Llama-3.3-70B-shaped "
                                        f"Q4_K_M decoder on one GPU (no exchange), {args.layers} layers")
                           if args.shard_of > 1 else
                           f"decode b{B}, {names[args.model]}, HBM-resident, {args.layers} layers",
                           "batch": B, "prompt": args.prompt,
                           "parallelism": f"tp{world}, all-reduce x2 per layer: {allreduce}" if world > 1 else "1 GPU",
                           "l2": "inputs larger than L2 (each step reads the layers' weights: 39.5 GB at 70B, 4.4 GB at 8B, "
                                 "1.8 GB or more for the MoE)"},
                "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": 4 * B, "d2h_bytes_per_step": 4 * B,
                        "call": "wl_forward_argmax" if B == 1 else "wl_forward_batch_argmax",
                        "logits_returning": {"value": e2e_logits, "call": "wl_forward" if B == 1 else
                                             "wl_forward_batch", "d2h_bytes_per_step": 4 * B * spec.vocab},
                        "device_chained": {"value": e2e_chained, "call": "wl_generate_greedy, chunk 16"}
                        if e2e_chained else None},
                "roofline": roofline, "cpu_baseline": cpu, "clocks": clk.summary(), "gpu_launches": launches,
                "load_s": load_s, "prefill_s": prefill_s,
                "prefill_tok_s": B * args.prompt / prefill_s}
        print(json.dumps(line))
    m.close()
    if dist:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
