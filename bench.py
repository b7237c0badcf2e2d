#!/usr/bin/env python
"""Batch-1 int8 decode throughput of the Qwen3.5-0.8B hybrid decoder on B200.

    python bench.py [--gpus N --steps K --warmup W] [--impl b200|reference]

Workload (config 0 of the build): random-init Qwen3.5-0.8B (seed 1234), a
16-token prompt (default_rng(0)) prefilled one token at a time (untimed), then
64 greedy decode steps (timed), repeated as "episodes" until K decode steps
have been timed.  A step is one decode_step: embed, 24 layers, tied head,
argmax.  Algorithmic bytes of a step attending T positions:
B(T) = 758,248,704 + 24,576 * T (int8 weights + row scales + fp32 small
tensors, plus fp32 K/V reads of the 6 attention layers).

Under torchrun (N > 1) the N ranks decode ONE sequence with tensor
parallelism (qwen_fpga_b200.tp: heads, FFN columns and the vocab split across
the GPUs, the row-parallel partial sums and the argmax exchanged inside the
decode kernel over NVLink); the throughput is that sequence's tokens/s
(strong scaling).  --replicas instead runs N independent sequences, one per
GPU, and sums their throughput (weak scaling).

--impl reference times the reference's own CPU decoder (the HLS C++ qwen_top
compiled from the reference sources into oracle/_ref, single thread) on a
bounded sample of the same workload; without that build it times the oracle
port (numpy restatement of golden/model.py) instead.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "batch-1 decode tokens/s (int8, ~0.76 GB/token) and achieved HBM GB/s vs peak"
UNIT = "tokens/s"
B_WEIGHTS = 758_248_704
KV_PER_POS = 24_576
STATE_RW = 41_287_680
PROMPT_LEN, EPISODE = 16, 64
VOCAB = 248320


def bytes_per_step(T):
    return B_WEIGHTS + KV_PER_POS * T


def peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    return 6650.0, "fallback 6.65 TB/s"


def prompt_ids():
    return np.random.default_rng(0).integers(0, VOCAB, PROMPT_LEN).astype(np.int32)


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id=None):
        self.gpu_id = gpu_id
        self.proc = None
        self.path = os.path.join("/tmp", f"qwen_b200_clocks_{os.getpid()}.csv")

    def __enter__(self):
        cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
               "-lms", "200"]
        if self.gpu_id is not None:
            cmd += ["-i", str(self.gpu_id)]
        self.cmd = cmd
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(cmd, stdout=self.fh, stderr=subprocess.DEVNULL)
            # the timed region starts once the sampler is producing rows
            t0 = time.time()
            while os.path.getsize(self.path) == 0 and time.time() - t0 < 3.0:
                time.sleep(0.02)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            # one more sample at the end of the region (a short region may fall
            # between the 200 ms ticks)
            try:
                one = [c for c in self.cmd if c not in ("-lms", "200")]
                self.fh.flush()
                subprocess.run(one, stdout=self.fh, stderr=subprocess.DEVNULL, timeout=10)
            except Exception:
                pass
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.fh.close()

    def summary(self):
        if self.proc is None or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows), "power_w_max": max(float(r[3]) for r in rows
                                                         if r[3].replace(".", "").isdigit())}


def blas_threads():
    try:
        from threadpoolctl import threadpool_info
        n = [i.get("num_threads", 1) for i in threadpool_info() if i.get("user_api") == "blas"]
        return int(max(n)) if n else 1
    except Exception:
        return os.cpu_count() or 1


def cpu_baseline_port(blob_path, n_steps):
    """The oracle port (numpy restatement of golden/model.py) on this host's cores:
    16-token prefill untimed, then n_steps greedy decode steps timed."""
    from oracle import golden_port as P
    from qwen_fpga_b200 import synth
    cfg = synth.model_config()
    dec = P.PortDecoder(synth.Blob(blob_path).fake_quant(), cfg)
    st = P.PortState.zeros(cfg)
    lg = None
    for t in prompt_ids():
        lg = dec.step(int(t), st)
    t0 = time.perf_counter()
    for _ in range(n_steps):
        lg = dec.step(int(np.argmax(lg)), st)
    dt = time.perf_counter() - t0
    return {"value": n_steps / dt, "unit": UNIT, "cores": blas_threads(), "kind": "port",
            "sample": f"oracle port (numpy golden restatement), config0 prompt prefill untimed + "
                      f"{n_steps} greedy decode steps timed"}


def cpu_reference_hls(blob_path, n_steps):
    """The reference's HLS C++ decoder (oracle/_ref), single thread, same sample shape."""
    from oracle import native
    ref = native.HlsRef(blob_path)
    am = 0
    for t in prompt_ids():
        am, _ = ref.step(int(t))
    t0 = time.perf_counter()
    for _ in range(n_steps):
        am, _ = ref.step(am)
    dt = time.perf_counter() - t0
    ref.close()
    return {"value": n_steps / dt, "unit": UNIT, "cores": 1, "kind": "reference",
            "sample": f"reference HLS C++ qwen_top (hls/src/qwen_synth.hpp, g++ -O2, 1 thread), "
                      f"config0 prompt prefill untimed + {n_steps} greedy decode steps timed"}


def load_traffic():
    p = os.path.join(REPO, "profiles", "traffic.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f)
    return None


def run_profile(args):
    """Target for ncu: build the context, then exactly args.profile decode steps."""
    from qwen_fpga_b200 import api, synth
    dec = api.Decoder(synth.ensure_blob(1234), max_ctx=PROMPT_LEN + args.profile + 8)
    dec.set_engine(args.engine)
    for t in prompt_ids()[:args.profile]:
        dec.decode_step(int(t), want_logits=False)
    dec.close()
    print("profile ok")
    return 0


def run_reference(args, rank):
    if rank != 0:
        return 0
    from qwen_fpga_b200 import synth
    blob_path = synth.ensure_blob(1234)
    from oracle import native
    n = max(1, min(args.steps, 32))
    if native.have_ref():
        cb = cpu_reference_hls(blob_path, n)
    else:
        cb = cpu_baseline_port(blob_path, n)
    line = {"impl": "reference", "metric": METRIC, "value": cb["value"], "unit": UNIT,
            "n_gpus": args.gpus, "steps": n, "warmup": 0, "ms_per_step": 1e3 / cb["value"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32 (int8 weights dequantised on the fly)", "data": "synthetic",
            "config": {"workload": "config0 (random-init Qwen3.5-0.8B, 16-token prompt, greedy)",
                       "batch": 1},
            "cpu_baseline": cb,
            "e2e": {"value": cb["value"], "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


GEMV_SHAPES = [(6144, 1024), (2048, 1024), (7168, 1024), (1024, 3584), (1024, 2048), (4096, 1024),
               (248320, 1024)]


def run_gemv(args):
    """Config 1 (GEMV microbench): qwen_gemv_i8_i8 on every shape, W int8
    rng.integers(-127, 128), scales U[1e-3, 1e-2], x int8 U[-127, 127] with s_x
    U[1e-3, 1e-2], seed 0 per shape.  Bytes per call = N*K + 4N + K + 4 + 4N
    (+ 4N for the int32 accumulators also written).  Each timed call reads a
    different copy of the weights, enough copies that a pass reads more than
    L2, so the weights come from HBM.  The int32 accumulators of one call per
    shape are checked against numpy exactly.  One JSON line."""
    import torch
    from qwen_fpga_b200 import api
    torch.cuda.set_device(0)
    peak, src = peaks()
    rows = []
    for N, K in GEMV_SHAPES:
        if args.gemv_n and N != args.gemv_n:
            continue
        rng = np.random.default_rng(0)
        w = rng.integers(-127, 128, (N, K), dtype=np.int8)
        sw = rng.uniform(1e-3, 1e-2, N).astype(np.float32)
        xq = rng.integers(-127, 128, K, dtype=np.int8)
        sx = float(rng.uniform(1e-3, 1e-2))
        ncopy = max(1, min(128, -(-(256 << 20) // (N * K))))    # > 2x L2 (126 MB) per pass
        ws = [torch.from_numpy(w).cuda() for _ in range(ncopy)]
        dsw, dxq = torch.from_numpy(sw).cuda(), torch.from_numpy(xq).cuda()
        acc = torch.empty(N, dtype=torch.int32, device="cuda")
        y = torch.empty(N, dtype=torch.float32, device="cuda")
        api.gemv_i8_i8(ws[0], dsw, dxq, sx, acc=acc, y=y)
        torch.cuda.synchronize()
        ref = w.astype(np.int64) @ xq.astype(np.int64)
        exact = bool(np.array_equal(acc.cpu().numpy().astype(np.int64), ref))
        # one pass over every copy, captured once as a CUDA graph so that host
        # launch overhead stays out of the timed region
        st = torch.cuda.Stream()
        n = max(8, ncopy)
        with torch.cuda.stream(st):
            for i in range(max(args.warmup, 3)):
                api.gemv_i8_i8(ws[i % ncopy], dsw, dxq, sx, acc=acc, y=y, stream=st)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            for i in range(n):
                api.gemv_i8_i8(ws[i % ncopy], dsw, dxq, sx, acc=acc, y=y, stream=st)
        reps = 3
        with torch.cuda.stream(st):
            g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        with torch.cuda.stream(st):
            for _ in range(reps):
                g.replay()
        e1.record(st)
        torch.cuda.synchronize()
        n *= reps
        us = e0.elapsed_time(e1) * 1e3 / n
        nbytes = N * K + 4 * N + K + 4 + 4 * N + 4 * N
        gbs = nbytes / (us * 1e-6) / 1e9
        rows.append({"N": N, "K": K, "us": round(us, 3), "bytes": nbytes, "GB_s": round(gbs, 1),
                     "frac": round(gbs / peak, 4), "acc_exact": exact, "weight_copies": ncopy})
        del ws
        torch.cuda.empty_cache()
    print(json.dumps({"metric": "config-1 int8 GEMV achieved HBM GB/s", "unit": "GB/s", "peak": peak,
                      "peak_source": src, "kernel": "k_gemv (qwen_gemv_i8_i8)", "shapes": rows}))
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64 * 64, help="timed decode steps (multiple of 64)")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--e2e-episodes", type=int, default=8)
    ap.add_argument("--cpu-steps", type=int, default=24)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--replicas", action="store_true",
                    help="N > 1: independent sequences per GPU instead of tensor parallelism")
    ap.add_argument("--engine", type=int, default=1,
                    help="1 = persistent weight-streaming kernel, 0 = graph of phase kernels")
    ap.add_argument("--gemv", action="store_true", help="config-1 GEMV microbench (one JSON line)")
    ap.add_argument("--gemv-n", type=int, default=0, help="with --gemv: only the shape with this N")
    ap.add_argument("--profile", type=int, default=0,
                    help="run N decode steps of the config-0 prompt (no timing, no JSON) for ncu")
    args = ap.parse_args()
    if args.profile:
        return run_profile(args)
    if args.gemv:
        return run_gemv(args)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank)

    import torch
    import torch.distributed as dist
    from datetime import timedelta

    from qwen_fpga_b200 import api, synth

    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(minutes=10))
    if rank == 0:
        blob_path = synth.ensure_blob(1234)
    if world > 1:
        dist.barrier()
    blob_path = synth.ensure_blob(1234)

    episodes = max(1, args.steps // EPISODE)
    K = episodes * EPISODE
    tp = world > 1 and not args.replicas
    if tp:
        from qwen_fpga_b200.tp import TPDecoder
        tpd = TPDecoder(blob_path, device=local, max_ctx=PROMPT_LEN + EPISODE + 64)
        dec = tpd.dec
    else:
        dec = api.Decoder(blob_path, device=local, max_ctx=PROMPT_LEN + EPISODE + 64)
        dec.set_engine(args.engine)
    engine = dec.engine
    seqs = 1 if tp else world   # sequences decoded by the whole job
    launches_per_step = 1 if engine == 1 else 24 * 5 + 2
    kernel_name = ("k_decode_persistent (one cooperative launch per step)" if engine == 1
                   else "whole decode step (CUDA graph of 122 kernels)")
    prompt = prompt_ids()

    # warm-up: W untimed steps
    dec.reset()
    if world > 1:
        dist.barrier()
    dec.generate(prompt[:1], max(args.warmup, 3))

    # timed: K decode steps in episodes of (16-token prefill untimed, 64 decode timed)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    dev_sec = 0.0
    ids0 = None
    with ClockSampler(local if world == 1 else local) as clk:
        for e in range(episodes):
            dec.reset()
            if tp:
                dist.barrier()
            ids, sec = dec.generate(prompt, EPISODE)
            dev_sec += sec
            if ids0 is None:
                ids0 = ids
            elif ids != ids0:
                raise RuntimeError("episodes produced different tokens")
    torch.cuda.synchronize()
    if world > 1:
        t = torch.tensor([dev_sec], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dev_sec = float(t.item())
        dist.barrier()
    ms_per_step = dev_sec / K * 1e3
    value = seqs * K / dev_sec

    # end to end through the C ABI: host token in, host argmax out, every step
    e2e_sec = 0.0
    e2e_steps = 0
    for e in range(max(1, args.e2e_episodes)):
        dec.reset()
        if tp:
            dist.barrier()
        am = 0
        for t in prompt:
            am, _ = dec.decode_step(int(t), want_logits=False)
        t0 = time.perf_counter()
        for _ in range(EPISODE):
            am, _ = dec.decode_step(am, want_logits=False)
        e2e_sec += time.perf_counter() - t0
        e2e_steps += EPISODE
    # with the fp32 logits returned to host memory each step (what golden decode_step returns;
    # under TP each rank returns its vocab slice)
    dec.reset()
    if tp:
        dist.barrier()
    am = 0
    for t in prompt:
        am, _ = dec.decode_step(int(t), want_logits=False)
    t0 = time.perf_counter()
    for _ in range(EPISODE):
        am, lg = dec.decode_step(am, want_logits=True)
    lg_sec = time.perf_counter() - t0
    if world > 1:
        t = torch.tensor([e2e_sec, lg_sec], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_sec, lg_sec = (float(v) for v in t.tolist())
    if world > 1:
        dist.barrier()   # every rank's last step is done before any context goes away
    dec.close()

    clocks = clk.summary()
    if rank != 0:
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return 0

    peak, peak_src = peaks()
    t_mean = PROMPT_LEN + 1 + (EPISODE - 1) / 2.0
    bstep = bytes_per_step(t_mean)
    achieved = bstep / (ms_per_step * 1e-3) / 1e9
    if tp:
        peak = peak * world   # one step's bytes are spread over every rank's HBM
        peak_src = f"{peak_src} x {world} GPUs (aggregate)"
    traffic = load_traffic()
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": K,
        "warmup": max(args.warmup, 3), "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "strong" if tp else "weak", "vs_baseline": None,
        "dtype": "int8 weights x fp32 activations -> int32 digit accumulators",
        "data": "synthetic (random-init Qwen3.5-0.8B, seed 1234)",
        "config": {"workload": "config0: 16-token prompt prefill (untimed) + 64 greedy decode "
                               "steps (timed), repeated", "model": "Qwen3.5-0.8B (random init)",
                   "batch": 1, "global_batch": seqs, "episodes": episodes,
                   "T_ctx": f"{PROMPT_LEN + 1}..{PROMPT_LEN + EPISODE}",
                   "l2": "no flush: 758 MB of weights per step > 126 MB L2",
                   "parallelism": ("1 GPU" if world == 1 else
                                   f"tp{world} (tensor parallel, one sequence)" if tp else
                                   f"{world} independent replicas")},
        "e2e": {"value": seqs * e2e_steps / e2e_sec, "unit": UNIT, "h2d_bytes_per_step": 44,
                "d2h_bytes_per_step": 20,
                "with_logits": {"value": seqs * EPISODE / lg_sec, "unit": UNIT,
                                "d2h_bytes_per_step": 20 + 4 * VOCAB}},
        "gpu_launches": K * launches_per_step,
        "engine": "persistent" if engine == 1 else "graph",
        "roofline": {"bound": "hbm", "kernel": kernel_name,
                     "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_source": peak_src,
                     "algorithmic_bytes_per_step": bstep,
                     "state_bytes_per_step": STATE_RW,
                     # the ncu capture is of the single-GPU kernel
                     "traffic": traffic.get("bytes_per_step") if traffic and not tp else None},
        "clocks": clocks,
    }
    if world == 1 and not args.no_cpu:
        try:
            line["cpu_baseline"] = cpu_baseline_port(blob_path, args.cpu_steps)
        except Exception as exc:  # the CPU leg never hides the GPU number
            line["cpu_baseline"] = {"value": None, "error": str(exc)}
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
