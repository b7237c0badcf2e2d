#!/usr/bin/env python
"""Batch-1 int8 decode throughput of the Qwen3.5-0.8B hybrid decoder on B200.

    python bench.py [--gpus N --steps K --warmup W] [--impl b200|reference]

Headline workload (config 0 of the build): random-init Qwen3.5-0.8B (seed
1234), a 16-token prompt (default_rng(0)) prefilled one token at a time
(untimed), then greedy decode steps (timed) in episodes of at most 64, until
exactly K decode steps have been timed.  A step is one decode_step: embed, 24
layers, tied head, argmax.  Algorithmic bytes of a step attending T positions:
B(T) = 758,248,704 + 24,576 * T (int8 weights + row scales + fp32 small
tensors, plus fp32 K/V reads of the 6 attention layers).

The same JSON line carries the other configs as sub-objects (each a stated
sample of its workload): "gemv" (config 1: every int8 GEMV microbench shape,
GB/s against the HBM peak, int32 accumulators checked exactly), "config2"
(W8A8 warm start, 4096 cached positions, 256 greedy steps), "config3"
(W8A32, 32768 cached positions, 512 greedy steps) and "config4" (batched
decode: 64 sequences, each with its own 2048-position warm start and DeltaNet
state, W8A8 projections on the tcgen05 tensor cores; a stated sample of the
128 greedy steps).

Under torchrun (N > 1) the N ranks decode ONE sequence with tensor
parallelism (qwen_fpga_b200.tp: heads, FFN columns and the vocab split across
the GPUs, the row-parallel partial sums and the argmax exchanged inside the
decode kernel over NVLink); the throughput is that sequence's tokens/s
(strong scaling).  --replicas instead runs N independent sequences, one per
GPU, and sums their throughput (weak scaling).

--impl reference times the reference's CPU decode path on the host cores, on
a bounded sample of the same workload: the numpy decode step of
golden/model.py (through its restatement oracle/golden_port.py, pinned to the
golden's own outputs; the reference's Python cannot travel to the GPU box)
with every BLAS thread, and beside it the reference's HLS C++ decoder
(qwen_top, compiled from the reference sources into oracle/_ref), which is
single-threaded by construction.
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


def load_tensor_pipe():
    """Tensor-pipe utilisation of the batched GEMMs from the committed ncu
    summary (profiles/k_bt_gemm_config4.json), or None."""
    p = os.path.join(REPO, "profiles", "k_bt_gemm_config4.json")
    try:
        with open(p) as f:
            return json.load(f)
    except (OSError, ValueError):
        return None


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
    for t in prompt_ids()[:args.profile]:
        dec.decode_step(int(t), want_logits=False)
    dec.close()
    print("profile ok")
    return 0


def run_profile_c4(args):
    """Target for ncu: a config-4 batched context (args.c4_batch sequences,
    four distinct 2048-position warm starts), one step with host tokens, then
    args.profile_c4 greedy steps."""
    from qwen_fpga_b200 import api, synth
    B = args.c4_batch
    bd = api.BatchDecoder(synth.ensure_blob(1234), max_batch=B, max_ctx=C4_T0 + args.profile_c4 + 16,
                          act_int8=True)
    for i in range(4):
        st = synth.warm_state_arrays(C4_T0, 40 + i)
        for b in range(i, B, 4):
            bd.import_state(b, st)
    am, _ = bd.step([int(np.random.default_rng(100 + b).integers(0, VOCAB)) for b in range(B)])
    for _ in range(args.profile_c4):
        am, _ = bd.step_greedy(B)
    bd.close()
    print("profile ok")
    return 0


def run_reference(args, rank):
    """The reference arm: rank 0 alone times the reference's CPU decode path on a
    bounded sample of config 0 (see the module docstring); other ranks exit."""
    if rank != 0:
        return 0
    from qwen_fpga_b200 import synth
    blob_path = synth.ensure_blob(1234)
    from oracle import native
    n = max(1, min(args.steps, 32))
    cb = cpu_baseline_port(blob_path, n)
    hls = None
    if native.have_ref():
        hls = cpu_reference_hls(blob_path, max(1, min(args.steps, 16)))
    line = {"impl": "reference", "metric": METRIC, "value": cb["value"], "unit": UNIT,
            "n_gpus": args.gpus, "steps": n, "warmup": 0, "ms_per_step": 1e3 / cb["value"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32 (int8 weights dequantised, golden fake-quant)", "data": "synthetic",
            "config": {"workload": "config0 (random-init Qwen3.5-0.8B, 16-token prompt prefill "
                                   "untimed, greedy decode steps timed)", "batch": 1},
            "cpu_baseline": cb,
            "hls_reference": hls,
            "e2e": {"value": cb["value"], "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


GEMV_SHAPES = [(6144, 1024), (2048, 1024), (7168, 1024), (1024, 3584), (1024, 2048), (4096, 1024),
               (248320, 1024)]


def gemv_rows(warmup=3, only_n=0):
    """Config 1 (GEMV microbench): qwen_gemv_i8_i8 on every shape, W int8
    rng.integers(-127, 128), scales U[1e-3, 1e-2], x int8 U[-127, 127] with s_x
    U[1e-3, 1e-2], seed 0 per shape.  Bytes per call = N*K + 4N + K + 4 + 4N
    (+ 4N for the int32 accumulators also written).  Each timed call reads a
    different copy of the weights, enough copies that a pass reads more than
    L2, so the weights come from HBM.  The int32 accumulators of one call per
    shape are checked against numpy exactly."""
    import torch
    from qwen_fpga_b200 import api
    peak, _ = peaks()
    rows = []
    for N, K in GEMV_SHAPES:
        if only_n and N != only_n:
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
            for i in range(max(warmup, 3)):
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
        del ws, g
        torch.cuda.empty_cache()
    return rows


def run_gemv(args):
    """--gemv: the config-1 rows alone, one JSON line."""
    import torch
    torch.cuda.set_device(0)
    peak, src = peaks()
    rows = gemv_rows(args.warmup, args.gemv_n)
    print(json.dumps({"metric": "config-1 int8 GEMV achieved HBM GB/s", "unit": "GB/s", "peak": peak,
                      "peak_source": src, "kernel": "k_gemv (qwen_gemv_i8_i8)", "shapes": rows}))
    return 0


def timed_decode(dec, prompt, steps, tp=False, dist=None):
    """Exactly `steps` greedy decode steps timed on the device (CUDA events in
    qwen_generate), in episodes of the prompt prefill (untimed) + at most
    EPISODE decode steps.  Returns (device seconds, tokens of the first episode)."""
    sec_total, done, ids0 = 0.0, 0, None
    while done < steps:
        n = min(EPISODE, steps - done)
        dec.reset()
        if tp:
            dist.barrier()
        ids, sec = dec.generate(prompt, n)
        sec_total += sec
        if ids0 is None:
            ids0 = ids
        elif ids != ids0[:len(ids)]:
            raise RuntimeError("episodes produced different tokens")
        done += n
    return sec_total, ids0


# config 4 (batched decode): per step, every sequence reads its KV (T positions
# x 6 layers x K and V x 2 heads x 256 fp32) and reads + writes its DeltaNet
# state (18 x 16 x 128 x 128 fp32 + conv history); the weights are read once
# for the whole batch
C4_BATCH, C4_T0 = 64, 2048
C4_STATE = 2 * (18 * 16 * 128 * 128 * 4) + 2 * (18 * 6144 * 4)


def c4_bytes_per_step(B, T):
    return B_WEIGHTS + B * (KV_PER_POS * T + C4_STATE)


def config4(blob_path, device, steps, warmup, B=C4_BATCH, T0=C4_T0):
    """Config 4: B sequences with 2048-position warm starts (four distinct
    synth.warm_state_arrays draws, seeds 40-43, each imported into B/4 slots),
    first tokens default_rng(100 + b); one untimed step, `warmup` untimed
    greedy steps, then `steps` greedy steps timed on the device
    (qwen_decode_timed: tokens fed back on the device), then the same number
    end to end through qwen_decode_step (host tokens in, host argmax out)."""
    from qwen_fpga_b200 import api, synth
    n_e2e = steps
    bd = api.BatchDecoder(blob_path, max_batch=B, device=device,
                          max_ctx=T0 + 1 + warmup + steps + n_e2e + 8, act_int8=True)
    try:
        for i in range(4):
            st = synth.warm_state_arrays(T0, 40 + i)
            for b in range(i, B, 4):
                bd.import_state(b, st)
            del st
        first = [int(np.random.default_rng(100 + b).integers(0, VOCAB)) for b in range(B)]
        am, _ = bd.step(first)
        bd.timed(B, warmup)
        t_mean = T0 + 1 + warmup + (steps - 1) / 2.0
        sec = bd.timed(B, steps)
        t0 = time.perf_counter()
        for _ in range(n_e2e):
            am, _ = bd.step(am)
        e2e_sec = time.perf_counter() - t0
    finally:
        bd.close()
    bstep = c4_bytes_per_step(B, t_mean)
    return {"sec": sec, "steps": steps, "bytes_per_step": bstep, "e2e_sec": e2e_sec, "e2e_steps": n_e2e,
            "t_mean": t_mean, "B": B}


def warm_config(dec, T0, seed, n_steps, act_int8, tp=False, dist=None):
    """Configs 2 and 3: import the warm start (synth.warm_state_arrays: rec
    N(0, 0.1), T0 cached positions N(0, 1), the fixtures' recipe), feed the
    first token (default_rng(0), untimed), then time n_steps greedy steps."""
    from qwen_fpga_b200 import synth
    st = synth.warm_state_arrays(T0, seed)
    first = int(np.random.default_rng(0).integers(0, VOCAB))
    dec.reset()
    dec.set_act_int8(act_int8)
    try:
        dec.import_state(st)
        del st
        if tp:
            dist.barrier()
        ids, sec = dec.generate([first], n_steps)
    finally:
        dec.set_act_int8(False)
    t_mean = T0 + 1 + (n_steps - 1) / 2.0
    return sec, ids, t_mean


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64 * 64, help="timed decode steps (exactly)")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--e2e-episodes", type=int, default=4)
    ap.add_argument("--cpu-steps", type=int, default=24)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--configs", default="1,2,3,4",
                    help="extra configs measured into the same line (comma list of 1, 2, 3, 4; '' = none)")
    ap.add_argument("--c4-steps", type=int, default=32, help="config 4: timed steps (a sample of its 128)")
    ap.add_argument("--replicas", action="store_true",
                    help="N > 1: independent sequences per GPU instead of tensor parallelism")
    ap.add_argument("--gemv", action="store_true", help="config-1 GEMV microbench (one JSON line)")
    ap.add_argument("--gemv-n", type=int, default=0, help="with --gemv: only the shape with this N")
    ap.add_argument("--profile", type=int, default=0,
                    help="run N decode steps of the config-0 prompt (no timing, no JSON) for ncu")
    ap.add_argument("--profile-c4", type=int, default=0,
                    help="config 4 for ncu: one step, then N greedy steps of a batched context (no timing)")
    ap.add_argument("--c4-batch", type=int, default=C4_BATCH, help="config 4: sequences per GPU")
    args = ap.parse_args()
    if args.profile:
        return run_profile(args)
    if args.profile_c4:
        return run_profile_c4(args)
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

    K = max(1, args.steps)
    W = max(args.warmup, 3)
    configs = {c.strip() for c in args.configs.split(",") if c.strip()}
    tp = world > 1 and not args.replicas
    max_ctx = 32768 + 512 + 64 if "3" in configs else 4096 + 256 + 64
    if tp:
        from qwen_fpga_b200.tp import TPDecoder
        tpd = TPDecoder(blob_path, device=local, max_ctx=max_ctx)
        dec = tpd.dec
    else:
        dec = api.Decoder(blob_path, device=local, max_ctx=max_ctx)
    seqs = 1 if tp else world   # sequences decoded by the whole job
    launches_per_step = 1
    kernel_name = "k_decode_persistent (one cooperative launch per step)"
    prompt = prompt_ids()

    # warm-up: W untimed steps
    dec.reset()
    if world > 1:
        dist.barrier()
    dec.generate(prompt[:1], W)

    # timed: exactly K decode steps (episodes of 16-token prefill untimed + <= 64 decode timed)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        dev_sec, ids0 = timed_decode(dec, prompt, K, tp, dist)
    torch.cuda.synchronize()
    if world > 1:
        t = torch.tensor([dev_sec], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dev_sec = float(t.item())
        dist.barrier()
    ms_per_step = dev_sec / K * 1e3
    value = seqs * K / dev_sec

    # end to end through the C ABI, host token in and the step's result out
    # every step: with the fp32 logits (what golden decode_step returns; pinned
    # host buffer; under TP each rank returns its vocab slice), and argmax only
    lg_buf = torch.empty(VOCAB, dtype=torch.float32, pin_memory=True).numpy()
    e2e = {}
    for mode in ("logits", "argmax"):
        sec, nsteps = 0.0, 0
        for e in range(max(1, args.e2e_episodes)):
            dec.reset()
            if tp:
                dist.barrier()
            am = 0
            for t in prompt:
                am, _ = dec.decode_step(int(t), want_logits=False)
            t0 = time.perf_counter()
            for _ in range(EPISODE):
                if mode == "logits":
                    am, _ = dec.decode_step(am, out=lg_buf)
                else:
                    am, _ = dec.decode_step(am, want_logits=False)
            sec += time.perf_counter() - t0
            nsteps += EPISODE
        if world > 1:
            t = torch.tensor([sec], dtype=torch.float64, device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            sec = float(t.item())
        e2e[mode] = seqs * nsteps / sec

    peak, peak_src = peaks()
    peak_n = peak * world if tp else peak   # TP: one step's bytes are spread over every rank's HBM
    extra = {}
    # prefill (qwen_prefill, single GPU): the config-0 prompt and a 256-token
    # prompt at once, against the same tokens one decode step at a time
    if not tp and world == 1:
        toks = np.random.default_rng(5).integers(0, VOCAB, 256).tolist()
        pf = {}
        for name, ptoks in (("config0_prompt_16", prompt.tolist() if hasattr(prompt, "tolist") else list(prompt)),
                            ("prompt_256", toks)):
            best = 1e9
            for _ in range(3):
                dec.reset()
                torch.cuda.synchronize()
                t0 = time.perf_counter()
                dec.prefill(ptoks, want_logits=False)
                best = min(best, time.perf_counter() - t0)
            dec.reset()
            t0 = time.perf_counter()
            for t in ptoks:
                dec.decode_step(int(t), want_logits=False)
            stepwise = time.perf_counter() - t0
            pf[name] = {"tokens": len(ptoks), "prefill_ms": best * 1e3, "prefill_tok_s": len(ptoks) / best,
                        "stepwise_ms": stepwise * 1e3, "stepwise_tok_s": len(ptoks) / stepwise}
        extra["prefill"] = {"what": "qwen_prefill (chunked delta rule, tokens through every layer at once, "
                                    "host wall clock) against one qwen_decode_step per token", **pf}
    # config 2: W8A8 warm start at 4096 positions, 256 greedy steps
    if "2" in configs:
        sec, ids, tm = warm_config(dec, 4096, 2, 256, True, tp, dist)
        if world > 1:
            t = torch.tensor([sec], dtype=torch.float64, device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            sec = float(t.item())
        ach = bytes_per_step(tm) * 256 / sec / 1e9
        extra["config2"] = {"workload": "W8A8 (ACT_INT8), warm start: rec N(0,0.1), 4096 cached positions "
                                        "N(0,1); 256 greedy decode steps timed", "steps": 256,
                            "value": seqs * 256 / sec, "unit": UNIT, "ms_per_step": sec / 256 * 1e3,
                            "bytes_per_step": bytes_per_step(tm), "achieved_GB_s": ach,
                            "frac": ach / peak_n, "first_ids": ids[:8]}
    # config 3: W8A32 at 32768 cached positions, 512 greedy steps
    if "3" in configs:
        sec, ids, tm = warm_config(dec, 32768, 3, 512, False, tp, dist)
        if world > 1:
            t = torch.tensor([sec], dtype=torch.float64, device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            sec = float(t.item())
        ach = bytes_per_step(tm) * 512 / sec / 1e9
        extra["config3"] = {"workload": "W8A32, warm start: rec N(0,0.1), 32768 cached positions N(0,1); "
                                        "512 greedy decode steps timed", "steps": 512,
                            "value": seqs * 512 / sec, "unit": UNIT, "ms_per_step": sec / 512 * 1e3,
                            "bytes_per_step": bytes_per_step(tm), "achieved_GB_s": ach,
                            "frac": ach / peak_n, "first_ids": ids[:8]}
    if world > 1:
        dist.barrier()   # every rank's last step is done before any context goes away
    dec.close()
    # config 4: batched decode, every rank its own batch of 64 sequences (data parallel)
    if "4" in configs:
        r4 = config4(blob_path, local, max(1, args.c4_steps), W, B=args.c4_batch)
        sec4, e2e4 = r4["sec"], r4["e2e_sec"]
        if world > 1:
            t = torch.tensor([sec4, e2e4], dtype=torch.float64, device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            sec4, e2e4 = float(t[0].item()), float(t[1].item())
        st4 = r4["steps"]
        ach4 = r4["bytes_per_step"] * st4 / sec4 / 1e9
        extra["config4"] = {
            "workload": f"batched decode: {r4['B']} sequences per GPU, each its own 2048-position warm start "
                        "(rec N(0,0.1), K/V N(0,1)); W8A8 (ACT_INT8) projections as tcgen05 int8 GEMMs; "
                        f"{st4} of the 128 greedy steps timed (device-fed tokens), then {r4['e2e_steps']} more "
                        "end to end", "batch_per_gpu": r4["B"], "n_gpus": world,
            "parallelism": "1 GPU" if world == 1 else f"{world} GPUs, one batch each (data parallel)",
            "scaling": "weak",
            "value": world * r4["B"] * st4 / sec4, "unit": UNIT, "ms_per_step": sec4 / st4 * 1e3,
            "bytes_per_step": r4["bytes_per_step"], "achieved_GB_s": ach4, "frac": ach4 / peak,
            "mean_T": r4["t_mean"],
            "e2e": {"value": world * r4["B"] * r4["e2e_steps"] / e2e4, "unit": UNIT,
                    "h2d_bytes_per_step": 4 * r4["B"] + 800, "d2h_bytes_per_step": 4 * r4["B"] + 16,
                    "what": "qwen_decode_step(batch 64): host tokens in, host argmax out"},
            "tensor_pipe": load_tensor_pipe()}
    if "1" in configs and rank == 0 and world == 1:
        extra["gemv"] = {"workload": "config1: int8 x int8 GEMV microbench, every shape, weights from "
                                     "HBM (rotated copies > L2)", "kernel": "k_gemv (qwen_gemv_i8_i8)",
                         "shapes": gemv_rows(W)}

    clocks = clk.summary()
    if rank != 0:
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return 0

    # mean attended positions over the timed steps (episodes restart at T = 17)
    ts = [PROMPT_LEN + 1 + (i % EPISODE) for i in range(K)]
    bstep = bytes_per_step(float(np.mean(ts)))
    achieved = bstep / (ms_per_step * 1e-3) / 1e9
    if tp:
        peak_src = f"{peak_src} x {world} GPUs (aggregate)"
    traffic = load_traffic()
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": K,
        "warmup": W, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "strong" if tp else "weak", "vs_baseline": None,
        "dtype": "int8 weights x fp32 activations -> int32 digit accumulators",
        "data": "synthetic (random-init Qwen3.5-0.8B, seed 1234)",
        "config": {"workload": "config0: 16-token prompt prefill (untimed) + greedy decode steps "
                               "(timed) in episodes of <= 64", "model": "Qwen3.5-0.8B (random init)",
                   "batch": 1, "global_batch": seqs, "episodes": -(-K // EPISODE),
                   "T_ctx": f"{PROMPT_LEN + 1}..{PROMPT_LEN + min(K, EPISODE)}",
                   "l2": "no flush: 758 MB of weights per step > 126 MB L2",
                   "parallelism": ("1 GPU" if world == 1 else
                                   f"tp{world} (tensor parallel, one sequence)" if tp else
                                   f"{world} independent replicas")},
        "e2e": {"value": e2e["logits"], "unit": UNIT, "h2d_bytes_per_step": 4 + 40,
                "d2h_bytes_per_step": 4 * VOCAB + 20,
                "what": "qwen_decode_step per token: host token in, fp32 logits [248320] + argmax "
                        "out to pinned host memory (golden decode_step's return value)",
                "argmax_only": {"value": e2e["argmax"], "unit": UNIT, "d2h_bytes_per_step": 20}},
        "gpu_launches": K * launches_per_step,
        "roofline": {"bound": "hbm", "kernel": kernel_name,
                     "achieved": achieved, "peak": peak_n, "unit": "GB/s",
                     "frac": achieved / peak_n, "peak_source": peak_src,
                     "algorithmic_bytes_per_step": bstep,
                     "state_bytes_per_step": STATE_RW,
                     # the ncu capture is of the single-GPU kernel
                     "traffic": traffic.get("bytes_per_step") if traffic and not tp else None},
        "clocks": clocks,
        "first_ids": ids0[:8],
    }
    line.update(extra)
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
