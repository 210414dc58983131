#!/usr/bin/env python
"""Benchmark of the B200 verify path: the quantized verify-GEMM sweep.

One step = every product of the sweep: weights [5120x5120], [6144x5120], [17408x5120], [5120x17408] quantized (from
f32 N(0, 0.02), fixed seed) to Q4_K, Q5_K, Q6_K, Q8_0 and IQ4_XS, against N = 2, 4 and 8 activation rows (f32
N(0, 1)): 60 srhpm_mul_mat calls, ~2.6 GB of weight bytes per step. Consecutive calls use different matrices and
the 20 matrices (864 MB) are far larger than L2, so no call reads another's weights from L2 (no flush needed).

value  = algorithmic bytes (weights + activations read + outputs written) / device time of the step, GB/s, summed
         over ranks. With N GPUs every matrix is sharded by output rows (each rank computes rows/N rows, then
         an all-gather of Y over NCCL): strong scaling.
e2e    = the same products through the public API with host buffers: each call copies its activations from
         pinned host memory to the device, runs, and copies Y back, all inside the timed region.
roofline: the matmul op (activation quantizer + GEMM kernel, PDL-overlapped) timed per call with CUDA events on
         its stream; achieved = algorithmic bytes / summed op time, against the measured HBM copy bandwidth.
cpu_baseline: the reference's own SRV kernels (compiled from its patch into oracle/_ref; Q8_0 has no SRV kernel,
         so its share runs the restated stock path) on the host cores, over a row sample of the same sweep.

--impl reference runs that CPU implementation alone as the reference arm (rank 0 only).
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "sr-hpm_b200"))

METRIC = "quantized verify-GEMM HBM GB/s (% peak) at k=2–8; 27B verify steps/sec"
SHAPES = [(5120, 5120), (6144, 5120), (17408, 5120), (5120, 17408)]
TYPE_NAMES = ["q4_K", "q5_K", "q6_K", "q8_0", "iq4_xs"]
TYPE_IDS = {"q4_K": 12, "q5_K": 13, "q6_K": 14, "q8_0": 8, "iq4_xs": 23}
BLOCK = {12: (256, 144), 13: (256, 176), 14: (256, 210), 8: (32, 34), 23: (256, 136)}
NS = [2, 4, 8]
SEED = 1234


def row_bytes(t, K):
    qk, bs = BLOCK[t]
    return K // qk * bs


def op_bytes(t, rows, K, N):
    return rows * row_bytes(t, K) + N * K * 4 + N * rows * 4


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        j = json.load(open(p))
        return float(j["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# ------------------------------------------------------------------------------------------------------------------
# clocks during the timed region

class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                                          "-i", str(self.idx), "-lms", "100", "-f", self.path],
                                         stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
        except (OSError, ValueError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                rows.append((float(f[1]), float(f[2]), f[5], f[6], f[7], f[8]))
            except ValueError:
                continue
        os.unlink(self.path)
        if not rows:
            return None
        reasons = set()
        for r in rows:
            for name, v in zip(("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"), r[2:]):
                if v.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": sorted(reasons), "samples": len(rows)}


# ------------------------------------------------------------------------------------------------------------------
# inputs

def make_host_weights():
    """{(type, rows, K): packed blocks (numpy uint8 [rows, row_bytes])}: one f32 matrix per shape, each type."""
    import srhpm_b200 as S
    rng = np.random.default_rng(SEED)
    out = {}
    for rows, K in SHAPES:
        w = rng.standard_normal((rows, K), dtype=np.float32) * np.float32(0.02)
        for name in TYPE_NAMES:
            t = TYPE_IDS[name]
            out[(t, rows, K)] = S.quantize_chunk(w, t)
    return out


def make_host_acts():
    rng = np.random.default_rng(SEED + 1)
    return {(N, K): rng.standard_normal((N, K), dtype=np.float32) for N in NS for K in sorted({k for _, k in SHAPES})}


def sweep_ops():
    return [(N, TYPE_IDS[name], rows, K) for N in NS for (rows, K) in SHAPES for name in TYPE_NAMES]


# ------------------------------------------------------------------------------------------------------------------
# CPU baseline: the reference's own kernels

def cpu_sample(host_w, host_x, frac_rows, reps=1):
    """Runs the sweep on the host cores over the first rows*frac_rows rows of every matrix; returns (GB/s, secs,
    threads, kind)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    ref = O.load_ref()
    nth = os.cpu_count() or 1
    total_b, total_t = 0.0, 0.0
    kinds = set()
    for _ in range(reps):
        for N, t, rows, K in sweep_ops():
            r = max(16, int(rows * frac_rows))
            W = host_w[(t, rows, K)][:r]
            X = host_x[(N, K)]
            t0 = time.perf_counter()
            if t == TYPE_IDS["q8_0"] or ref is None:
                O.mul_mat_q8_0_f32(W, r, K, X, nth=nth) if t == TYPE_IDS["q8_0"] else O.mul_mat(t, W, r, K, X)
                kinds.add("port" if t == TYPE_IDS["q8_0"] else "port-scalar")
            else:
                O.ref_mul_mat(t, W, r, K, X, nth=nth, off=1, paired=1, lib=ref)
                kinds.add("reference")
            total_t += time.perf_counter() - t0
            total_b += op_bytes(t, r, K, N)
    kind = "reference" if kinds == {"reference", "port"} or kinds == {"reference"} else "port"
    return total_b / total_t / 1e9, total_t, nth, kind, (O.ref_variant() or "none")


# ------------------------------------------------------------------------------------------------------------------

def dist_setup():
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1 and not dist.is_initialized():
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    return world, rank, local


def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    host_w = make_host_weights()
    host_x = make_host_acts()
    frac = args.cpu_frac
    for _ in range(args.warmup):
        cpu_sample(host_w, host_x, frac / 4)
    t0 = time.perf_counter()
    gbs, secs, nth, kind, variant = cpu_sample(host_w, host_x, frac, reps=args.steps)
    wall = time.perf_counter() - t0
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(secs / args.steps * 1e3, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8xq", "data": "synthetic",
        "config": {"workload": "verify-GEMM sweep (5 types x 4 shapes x N=2,4,8)", "sample_rows_frac": frac,
                   "parallelism": "host threads"},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": nth, "kind": kind,
                         "sample": f"first {frac:.4f} of the rows of every product of the sweep, {args.steps} steps, "
                                   f"srv kernels build {variant}"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "wall_s": round(wall, 2),
    }
    print(json.dumps(line))
    return 0


def run_gpu(args):
    import torch
    import torch.distributed as dist
    import srhpm_b200 as S
    world, rank, local = dist_setup()
    dev = torch.device("cuda", local)
    ctx = S.Context(local)
    host_w = make_host_weights()
    host_x = make_host_acts()

    # device tensors: each rank holds its row shard of every matrix
    shards = {}
    for (t, rows, K), blocks in host_w.items():
        r0 = rows * rank // world
        r1 = rows * (rank + 1) // world
        shards[(t, rows, K)] = (S.QuantTensor.from_blocks(blocks[r0:r1], t, r1 - r0, K, dev), r0, r1)
    xs = {key: torch.from_numpy(v).to(dev) for key, v in host_x.items()}
    xs_pinned = {key: torch.from_numpy(v).pin_memory() for key, v in host_x.items()}
    ops = sweep_ops()
    ys = {}
    for N, t, rows, K in ops:
        ys[(N, t, rows, K)] = torch.empty((N, rows), dtype=torch.float32, device=dev)
    ws = max(ctx.mul_mat_work_size(shards[(t, rows, K)][0], xs[(N, K)])[1] for N, t, rows, K in ops)
    work = torch.empty(ws, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()

    def one_op(N, t, rows, K, x=None):
        W, r0, r1 = shards[(t, rows, K)]
        y = ys[(N, t, rows, K)]
        if world == 1:
            ctx.mul_mat(W, xs[(N, K)] if x is None else x, out=y, work=work)
        else:
            part = torch.empty((N, r1 - r0), dtype=torch.float32, device=dev)
            ctx.mul_mat(W, xs[(N, K)] if x is None else x, out=part, work=work)
            gathered = [torch.empty((N, rows * (i + 1) // world - rows * i // world), dtype=torch.float32,
                                    device=dev) for i in range(world)]
            dist.all_gather(gathered, part)
            torch.cat(gathered, dim=1, out=y)

    def step(events=None):
        for i, op in enumerate(ops):
            if events is not None:
                events[i][0].record(stream)
            one_op(*op)
            if events is not None:
                events[i][1].record(stream)

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    ctx.check()

    ev = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in ops]
          for _ in range(args.steps)]
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(local) if rank == 0 else None
    if clocks:
        clocks.start()
        time.sleep(0.3)
    barrier()
    torch.cuda.synchronize()
    ctx.launch_count(reset=True)
    t_start.record(stream)
    for s in range(args.steps):
        step(ev[s])
    t_end.record(stream)
    torch.cuda.synchronize()
    barrier()
    launches = ctx.launch_count()
    clk = clocks.stop() if clocks else None
    ms = t_start.elapsed_time(t_end)
    if world > 1:
        tt = torch.tensor([ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
    ms_step = ms / args.steps
    step_bytes = sum(op_bytes(t, rows, K, N) for N, t, rows, K in ops)
    value = step_bytes / (ms_step * 1e-3) / 1e9

    # roofline: per-op durations (quantize + GEMM) of this rank, summed over the timed steps
    op_ms = [sum(ev[s][i][0].elapsed_time(ev[s][i][1]) for s in range(args.steps)) / args.steps
             for i in range(len(ops))]
    my_bytes = [shards[(t, rows, K)][0].nbytes + N * K * 4 + N * (shards[(t, rows, K)][2] - shards[(t, rows, K)][1]) * 4
                for N, t, rows, K in ops]
    achieved = sum(my_bytes) / (sum(op_ms) * 1e-3) / 1e9
    peak, peak_kind = peaks()
    per_type = {}
    for i, (N, t, rows, K) in enumerate(ops):
        name = [k for k, v in TYPE_IDS.items() if v == t][0]
        per_type.setdefault(name, [0.0, 0.0])
        per_type[name][0] += my_bytes[i]
        per_type[name][1] += op_ms[i]
    per_n = {}
    for i, (N, t, rows, K) in enumerate(ops):
        per_n.setdefault(N, [0.0, 0.0])
        per_n[N][0] += my_bytes[i]
        per_n[N][1] += op_ms[i]
    c1 = [i for i, (N, t, rows, K) in enumerate(ops) if (N, t, rows, K) == (4, 12, 17408, 5120)]

    # e2e through the public API with host buffers (H2D of the activations, D2H of Y, per call)
    host_y = {key: torch.empty(y.shape, dtype=torch.float32).pin_memory() for key, y in ys.items()}
    h2d = sum(N * K * 4 for N, t, rows, K in ops)
    d2h = sum(N * rows * 4 for N, t, rows, K in ops)

    def e2e_step():
        for N, t, rows, K in ops:
            x = torch.empty((N, K), dtype=torch.float32, device=dev)
            x.copy_(xs_pinned[(N, K)], non_blocking=True)
            one_op(N, t, rows, K, x)
            host_y[(N, t, rows, K)].copy_(ys[(N, t, rows, K)], non_blocking=True)

    for _ in range(max(1, args.warmup)):
        e2e_step()
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = e0.elapsed_time(e1)
    if world > 1:
        tt = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e2e_ms = float(tt.item())
    e2e_value = step_bytes / (e2e_ms / args.steps * 1e-3) / 1e9
    ctx.check()

    line = None
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu:
            gbs, secs, nth, kind, variant = cpu_sample(host_w, host_x, args.cpu_frac)
            cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": nth, "kind": kind,
                   "sample": f"first {args.cpu_frac:.4f} of the rows of every product of the sweep (one pass, "
                             f"{secs:.1f} s); reference srv kernels build {variant}; Q8_0 restated stock path"}
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8xq4..q8 (int32 exact sums, f32 scales)",
            "data": "synthetic (seeded N(0,0.02) weights quantized on the host, N(0,1) activations)",
            "config": {"workload": "verify-GEMM sweep: Q4_K/Q5_K/Q6_K/Q8_0/IQ4_XS x [5120x5120, 6144x5120, "
                                   "17408x5120, 5120x17408] x N=2,4,8 (60 products per step)",
                       "step_bytes": step_bytes, "parallelism": f"row-sharded x{world}" if world > 1 else "1 GPU",
                       "l2": "inputs larger than L2 (864 MB of weights rotated per step)",
                       "config1_q4K_17408x5120_N4_gbs": round(
                           sum(my_bytes[i] for i in c1) / (sum(op_ms[i] for i in c1) * 1e-3) / 1e9, 2) if c1 else None,
                       "per_type_gbs": {k: round(b / (m * 1e-3) / 1e9, 1) for k, (b, m) in per_type.items()},
                       "per_N_gbs": {str(k): round(b / (m * 1e-3) / 1e9, 1) for k, (b, m) in sorted(per_n.items())}},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                         "kernel": "srv_gemm_kernel (+ activation quantizer, PDL-overlapped)",
                         "traffic": args.traffic},
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": int(launches),
            "clocks": clk,
        }
        print(json.dumps(line))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    ctx.close()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="srhpm", choices=["srhpm", "reference"])
    ap.add_argument("--cpu-frac", type=float, default=1.0 / 32, help="row fraction of the CPU baseline sample")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--traffic", type=float, default=None, help="ncu dram bytes per launch, when captured")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "srhpm":
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    return run_gpu(args)


if __name__ == "__main__":
    sys.exit(main())
