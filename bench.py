#!/usr/bin/env python
"""Benchmark of the B200 verify path: the quantized verify-GEMM sweep.

One step = every product of the sweep: weights [5120x5120], [6144x5120], [17408x5120], [5120x17408] quantized (from
f32 N(0, 0.02), fixed seed) to Q4_K, Q5_K, Q6_K, Q8_0 and IQ4_XS, against N = 2, 4 and 8 activation rows (f32
N(0, 1)): 60 srhpm_mul_mat calls, ~2.6 GB of weight bytes per step. Consecutive calls use different matrices and
the 20 matrices (864 MB) are far larger than L2, so no call reads another's weights from L2 (no flush needed).

value  = algorithmic bytes (weights + activations read + outputs written) / device time of the step, GB/s, summed
         over ranks. With N GPUs every matrix is sharded by output rows (each rank computes rows/N rows, then
         an all-gather of Y over NCCL): strong scaling.
         The timed steps replay a CUDA graph of one step (1 GPU); --eager times the calls as issued.
e2e    = the same products through the public API with host buffers: H2D copies of the step's activations from
         pinned host memory, the 60 products, and D2H copies of every output into pinned host memory, all timed.
         One GPU: the activations come over in one copy per (N, K) block on a second stream, products waiting for
         the blocks they need, and the outputs go back in 20 chunks on that stream as their products finish; several
         ranks: one H2D, then 6 chunks, each read back after its all-gather. The step's calls and copies are
         captured once into a CUDA graph and replayed, as a serving loop runs them. The same step issued call by
         call from the host is reported beside it (measurements.e2e_calls_issued_eagerly_gbs). The line's e2e
         "copies" says which ran.
roofline: achieved = algorithmic bytes of the step / timed step time (the quantizer kernels count against the GEMM),
         against the measured HBM copy bandwidth; per-product times for the breakdown come from a second graph with
         CUDA events between the products, replayed after the timed region.
cpu_baseline: the reference's own SRV kernels (compiled from its patch into oracle/_ref; Q8_0 has no SRV kernel,
         so its share runs the restated stock path) on all host cores, full passes of the same workload. Beside the
         attention and acceptance figures, the same shapes on the host: the reference's own grouped attention
         function (oracle/_ref, all threads) and the oracle's acceptance (one thread).

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

JSON_OUT = sys.stdout  # replaced in main() by a private handle on the real stdout
METRIC = "quantized verify-GEMM HBM GB/s (% peak) at k=2–8; 27B verify steps/sec"
SHAPES = [(5120, 5120), (6144, 5120), (17408, 5120), (5120, 17408)]
TYPE_NAMES = ["q4_K", "q5_K", "q6_K", "q8_0", "iq4_xs"]
TYPE_IDS = {"q4_K": 12, "q5_K": 13, "q6_K": 14, "q8_0": 8, "iq4_xs": 23, "q3_K": 11}  # q3_K: --only (the 27B FFN)
BLOCK = {12: (256, 144), 13: (256, 176), 14: (256, 210), 8: (32, 34), 23: (256, 136), 11: (256, 110)}
NS = [2, 4, 8]
SEED = 1234
DATA_DESC = "synthetic (seeded N(0,0.02) weights quantized on the host, N(0,1) activations)"
# DRAM bytes (read + write) per srv_gemm_kernel launch over one step of the default sweep on one GPU, from one ncu
# capture (profiles/srv_gemm_sweep_60products_launches.md): 2611.35 MB over the 60 launches; the algorithmic bytes
# per launch are 43.53 MB
SWEEP_TRAFFIC_PER_LAUNCH = 43.522e6


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

def make_host_weights(ops, quantize):
    """{(type, rows, K): packed blocks (numpy uint8 [rows, row_bytes])}: one f32 N(0, 0.02) matrix per shape (the
    same matrix for every type, in shape order), quantized to each type the products use by quantize(w, type): the
    library's quantizer on the device arm, the oracle's round-to-nearest one on the reference arm (which loads
    nothing of the product)."""
    rng = np.random.default_rng(SEED)
    out = {}
    shapes = sorted({(rows, K) for _, _, rows, K in ops}, key=lambda sh: SHAPES.index(sh) if sh in SHAPES else 99)
    for rows, K in shapes:
        w = rng.standard_normal((rows, K), dtype=np.float32) * np.float32(0.02)
        for t in sorted({t for _, t, r, k in ops if (r, k) == (rows, K)}):
            out[(t, rows, K)] = quantize(w, t)
    return out


def product_quantizer():
    import srhpm_b200 as S
    return S.quantize_chunk


def oracle_quantizer():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    return lambda w, t: O.quantize_rtn(t, w)


def make_host_acts(ops):
    rng = np.random.default_rng(SEED + 1)
    return {(N, K): rng.standard_normal((N, K), dtype=np.float32) for N, K in sorted({(N, K) for N, _, _, K in ops})}


def sweep_ops(only=None):
    """(N, type, rows, K) of one step. only = "TYPE:ROWSxK:N" restricts the step to that product."""
    if only:
        name, shape, n = only.split(":")
        rows, K = (int(v) for v in shape.lower().split("x"))
        return [(int(n), TYPE_IDS[name], rows, K)]
    return [(N, TYPE_IDS[name], rows, K) for N in NS for (rows, K) in SHAPES for name in TYPE_NAMES]


# ------------------------------------------------------------------------------------------------------------------
# CPU baseline: the reference's own kernels

def cpu_pass(host_w, host_x, ops, nth, O, ref):
    """One pass of `ops` on the host cores; returns (bytes, seconds, kinds)."""
    total_b, total_t, kinds = 0.0, 0.0, set()
    for N, t, rows, K in ops:
        W = host_w[(t, rows, K)]
        X = host_x[(N, K)]
        t0 = time.perf_counter()
        if t == TYPE_IDS["q8_0"]:
            O.mul_mat_q8_0_f32(W, rows, K, X, nth=nth)
            kinds.add("port")
        elif ref is None:
            raise RuntimeError("the reference kernels (oracle/_ref) are not built")
        else:
            O.ref_mul_mat(t, W, rows, K, X, nth=nth, off=1, paired=1, lib=ref)
            kinds.add("reference")
        total_t += time.perf_counter() - t0
        total_b += op_bytes(t, rows, K, N)
    return total_b, total_t, kinds


def cpu_sample(host_w, host_x, ops, target_s):
    """Full passes of the workload on all host cores until target_s seconds of CPU time; (GB/s, s, passes, threads,
    kind, build)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    ref = O.load_ref()
    nth = os.cpu_count() or 1
    cpu_pass(host_w, host_x, ops[:1], nth, O, ref)  # warm the thread pool / pages
    b, t, kinds, passes = 0.0, 0.0, set(), 0
    while t < target_s or passes == 0:
        pb, pt, pk = cpu_pass(host_w, host_x, ops, nth, O, ref)
        b, t, passes = b + pb, t + pt, passes + 1
        kinds |= pk
    kind = "reference" if "reference" in kinds else "port"
    return b / t / 1e9, t, passes, nth, kind, (O.ref_variant() or "none")


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
    """The reference arm: the reference's own CPU kernels on all host cores, one full pass of the workload per step."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    ref = O.load_ref()
    ops = sweep_ops(args.only)
    host_w = make_host_weights(ops, oracle_quantizer())
    host_x = make_host_acts(ops)
    nth = os.cpu_count() or 1
    for _ in range(args.warmup):
        cpu_pass(host_w, host_x, ops, nth, O, ref)
    b, t, kinds = 0.0, 0.0, set()
    for _ in range(args.steps):
        pb, pt, pk = cpu_pass(host_w, host_x, ops, nth, O, ref)
        b, t, kinds = b + pb, t + pt, kinds | pk
    gbs = b / t / 1e9
    kind = "reference" if "reference" in kinds else "port"
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(t / args.steps * 1e3, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8 x quantized (int32 sums)",
        "data": DATA_DESC, "config": workload_config(ops, world),
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": nth, "kind": kind,
                         "sample": f"{args.steps} full passes of the workload; reference srv kernels build "
                                   f"{O.ref_variant() or 'none'} (Q8_0: restated stock path)"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), file=JSON_OUT, flush=True)
    return 0


def workload_config(ops, world):
    if len(ops) == 1:
        N, t, rows, K = ops[0]
        name = [k for k, v in TYPE_IDS.items() if v == t][0]
        wl = f"single product {name} {rows}x{K}, N={N}"
    else:
        wl = ("verify-GEMM sweep: Q4_K/Q5_K/Q6_K/Q8_0/IQ4_XS x [5120x5120, 6144x5120, 17408x5120, 5120x17408] x "
              "N=2,4,8 (60 products per step)")
    return {"workload": wl, "step_bytes": sum(op_bytes(t, rows, K, N) for N, t, rows, K in ops),
            "parallelism": f"rows sharded x{world}" if world > 1 else "1 GPU",
            "l2": "inputs larger than L2: every product in a step reads a different weight matrix (>= 300 MB rotated)"}


def run_gpu(args):
    import torch
    import torch.distributed as dist
    import srhpm_b200 as S
    from srhpm_b200 import shard
    world, rank, local = dist_setup()
    dev = torch.device("cuda", local)
    ctx = S.Context(local)
    base_ops = sweep_ops(args.only)
    host_w = make_host_weights(base_ops, product_quantizer())
    host_x = make_host_acts(base_ops)
    # with a single product, rotate over copies of its matrix so that consecutive calls never hit L2
    ncopy = 1
    if len(base_ops) == 1:
        N, t, rows, K = base_ops[0]
        ncopy = max(2, -(-300_000_000 // (rows * row_bytes(t, K))))
    ops = [op for op in base_ops for _ in range(ncopy)]
    copy_of = [i % ncopy for i in range(len(ops))]

    shards = {}
    for (N, t, rows, K), c in zip(ops, copy_of):
        if (t, rows, K, c) in shards:
            continue
        r0, r1 = shard.row_range(rows, world, rank)
        shards[(t, rows, K, c)] = (S.QuantTensor.from_blocks(host_w[(t, rows, K)][r0:r1], t, r1 - r0, K, dev), r0, r1)
    # activations of a step, packed in one buffer (one H2D per step in the end-to-end pass)
    keys = sorted({(N, K) for N, t, rows, K in ops})
    xoff, off = {}, 0
    for key in keys:
        xoff[key] = off
        off += key[0] * key[1]
    x_host = torch.empty(off, dtype=torch.float32).pin_memory()
    for key in keys:
        x_host[xoff[key]:xoff[key] + key[0] * key[1]].copy_(torch.from_numpy(host_x[key]).reshape(-1))
    x_dev = x_host.to(dev)
    xs = {key: x_dev[xoff[key]:xoff[key] + key[0] * key[1]].view(key[0], key[1]) for key in keys}
    yoff, off = [], 0
    for N, t, rows, K in ops:
        yoff.append(off)
        off += N * rows
    y_dev = torch.zeros(off, dtype=torch.float32, device=dev)
    y_host = torch.empty(off, dtype=torch.float32).pin_memory()
    ys = [y_dev[o:o + N * rows].view(N, rows) for o, (N, t, rows, K) in zip(yoff, ops)]
    ws = max(ctx.mul_mat_work_size(shards[(t, rows, K, c)][0], xs[(N, K)])[1]
             for (N, t, rows, K), c in zip(ops, copy_of))
    work = torch.empty(ws, dtype=torch.uint8, device=dev)
    runs = []
    # several ranks: every product writes its row slice into one packed buffer (slices padded to ceil(rows / world)
    # rows so that all ranks' buffers have one size) and one all-gather per step hands every rank all the slices;
    # y_dev is then the gathered buffer [world][packed slices]
    if world > 1:
        packed = shard.PackedSlices([(N, rows) for N, t, rows, K in ops], world)
        y_local = torch.zeros(packed.size, dtype=torch.float32, device=dev)
        y_dev = torch.zeros(world * packed.size, dtype=torch.float32, device=dev)
        y_host = torch.empty(world * packed.size, dtype=torch.float32).pin_memory()
    for i, ((N, t, rows, K), c) in enumerate(zip(ops, copy_of)):
        W, r0, r1 = shards[(t, rows, K, c)]
        if world == 1:
            runs.append(ctx.prepare_mul_mat(W, xs[(N, K)], ys[i], work))
        else:
            runs.append(ctx.prepare_mul_mat(W, xs[(N, K)], packed.local_view(y_local, i, rank), work))

    def step(events=None):
        for i, run in enumerate(runs):
            if events is not None:
                events[i][0].record()
            run()
            if events is not None:
                events[i][1].record()
        if world > 1:
            dist.all_gather_into_tensor(y_dev, y_local)

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    ctx.check()

    # the timed step is replayed from a CUDA graph (no host launch gaps between the 2 kernels of each product; with
    # several ranks the graph holds the step's NCCL all-gather too)
    # "external" events stay real timing events when recorded inside a captured graph
    op_ev = [(torch.cuda.Event(enable_timing=True, external=True), torch.cuda.Event(enable_timing=True, external=True))
             for _ in ops]
    graph = None
    if not args.eager:
        graph = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            step()  # one more eager step on the capture stream before capturing
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        ctx.launch_count(reset=True)
        with torch.cuda.graph(graph):
            step()
        launches_per_step = ctx.launch_count(reset=True)
        # a second graph with timing events between the products, replayed after the timed region for the
        # per-product breakdown (events inside the timed graph would add gaps to it)
        graph_ev = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph_ev):
            step(op_ev)
        ctx.launch_count(reset=True)
        for _ in range(2):
            graph.replay()
        torch.cuda.synchronize()
        ctx.check()
    stream = torch.cuda.current_stream()
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(local) if rank == 0 else None
    if clocks:
        clocks.start()
        time.sleep(0.5)
    barrier()
    torch.cuda.synchronize()
    ctx.launch_count(reset=True)
    op_ms = [0.0] * len(ops)
    t_start.record(stream)
    for _ in range(args.steps):
        if graph is not None:
            graph.replay()
        else:
            step(op_ev)
    t_end.record(stream)
    torch.cuda.synchronize()
    barrier()
    launches = launches_per_step * args.steps if graph is not None else ctx.launch_count()
    clk = clocks.stop() if clocks else None
    ms = t_start.elapsed_time(t_end)
    if world > 1:
        tt = torch.tensor([ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
    ms_step = ms / args.steps
    step_bytes = sum(op_bytes(t, rows, K, N) for N, t, rows, K in ops)
    value = step_bytes / (ms_step * 1e-3) / 1e9

    # per-product op times from the instrumented graph (after the timed region)
    op_ms = None
    if graph is not None:
        try:
            sums = [0.0] * len(ops)
            for _ in range(3):
                graph_ev.replay()
                torch.cuda.synchronize()
                for i, (a, b) in enumerate(op_ev):
                    sums[i] += a.elapsed_time(b) / 3
            op_ms = sums
        except RuntimeError:
            op_ms = None
    my_bytes = [shards[(t, rows, K, c)][0].nbytes + N * K * 4 + N * (shards[(t, rows, K, c)][2] -
                shards[(t, rows, K, c)][1]) * 4 for (N, t, rows, K), c in zip(ops, copy_of)]
    # the step is nothing but these products: achieved = algorithmic bytes / timed step time (a conservative figure:
    # the quantizer kernels' share of the time counts against the GEMM)
    achieved = sum(my_bytes) / (ms_step * 1e-3) / 1e9
    peak, peak_kind = peaks()

    def group(keyf):
        acc = {}
        for i, op in enumerate(ops):
            k = keyf(op)
            b, m = acc.get(k, (0.0, 0.0))
            acc[k] = (b + my_bytes[i], m + (op_ms[i] if op_ms else 0.0))
        return {str(k): round(b / (m * 1e-3) / 1e9, 1) for k, (b, m) in acc.items() if m > 0}

    # e2e through the public API with host buffers: one H2D of the step's activations, the products (issued
    # call by call, no graph), a D2H of every output
    h2d, d2h = x_host.numel() * 4, y_host.numel() * 4

    def e2e_step_serial():
        x_dev.copy_(x_host, non_blocking=True)
        step()
        y_host.copy_(y_dev, non_blocking=True)

    # one GPU: the activations come over on a second stream, one copy per (N, K) activation block, and each product
    # waits only for its own block; the outputs go back in chunks of consecutive products on the same stream, each
    # chunk once its products are done, so the copies overlap the products still running; a chunk's products wait for
    # the previous step's read of their outputs (with several ranks the outputs arrive together with the step's
    # all-gather: chunks of their own below)
    copy_s = torch.cuda.Stream(dev)
    nchunk = max(1, min(20 if world == 1 else 6, len(runs)))
    cb = [len(runs) * c // nchunk for c in range(nchunk + 1)]
    ybound = yoff + [y_dev.numel()]
    ran = [torch.cuda.Event() for _ in range(nchunk)]     # a chunk's products are done
    copied = [torch.cuda.Event() for _ in range(nchunk)]  # a chunk's outputs are on the host
    first_use = {}
    for i, (N, t, rows, K) in enumerate(ops):
        first_use.setdefault((N, K), i)
    key_order = sorted(first_use, key=first_use.get)
    # the copies run in first-use order on one stream: the first product waits for the first block, the first user
    # of the second block for the last copy (so for every block); two waits, not one per block, so that the graph
    # keeps its programmatic launch edges between the other products
    h2d_first, h2d_last = torch.cuda.Event(), torch.cuda.Event()
    wait_at = {first_use[key_order[0]]: h2d_first}
    if len(key_order) > 1:
        wait_at[first_use[key_order[1]]] = h2d_last

    # captured=True: the form recorded into a CUDA graph, which replays step after step: no wait on the previous
    # step's reads (the replays are serial), and the copy stream joins the step's stream at its end
    def e2e_step_pipelined(captured=False):
        cur = torch.cuda.current_stream()
        copy_s.wait_stream(cur)  # the previous step's products are done with the activations
        with torch.cuda.stream(copy_s):
            for j, key in enumerate(key_order):
                lo, n_el = xoff[key], key[0] * key[1]
                x_dev[lo:lo + n_el].copy_(x_host[lo:lo + n_el], non_blocking=True)
                if j == 0:
                    h2d_first.record(copy_s)
            h2d_last.record(copy_s)
        for c in range(nchunk):
            if not captured:
                cur.wait_event(copied[c])
            for i in range(cb[c], cb[c + 1]):
                if i in wait_at:
                    cur.wait_event(wait_at[i])
                runs[i]()
            ran[c].record(cur)
            copy_s.wait_event(ran[c])
            lo, hi = ybound[cb[c]], ybound[cb[c + 1]]
            with torch.cuda.stream(copy_s):
                y_host[lo:hi].copy_(y_dev[lo:hi], non_blocking=True)
            copied[c].record(copy_s)
        if captured:
            cur.wait_event(copied[nchunk - 1])

    def time_e2e(e2e_step, tail=None):
        for _ in range(max(1, args.warmup)):
            e2e_step()
        torch.cuda.synchronize()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            e2e_step()
        if tail is not None:
            stream.wait_event(tail)  # the last step's last read is inside the timed region
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        return e0.elapsed_time(e1)

    # the same step's API calls and copies captured once into a CUDA graph and replayed (what a serving loop does)
    def time_e2e_graph(e2e_step):
        for _ in range(max(1, args.warmup)):
            e2e_step()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        cs = torch.cuda.Stream(dev)
        cs.wait_stream(stream)
        with torch.cuda.stream(cs):
            with torch.cuda.graph(g, stream=cs):
                e2e_step(captured=True)
        torch.cuda.synchronize()
        g.replay()
        torch.cuda.synchronize()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            g.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        del g  # may hold NCCL calls: released before the process group
        return e0.elapsed_time(e1)

    # several ranks: the same chunks, each with its own packed buffers and all-gather; a chunk's gathered outputs go
    # back on the copy stream while the next chunk's products and all-gather run
    def chunked_multi():
        out = []
        for c in range(nchunk):
            idx = list(range(cb[c], cb[c + 1]))
            pk = shard.PackedSlices([(ops[i][0], ops[i][2]) for i in idx], world)
            yl = torch.zeros(pk.size, dtype=torch.float32, device=dev)
            yg = torch.zeros(world * pk.size, dtype=torch.float32, device=dev)
            yh = torch.empty(world * pk.size, dtype=torch.float32).pin_memory()
            rr = []
            for j, i in enumerate(idx):
                N, t, rows, K = ops[i]
                W = shards[(t, rows, K, copy_of[i])][0]
                rr.append(ctx.prepare_mul_mat(W, xs[(N, K)], pk.local_view(yl, j, rank), work))
            out.append((rr, yl, yg, yh))
        return out

    def e2e_step_pipelined_multi(captured=False):
        cur = torch.cuda.current_stream()
        x_dev.copy_(x_host, non_blocking=True)
        for c, (rr, yl, yg, yh) in enumerate(chunks):
            if not captured:
                cur.wait_event(copied[c])
            for run in rr:
                run()
            dist.all_gather_into_tensor(yg, yl)
            ran[c].record(cur)
            copy_s.wait_event(ran[c])
            with torch.cuda.stream(copy_s):
                yh.copy_(yg, non_blocking=True)
            copied[c].record(copy_s)
        if captured:
            cur.wait_event(copied[nchunk - 1])

    e2e_mode = "serial: H2D, the products, one D2H of all outputs"
    e2e_eager_ms = None
    if world == 1:
        try:
            e2e_eager_ms = time_e2e(e2e_step_pipelined, copied[-1])
            e2e_ms = time_e2e_graph(e2e_step_pipelined)
            e2e_mode = (f"the step's API calls and copies as one CUDA graph, replayed: H2D of the activations in "
                        f"{len(key_order)} blocks on a second stream in first-use order (the first product waits for "
                        f"the first block, the first user of the second for all), the outputs read back in {nchunk} "
                        f"chunks on that stream as their products finish")
        except Exception as e:  # measured the serial way instead, and said so
            torch.cuda.synchronize()
            e2e_ms = time_e2e(e2e_step_serial)
            e2e_mode += f" (chunked form failed: {type(e).__name__})"
    else:  # every rank takes the same path (collectives inside): no per-rank fallback
        chunks = chunked_multi()
        d2h = sum(ch[3].numel() * 4 for ch in chunks)
        e2e_eager_ms = time_e2e(e2e_step_pipelined_multi, copied[-1])
        e2e_ms = time_e2e_graph(e2e_step_pipelined_multi)
        e2e_mode = (f"the step's API calls, collectives and copies as one CUDA graph, replayed: {nchunk} chunks, "
                    "each its products, its all-gather and its D2H on a second stream while the next chunk runs")
    if e2e_eager_ms is not None and world > 1:
        tt = torch.tensor([e2e_eager_ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e2e_eager_ms = float(tt.item())
    if world > 1:
        tt = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e2e_ms = float(tt.item())
    e2e_value = step_bytes / (e2e_ms / args.steps * 1e-3) / 1e9
    ctx.check()
    meas = {}
    if e2e_eager_ms is not None:  # the same copies and calls issued one by one from the host, for comparison
        meas["e2e_calls_issued_eagerly_gbs"] = round(step_bytes / (e2e_eager_ms / args.steps * 1e-3) / 1e9, 2)
    # the sharded step's gathered outputs against the same products whole on one GPU (after the timed regions)
    sweep_par = None
    if world > 1:
        try:
            sweep_par = sweep_parity_multi(ctx, dev, rank, world, ops, host_w, xs, y_dev, packed)
        except Exception as e:  # recorded beside the sweep rather than losing its line
            sweep_par = {"error": f"{type(e).__name__}: {str(e)[:200]}"}
    n1 = None
    if world == 1 and not args.only:
        n1 = measure_sweep_n1(ctx, dev, shards, peak)

    step_tp = step_tp_q8 = None
    if world > 1 and not args.no_step:  # every rank takes part (collectives inside the step)
        try:
            step_tp = measure_step_27b_tp(ctx, dev, rank, world, ks_extra=(2, 4))
        except Exception as e:  # recorded beside the sweep rather than losing its line
            step_tp = {"error": f"{type(e).__name__}: {str(e)[:200]}"}
        torch.cuda.empty_cache()
        try:
            step_tp_q8 = measure_step_27b_tp(ctx, dev, rank, world, n_past=131072, reps=5, kv_q8=True)
        except Exception as e:  # recorded beside the sweep rather than losing its line
            step_tp_q8 = {"error": f"{type(e).__name__}: {str(e)[:200]}"}
        torch.cuda.empty_cache()
    attn_split = attn_heads = None
    if world > 1 and not args.no_attn:  # every rank takes part (an all-gather per call)
        try:
            attn_split = measure_attention_split(ctx, dev, rank, world, peak)
        except Exception as e:  # recorded beside the sweep rather than losing its line
            attn_split = {"error": f"{type(e).__name__}: {str(e)[:200]}"}
        if 4 % world == 0:  # the 4 KV heads of the verify attention split whole over 2 or 4 ranks
            try:
                attn_heads = measure_attention_kv_heads(ctx, dev, rank, world, peak)
            except Exception as e:  # recorded beside the sweep rather than losing its line
                attn_heads = {"error": f"{type(e).__name__}: {str(e)[:200]}"}
    traffic, traffic_src = args.traffic, "--traffic" if args.traffic is not None else None
    if traffic is None and world == 1 and not args.only:
        traffic, traffic_src = SWEEP_TRAFFIC_PER_LAUNCH, "ncu capture of one sweep step on one B200 (profiles/)"
    if rank == 0:
        cfg = workload_config(base_ops, world)
        meas["timed"] = "CUDA graph of one step, replayed" if graph is not None else "eager calls"
        if step_tp is not None:
            meas["verify_step_27b_f16kv_2048_tp"] = step_tp
        if step_tp_q8 is not None:
            meas["verify_step_27b_q8kv_131072_tp"] = step_tp_q8
        if attn_split is not None:
            meas["attention_q8_0_split_k"] = attn_split
        if attn_heads is not None:
            meas["attention_q8_0_kv_heads"] = attn_heads
        if sweep_par is not None:
            meas["sweep_parity_vs_1gpu"] = sweep_par
        if ncopy > 1:
            meas["copies_rotated"] = ncopy
        meas["per_type_gbs"] = group(lambda op: [k for k, v in TYPE_IDS.items() if v == op[1]][0])
        meas["per_N_gbs"] = group(lambda op: op[0])
        meas["per_shape_gbs"] = group(lambda op: f"{op[2]}x{op[3]}")
        c1 = [i for i, op in enumerate(ops) if op == (4, 12, 17408, 5120)]
        if op_ms and c1:
            meas["q4_K_17408x5120_N4_us_in_sweep"] = round(sum(op_ms[i] for i in c1) / len(c1) * 1e3, 2)
        if world == 1 and not args.only:
            meas["single_q4_K_17408x5120_N4"] = measure_one_product(ctx, dev, host_w, host_x, (4, 12, 17408, 5120),
                                                                     peak)
            meas["sweep_N1"] = n1
        if world == 1 and not args.no_attn:
            meas["attention_q8_0"] = measure_attention(ctx, dev, peak)
            meas["accept_k8_vocab151936"] = measure_accept(ctx, dev)
            if not args.no_cpu:  # the same shapes on the host cores, beside the device figures
                try:
                    meas["attention_q8_0_cpu_reference"] = cpu_attention_reference()
                    meas["accept_k8_vocab151936_cpu_port"] = cpu_accept_port()
                except Exception as e:  # recorded beside the line rather than losing it
                    meas["attention_q8_0_cpu_reference"] = {"error": f"{type(e).__name__}: {str(e)[:200]}"}
        if world == 1 and not args.no_step:
            from srhpm_b200 import _lib as L
            meas["verify_step_27b_f16kv_2048"] = measure_step_27b(ctx, dev, peak)
            meas["verify_step_27b_q8kv_131072"] = measure_step_27b(ctx, dev, peak, ks=(8,), kv_type=L.Q8_0,
                                                                   n_past=131072, reps=5)
        cpu = None
        if world == 1 and not args.no_cpu:
            gbs, secs, passes, nth, kind, variant = cpu_sample(host_w, host_x, base_ops, args.cpu_seconds)
            cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": nth, "kind": kind,
                   "sample": f"{passes} full passes of the workload ({secs:.1f} s of CPU time); reference srv "
                             f"kernels build {variant}; Q8_0 (no srv kernel) through the restated stock path"}
            # the baseline's own outputs against the device's outputs of the timed step, every row of every product
            try:
                meas["sweep_parity_vs_reference_kernels"] = cpu_parity(host_w, host_x, ops, y_dev, yoff)
            except Exception as e:  # recorded beside the line rather than losing it
                meas["sweep_parity_vs_reference_kernels"] = {"error": f"{type(e).__name__}: {str(e)[:200]}"}
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8 x quantized (int32 exact sums, f32 scales)",
            "data": DATA_DESC,
            "config": cfg,
            "measurements": meas,
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                         "kernel": "srv_gemm_kernel (+ activation quantizer, PDL-overlapped)",
                         "algorithmic_bytes_per_launch": round(sum(my_bytes) / len(my_bytes)),
                         "launch_us": round(ms_step * 1e3 / len(ops), 3),
                         "traffic": traffic,
                         "traffic_source": traffic_src},
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "copies": e2e_mode},
            "gpu_launches": int(launches),
            "clocks": clk,
        }
        print(json.dumps(line), file=JSON_OUT, flush=True)
    graph = graph_ev = None
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    ctx.close()
    return 0


def rel_l2(a, b):
    """Relative L2 distance of a from b (numpy or torch, any shape), as a float."""
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    nb = float(np.linalg.norm(b))
    return float(np.linalg.norm(a - b) / nb) if nb > 0 else float(np.linalg.norm(a - b))


def graph_us(fn, calls, reps=20):
    """Device time of one call of fn (which issues `calls` calls) from CUDA-graph replays: warm-up, capture, then
    reps replays between CUDA events; returns microseconds per call."""
    import torch
    for _ in range(2):
        fn()
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph, stream=s):
            fn()
    torch.cuda.synchronize()
    graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (reps * calls)
    del graph
    return us


def measure_one_product(ctx, dev, host_w, host_x, op, peak):
    """One product alone (the single product Q4_K 17408x5120, N = 4): calls rotated over copies of its matrix that
    together exceed 300 MB (no call finds its weights in L2), graph-replayed; us per call and GB/s of its bytes."""
    import torch
    import srhpm_b200 as S
    N, t, rows, K = op
    ncopy = max(2, -(-300_000_000 // (rows * row_bytes(t, K))))
    Ws = [S.QuantTensor.from_blocks(host_w[(t, rows, K)], t, rows, K, dev) for _ in range(ncopy)]
    x = torch.from_numpy(host_x[(N, K)]).to(dev)
    y = torch.empty((N, rows), dtype=torch.float32, device=dev)
    ws = ctx.mul_mat_work_size(Ws[0], x)[1]
    work = torch.empty(ws, dtype=torch.uint8, device=dev)
    runs = [ctx.prepare_mul_mat(W, x, y, work) for W in Ws]

    def fn():
        for r in runs:
            r()

    us = graph_us(fn, len(runs))
    ctx.check()
    nbytes = op_bytes(t, rows, K, N)
    gbs = nbytes / (us * 1e-6) / 1e9
    del Ws, runs
    torch.cuda.empty_cache()
    return {"us": round(us, 2), "GBps": round(gbs, 1), "frac": round(gbs / peak, 4), "bytes": nbytes,
            "copies_rotated": ncopy, "timed": "CUDA graph of the calls over the copies, replayed"}


def measure_sweep_n1(ctx, dev, shards, peak):
    """The sweep's 20 matrices at N = 1 (one activation row: plain decode beside the verify widths), one graph of
    the 20 products; GB/s of their bytes."""
    import torch
    rng = np.random.default_rng(SEED + 2)
    ops1 = [(1, t, rows, K) for (t, rows, K, c) in shards if c == 0]
    xs = {K: torch.from_numpy(rng.standard_normal((1, K), dtype=np.float32)).to(dev) for K in {op[3] for op in ops1}}
    ys = [torch.empty((1, rows), dtype=torch.float32, device=dev) for (_, t, rows, K) in ops1]
    ws = max(ctx.mul_mat_work_size(shards[(t, rows, K, 0)][0], xs[K])[1] for (_, t, rows, K) in ops1)
    work = torch.empty(ws, dtype=torch.uint8, device=dev)
    runs = [ctx.prepare_mul_mat(shards[(t, rows, K, 0)][0], xs[K], y, work) for (_, t, rows, K), y in zip(ops1, ys)]

    def fn():
        for r in runs:
            r()

    us = graph_us(fn, 1)
    ctx.check()
    nbytes = sum(op_bytes(t, rows, K, 1) for (_, t, rows, K) in ops1)
    gbs = nbytes / (us * 1e-6) / 1e9
    return {"products": len(ops1), "us_per_pass": round(us, 1), "GBps": round(gbs, 1), "frac": round(gbs / peak, 4),
            "bytes": nbytes}


def cpu_parity(host_w, host_x, ops, y_dev, yoff):
    """Every product of the step through the reference's own kernels on the host cores (the CPU baseline's
    computation) against the device's outputs of the step: relative L2 per product, the largest reported, bar 1e-3
    (the reference's f32 accumulation against exact int32 sums)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    ref = O.load_ref()
    nth = os.cpu_count() or 1
    y = y_dev.cpu().numpy()
    worst, worst_op, per_type = 0.0, None, {}
    for i, (N, t, rows, K) in enumerate(ops):
        W, X = host_w[(t, rows, K)], host_x[(N, K)]
        want = O.mul_mat_q8_0_f32(W, rows, K, X, nth=nth) if t == TYPE_IDS["q8_0"] else \
            O.ref_mul_mat(t, W, rows, K, X, nth=nth, off=1, paired=1, lib=ref)
        got = y[yoff[i]:yoff[i] + N * rows].reshape(N, rows)
        e = rel_l2(got, want)
        name = [k for k, v in TYPE_IDS.items() if v == t][0]
        per_type[name] = max(per_type.get(name, 0.0), e)
        if e > worst or worst_op is None:
            worst, worst_op = e, f"{name} {rows}x{K} N={N}"
    return {"max_rel_l2": float(f"{worst:.3e}"), "worst": worst_op, "per_type_max": {k: float(f"{v:.3e}") for k, v in
            per_type.items()}, "products": len(ops), "rows": "all", "bar": 1e-3,
            "pass": bool(worst <= 1e-3), "checker": "the reference's srv kernels (oracle/_ref); Q8_0: restated stock path"}


def sweep_parity_multi(ctx, dev, rank, world, ops, host_w, xs, y_dev, packed):
    """Rank 0: every product of the sharded step (gathered from the ranks' row slices) against the same product
    computed whole on rank 0's one GPU; relative L2, bar 1e-5 (the rows' arithmetic is the same, only the split-K
    grouping of the sums may differ with the shard's size). The other ranks wait at a barrier."""
    import torch
    import torch.distributed as dist
    import srhpm_b200 as S
    out = None
    if rank == 0:
        try:
            out = _sweep_parity_rank0(ctx, dev, world, ops, host_w, xs, y_dev, packed)
        except Exception as e:  # reported; the other ranks must still leave the barrier below
            out = {"error": f"{type(e).__name__}: {str(e)[:200]}"}
    dist.barrier()
    return out


def _sweep_parity_rank0(ctx, dev, world, ops, host_w, xs, y_dev, packed):
    import torch
    import srhpm_b200 as S
    worst, worst_op, done = 0.0, None, {}
    for i, (N, t, rows, K) in enumerate(ops):
        if (N, t, rows, K) in done:
            continue
        W = S.QuantTensor.from_blocks(host_w[(t, rows, K)], t, rows, K, dev)
        want = ctx.mul_mat(W, xs[(N, K)]).float()
        got = packed.unpack(y_dev, i)
        torch.cuda.synchronize()
        e = float(torch.linalg.vector_norm(got - want) / torch.linalg.vector_norm(want))
        done[(N, t, rows, K)] = e
        if e > worst or worst_op is None:
            worst = e
            worst_op = f"{[k for k, v in TYPE_IDS.items() if v == t][0]} {rows}x{K} N={N}"
        del W
    torch.cuda.empty_cache()
    return {"max_rel_l2": float(f"{worst:.3e}"), "worst": worst_op, "products": len(done), "gpus": world,
            "bar": 1e-5, "pass": bool(worst <= 1e-5), "against": "the same products whole on one GPU"}


def _full_caches(cfg, dev, n_layer_cap, seed):
    """f16 K / V caches of the whole model ([cap, Hkv, 512] bytes per layer), the same values on every rank (one
    generator seed)."""
    import torch
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    kc, vc = [], []
    for _ in range(cfg.n_layer):
        for lst in (kc, vc):
            lst.append(torch.randn((n_layer_cap * cfg.Hkv, cfg.hd), device=dev, generator=g).half().view(
                torch.uint8).view(n_layer_cap, cfg.Hkv, 512))
    return kc, vc


def measure_step_27b_tp(ctx, dev, rank, world, k=8, n_past=2048, reps=10, seed=0, kv_q8=False, ks_extra=()):
    """The 27B-class verify step (k = 8, f16 KV of 2048 tokens; kv_q8: q8_0 KV of n_past tokens, the long-context step,
    timed without the parity pass; ks_extra: shorter drafts timed first with the same weights and caches, without a
    parity pass) on `world` GPUs in Megatron tensor parallelism
    (column-parallel QKV / gate|up / head, row-parallel O / down with the all-reduce fused into the next RMSNorm, KV
    heads split or replicated per rank, vocabulary-sharded acceptance). Every rank builds the same whole model
    (random blocks, one seed) and cuts its slices on the device (DeviceWeights.slice_of), and the same whole cache
    (its KV heads kept). The step (kernels + collectives) is one CUDA graph; time = max over ranks.

    Parity, after the timed region: rank 0 runs the same model whole on its one GPU. The drafted tokens are the
    one-GPU step's own greedy choices (built position by position, so all k are accepted there), and both runs
    score the same tokens: the gathered tensor-parallel logits against the one-GPU logits (relative L2), and the
    accepted ids against the one-GPU ones (rows whose top-1 margin exceeds the logits' difference must agree)."""
    import torch
    import torch.distributed as dist
    from srhpm_b200 import _lib as L
    from srhpm_b200 import verify_step as V
    cfg = V.DecoderConfig(kv_type=L.Q8_0 if kv_q8 else L.F16)
    full = V.DeviceWeights.random(cfg, dev, seed)
    w = V.DeviceWeights.slice_of(full, rank, world)
    g0, g1 = w.tp["g0"], w.tp["g1"]
    n = k + 1
    cap = n_past + n
    if kv_q8:  # this rank's KV heads only, N(0, 1) quantized on the device
        gen = torch.Generator(device=dev)
        gen.manual_seed(seed + 7 + rank)
        kc, vc = [], []
        for _ in range(cfg.n_layer):
            for lst in (kc, vc):
                x = torch.randn((cap * (g1 - g0), cfg.hd), device=dev, generator=gen)
                lst.append(ctx.quantize_rows_q8_0(x).view(cap, g1 - g0, 272))
                del x
        kc_full = vc_full = None
    else:
        kc_full, vc_full = _full_caches(cfg, dev, cap, seed + 7)
        kc = [c[:, g0:g1].contiguous() for c in kc_full]
        vc = [c[:, g0:g1].contiguous() for c in vc_full]
    tp = V.TensorParallel(rank, world)

    def timed(kk):
        """The step with kk drafted tokens as one replayed CUDA graph: (step, ms max over ranks, launches per rank)."""
        nn = kk + 1
        st = V.VerifyStep(ctx, cfg, w, kc, vc, nn, n_past, tp=tp)
        tok = torch.arange(nn, dtype=torch.int32, device=dev) * 977 % cfg.n_vocab  # the same tokens on every rank
        st.set_tokens(tok, tok[1:])
        for _ in range(2):
            st.run()
        torch.cuda.synchronize()
        cs = torch.cuda.Stream(dev)
        cs.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        ctx.launch_count(reset=True)
        with torch.cuda.stream(cs):
            with torch.cuda.graph(graph, stream=cs):
                st.run(cs)
        nl = ctx.launch_count(reset=True)
        for _ in range(2):
            graph.replay()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        ctx.check()
        tt = torch.tensor([e0.elapsed_time(e1) / reps], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        del graph  # holds NCCL calls: released before the process group
        return st, float(tt.item()), nl

    out = {}
    for kk in ks_extra:  # the shorter drafts, timed only (the same weights and caches)
        st, ms_k, nl = timed(kk)
        nb = step_bytes_27b(cfg, n_past, kk + 1)
        out[f"k{kk}"] = {"ms": round(ms_k, 3), "steps_per_s": round(1e3 / ms_k, 1), "gpus": world,
                         "GBps_per_gpu": round(nb / world / (ms_k * 1e-3) / 1e9, 1), "bytes": nb,
                         "kernel_launches_per_rank": nl}
        del st
    step, ms, launches = timed(k)
    ids = torch.arange(n, dtype=torch.int32, device=dev) * 977 % cfg.n_vocab

    if kv_q8:
        acc = int(step.out_n.item())
        del step, kc, vc, full, w
        torch.cuda.empty_cache()
        dist.barrier()
        nbytes = step_bytes_27b(cfg, n_past, n)
        out[f"k{k}"] = {"ms": round(ms, 3), "steps_per_s": round(1e3 / ms, 1), "gpus": world,
                        "GBps_per_gpu": round(nbytes / world / (ms * 1e-3) / 1e9, 1), "bytes": nbytes,
                        "kernel_launches_per_rank": launches, "accepted": acc, "kv": f"q8_0, {n_past} past tokens"}
        return out
    # parity against the whole model on rank 0's GPU
    par = None
    ids1 = torch.zeros(n, dtype=torch.int32, device=dev)
    one = None
    if rank == 0:
        try:
            one = V.VerifyStep(ctx, cfg, full, kc_full, vc_full, n, n_past)
            cur = ids.clone()
            for i in range(k):  # the one-GPU step's own greedy continuation, position by position
                one.set_tokens(cur, cur[1:])
                one.run()
                cur[i + 1] = one.logits[i].argmax().to(torch.int32)
            ids1.copy_(cur)
        except Exception as e:  # reported; the other ranks must still meet the collectives below
            par = {"error": f"{type(e).__name__}: {str(e)[:200]}"}
    dist.broadcast(ids1, 0)
    step.set_tokens(ids1, ids1[1:])
    step.run()
    torch.cuda.synchronize()
    # this rank's vocabulary slice of the logits, padded to one size, gathered in rank (= vocabulary) order
    vmax = max(V_r1 - V_r0 for V_r0, V_r1 in (shard_vocab(cfg.n_vocab, world, j) for j in range(world)))
    mine = torch.zeros((n, vmax), dtype=torch.float32, device=dev)
    mine[:, :step.logits.shape[1]].copy_(step.logits)
    allv = torch.empty((world, n, vmax), dtype=torch.float32, device=dev)
    dist.all_gather_into_tensor(allv, mine)
    if rank == 0 and par is None:
        try:
            one.set_tokens(ids1, ids1[1:])
            one.run()
            torch.cuda.synchronize()
            tp_logits = torch.cat([allv[j, :, :shard_vocab(cfg.n_vocab, world, j)[1] - shard_vocab(cfg.n_vocab,
                                   world, j)[0]] for j in range(world)], dim=1)
            ref = one.logits
            err = float(torch.linalg.vector_norm(tp_logits - ref) / torch.linalg.vector_norm(ref))
            top2 = ref.topk(2, dim=1).values
            margin = (top2[:, 0] - top2[:, 1]).cpu().tolist()
            dmax = float((tp_logits - ref).abs().max())
            acc_tp, acc_1 = step.accepted(), one.accepted()
            clear = all(m > 2 * dmax for m in margin[:len(acc_1)])
            par = {"logits_rel_l2": float(f"{err:.3e}"), "logits_max_abs_diff": float(f"{dmax:.3e}"),
                   "bar": 2e-2, "accepted_tp": acc_tp, "accepted_1gpu": acc_1,
                   "ids_equal": acc_tp == acc_1, "margins_clear": clear,
                   "pass": bool(err <= 2e-2 and (acc_tp == acc_1 or not clear)),
                   "against": "the same model and cache whole on one GPU, drafts = its own greedy choices"}
        except Exception as e:
            par = {"error": f"{type(e).__name__}: {str(e)[:200]}"}
    acc = int(step.out_n.item())
    del one
    dist.barrier()
    nbytes = step_bytes_27b(cfg, n_past, n)
    out[f"k{k}"] = {"ms": round(ms, 3), "steps_per_s": round(1e3 / ms, 1), "gpus": world,
                    "GBps_per_gpu": round(nbytes / world / (ms * 1e-3) / 1e9, 1), "bytes": nbytes,
                    "kernel_launches_per_rank": launches, "accepted": acc, "parity": par}
    return out


def shard_vocab(n_vocab, world, j):
    from srhpm_b200 import shard
    return shard.vocab_range(n_vocab, world, j)


def measure_attention(ctx, dev, peak, reps=20, lengths=(8192, 32768, 131072), N=8):
    """Verify attention: N query rows (8: the 8 draft rows; 9: the rows of the k = 8 verify step), 24 query heads,
    4 KV heads, head_dim 256, causal mask among the draft rows, q8_0 K/V (N(0,1) before quantization) of L past
    tokens, Q N(0,1) / 16. Timed as CUDA-graph replays over copies of the KV cache that together exceed L2."""
    import torch
    import srhpm_b200 as S
    H, Hkv, D = 24, 4, 256
    g = torch.Generator(device=dev)
    g.manual_seed(3)
    out = {}
    for L in lengths:
        nbytes = 2176 * L + 2 * H * N * D * 4
        ncopy = max(2, -(-400_000_000 // nbytes))
        q = torch.randn((H, N, D), device=dev, generator=g) / 16
        kv = []
        for _ in range(ncopy):
            pair = []
            for _ in range(2):
                x = torch.randn((Hkv * L, D), device=dev, generator=g)
                pair.append(ctx.quantize_rows_q8_0(x).view(Hkv, L, 272))
                del x
            kv.append(pair)
        mask = torch.zeros((N, L), dtype=torch.float16, device=dev)
        for t in range(N):
            mask[t, L - N + t + 1:] = float("-inf")
        o = torch.empty((N, H, D), device=dev)
        st, ws = ctx.flash_attn_ext_work_size(q, kv[0][0], kv[0][1], S.Q8_0)
        work = torch.empty(max(ws, 16), dtype=torch.uint8, device=dev)
        for i in range(3):
            ctx.flash_attn_ext(q, *kv[i % ncopy], S.Q8_0, mask=mask, out=o, work=work)
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(graph, stream=s):
                for i in range(ncopy):
                    ctx.flash_attn_ext(q, *kv[i], S.Q8_0, mask=mask, out=o, work=work)
        torch.cuda.synchronize()
        graph.replay()
        torch.cuda.synchronize()
        rounds = max(1, reps // ncopy)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(rounds):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        ctx.check()
        us = e0.elapsed_time(e1) * 1e3 / (rounds * ncopy)
        gbs = nbytes / (us * 1e-6) / 1e9
        out[str(L)] = {"us": round(us, 2), "GBps": round(gbs, 1), "frac": round(gbs / peak, 4), "bytes": nbytes}
        del graph, kv
        torch.cuda.empty_cache()
    return out


def _q80_cache(ctx, dev, Hkv, L, D, seed):
    """A q8_0 K or V cache [Hkv, L, 272] of N(0, 1) values, quantized on the device; the same bytes on every rank
    for one seed."""
    import torch
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    x = torch.randn((Hkv * L, D), device=dev, generator=g)
    out = ctx.quantize_rows_q8_0(x).view(Hkv, L, 272)
    del x
    return out


def _causal_mask(N, L, dev):
    import torch
    mask = torch.zeros((N, L), dtype=torch.float16, device=dev)
    for t in range(N):
        mask[t, L - N + t + 1:] = float("-inf")
    return mask


def measure_attention_split(ctx, dev, rank, world, peak, reps=20, lengths=(8192, 32768, 131072)):
    """The verify attention of measure_attention on `world` GPUs, split over the KV range: rank j holds tokens
    shard.kv_range(L, world, j) of the 4 KV heads' q8_0 cache; one call = the partial records of its range, an NCCL
    all-gather of the record sets (24 * 8 * 1032 bytes per rank) and the merge, all in one CUDA graph over copies of
    the rank's range that together exceed L2. Time = max over ranks; GB/s counts the whole cache once (plus Q and O),
    as on one GPU. Two exchanges of the records: an NCCL all-gather, and every rank reading the others'
    symmetric-memory buffers after a flag barrier (no collective). Parity: the first copy is the rank's range of one
    whole cache (same seed on every rank); its merged output against the whole-range call on rank 0's one GPU
    (relative L2, bar 1e-3)."""
    import torch
    import torch.distributed as dist
    import srhpm_b200 as S
    from srhpm_b200 import shard
    from srhpm_b200.split_attn import SplitKAttention
    H, Hkv, N, D = 24, 4, 8, 256
    g = torch.Generator(device=dev)
    g.manual_seed(3 + rank)
    out = {}
    for L in lengths:
        t0, t1 = shard.kv_range(L, world, rank)
        Lr = t1 - t0
        nbytes = 2176 * L + 2 * H * N * D * 4
        ncopy = max(2, -(-400_000_000 // max(1, 2176 * Lr)))
        q = torch.randn((H, N, D), device=dev, generator=torch.Generator(device=dev).manual_seed(3)) / 16
        kfull, vfull = _q80_cache(ctx, dev, Hkv, L, D, 11), _q80_cache(ctx, dev, Hkv, L, D, 12)
        kv = [(kfull[:, t0:t1].contiguous(), vfull[:, t0:t1].contiguous())]
        for _ in range(ncopy - 1):
            pair = []
            for _ in range(2):
                x = torch.randn((Hkv * Lr, D), device=dev, generator=g)
                pair.append(ctx.quantize_rows_q8_0(x).view(Hkv, Lr, 272))
                del x
            kv.append(pair)
        mask = _causal_mask(N, L, dev)
        mr = mask[:, t0:t1]
        st, ws = ctx.flash_attn_ext_work_size(q, kv[0][0], kv[0][1], S.Q8_0)
        work = torch.empty(max(ws, 16), dtype=torch.uint8, device=dev)
        res = {}
        for exchange in ("nccl", "peers"):
            att = SplitKAttention(ctx, rank, world, H, N, dev, exchange=exchange)
            for i in range(3):
                att(q, *kv[i % ncopy], S.Q8_0, mask=mr, work=work)
            torch.cuda.synchronize()
            s = torch.cuda.Stream(dev)
            s.wait_stream(torch.cuda.current_stream())
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.stream(s):
                with torch.cuda.graph(graph, stream=s):
                    for i in range(ncopy):
                        att(q, *kv[i], S.Q8_0, mask=mr, work=work)
            torch.cuda.synchronize()
            graph.replay()
            torch.cuda.synchronize()
            dist.barrier()
            rounds = max(1, reps // ncopy)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(rounds):
                graph.replay()
            e1.record()
            torch.cuda.synchronize()
            ctx.check()
            tt = torch.tensor([e0.elapsed_time(e1) * 1e3 / (rounds * ncopy)], device=dev)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            us = float(tt.item())
            del graph  # the graph holds NCCL calls: released before the process group
            # parity: the first copy (this rank's range of the whole cache) merged, against the whole range on one GPU
            got = att(q, *kv[0], S.Q8_0, mask=mr, work=work).clone()
            torch.cuda.synchronize()
            par = None
            if rank == 0:
                try:
                    want = ctx.flash_attn_ext(q, kfull, vfull, S.Q8_0, mask=mask)
                    torch.cuda.synchronize()
                    err = float(torch.linalg.vector_norm(got - want) / torch.linalg.vector_norm(want))
                    par = {"rel_l2": float(f"{err:.3e}"), "bar": 1e-3, "pass": bool(err <= 1e-3),
                           "against": "the whole range on one GPU"}
                except Exception as e:
                    par = {"error": f"{type(e).__name__}: {str(e)[:200]}"}
            dist.barrier()
            gbs = nbytes / (us * 1e-6) / 1e9
            res[exchange] = {"us": round(us, 2), "GBps": round(gbs, 1), "GBps_per_gpu": round(gbs / world, 1),
                             "frac_per_gpu": round(gbs / world / peak, 4), "parity": par}
            del att
        out[str(L)] = {"bytes": nbytes, "gpus": world, "exchange": res}
        del kv, kfull, vfull
        torch.cuda.empty_cache()
    return out


def measure_attention_kv_heads(ctx, dev, rank, world, peak, reps=20, lengths=(8192, 32768, 131072)):
    """The verify attention of measure_attention sharded by KV head (over 2 or 4 GPUs): rank j holds KV
    heads shard.kv_heads(4, world, j) of the q8_0 cache and computes their 6 query heads each over the whole range
    (no reduction); one NCCL all-gather assembles the [N, 24, 256] output on every rank. One call = the attention
    + the all-gather, in one CUDA graph over copies of the rank's heads that together exceed L2; time = max over
    ranks. Parity: the first copy is the rank's heads of one whole cache (same seed on every rank); the assembled
    output against the whole call on rank 0's one GPU (relative L2, bar 1e-3)."""
    import torch
    import torch.distributed as dist
    import srhpm_b200 as S
    from srhpm_b200 import shard
    H, Hkv, N, D = 24, 4, 8, 256
    G = H // Hkv
    g0, g1 = shard.kv_heads(Hkv, world, rank)
    hk = g1 - g0
    g = torch.Generator(device=dev)
    g.manual_seed(5 + rank)
    out = {}
    for L in lengths:
        nbytes = 2176 * L + 2 * H * N * D * 4
        ncopy = max(2, -(-400_000_000 // (544 * hk * L)))
        q = torch.randn((H, N, D), device=dev, generator=torch.Generator(device=dev).manual_seed(3)) / 16
        qr = q[g0 * G:g1 * G].contiguous()
        kfull, vfull = _q80_cache(ctx, dev, Hkv, L, D, 11), _q80_cache(ctx, dev, Hkv, L, D, 12)
        kv = [(kfull[g0:g1].contiguous(), vfull[g0:g1].contiguous())]
        for _ in range(ncopy - 1):
            pair = []
            for _ in range(2):
                x = torch.randn((hk * L, D), device=dev, generator=g)
                pair.append(ctx.quantize_rows_q8_0(x).view(hk, L, 272))
                del x
            kv.append(pair)
        mask = _causal_mask(N, L, dev)
        o_r = torch.empty((N, hk * G, D), dtype=torch.float32, device=dev)
        o_all = torch.empty((world, N, hk * G, D), dtype=torch.float32, device=dev)
        st, ws = ctx.flash_attn_ext_work_size(qr, kv[0][0], kv[0][1], S.Q8_0)
        work = torch.empty(max(ws, 16), dtype=torch.uint8, device=dev)

        def call(i):
            ctx.flash_attn_ext(qr, *kv[i], S.Q8_0, mask=mask, out=o_r, work=work)
            dist.all_gather_into_tensor(o_all, o_r)

        for i in range(3):
            call(i % ncopy)
        torch.cuda.synchronize()
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(graph, stream=s):
                for i in range(ncopy):
                    call(i)
        torch.cuda.synchronize()
        graph.replay()
        torch.cuda.synchronize()
        dist.barrier()
        rounds = max(1, reps // ncopy)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(rounds):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        ctx.check()
        tt = torch.tensor([e0.elapsed_time(e1) * 1e3 / (rounds * ncopy)], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        us = float(tt.item())
        del graph  # the graph holds NCCL calls: released before the process group
        call(0)
        got = o_all.permute(1, 0, 2, 3).reshape(N, H, D).clone()
        torch.cuda.synchronize()
        par = None
        if rank == 0:
            try:
                want = ctx.flash_attn_ext(q, kfull, vfull, S.Q8_0, mask=mask)
                torch.cuda.synchronize()
                err = float(torch.linalg.vector_norm(got - want) / torch.linalg.vector_norm(want))
                par = {"rel_l2": float(f"{err:.3e}"), "bar": 1e-3, "pass": bool(err <= 1e-3),
                       "against": "all heads on one GPU"}
            except Exception as e:
                par = {"error": f"{type(e).__name__}: {str(e)[:200]}"}
        dist.barrier()
        gbs = nbytes / (us * 1e-6) / 1e9
        out[str(L)] = {"us": round(us, 2), "GBps": round(gbs, 1), "GBps_per_gpu": round(gbs / world, 1),
                       "frac_per_gpu": round(gbs / world / peak, 4), "bytes": nbytes, "gpus": world,
                       "kv_heads_per_gpu": hk, "parity": par}
        del kv, kfull, vfull
        torch.cuda.empty_cache()
    return out


def cpu_attention_reference(lengths=(8192, 32768, 131072), target_s=6.0):
    """The verify attention of measure_attention on the host cores, through the reference's own grouped attention
    function (ggml_compute_forward_flash_attn_ext_gqa_small, compiled from its patch into oracle/_ref): the same
    shapes and q8_0 cache, all host threads, repeated calls for about target_s seconds in all."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    ref = O.load_ref()
    if ref is None:
        return {"unavailable": "the reference kernels (oracle/_ref) are not built"}
    H, Hkv, N, D = 24, 4, 8, 256
    rng = np.random.default_rng(3)
    nth = os.cpu_count() or 1
    out = {}
    for L in lengths:
        q = (rng.standard_normal((H, N, D), dtype=np.float32) / np.float32(16)).astype(np.float32)
        kv = [O.quantize_rtn(O.Q8_0, rng.standard_normal((Hkv * L, D), dtype=np.float32)).reshape(Hkv, L, 272)
              for _ in range(2)]
        mask = np.zeros((N, L), np.float16)
        for t in range(N):
            mask[t, L - N + t + 1:] = -np.inf
        m16 = mask.view(np.uint16)

        def call():
            O.ref_fa_gqa(q, O.Q8_0, kv[0], kv[1], D, L, Hkv, mask=m16, scale=1.0 / 16, nth=nth, lib=ref)

        call()  # warm-up
        reps, t0 = 0, time.perf_counter()
        while reps < 1 or (time.perf_counter() - t0 < target_s / len(lengths) and reps < 100):
            call()
            reps += 1
        us = (time.perf_counter() - t0) / reps * 1e6
        nbytes = 2176 * L + 2 * H * N * D * 4
        out[str(L)] = {"us": round(us, 1), "GBps": round(nbytes / (us * 1e-6) / 1e9, 2), "calls": reps,
                       "threads": nth}
        del kv
    return out


def cpu_accept_port(reps=20):
    """Greedy acceptance of 8 drafted tokens over the 151936-token head on one host core, through the oracle's C
    restatement (the reference's acceptance is upstream llama.cpp code, absent here): all drafted tokens accepted."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    rng = np.random.default_rng(5)
    logits = rng.standard_normal((9, 151936), dtype=np.float32)
    draft = np.argmax(logits[:8], axis=1).astype(np.int32)
    O.accept(logits, draft)
    t0 = time.perf_counter()
    for _ in range(reps):
        O.accept(logits, draft)
    return {"us": round((time.perf_counter() - t0) / reps * 1e6, 1), "threads": 1, "kind": "port"}


def measure_accept(ctx, dev, reps=50):
    """Greedy acceptance over the 27B-class head: logits f32 [9, 151936] (k = 8), all drafted tokens accepted
    (the longest scan)."""
    import torch
    V, k = 151936, 8
    g = torch.Generator(device=dev)
    g.manual_seed(4)
    ncopy = max(2, -(-400_000_000 // ((k + 1) * V * 4)))
    lgs = [torch.randn((k + 1, V), device=dev, generator=g) for _ in range(ncopy)]
    drafts = [lg[:k].argmax(dim=1).to(torch.int32) for lg in lgs]
    for i in range(3):
        ctx.sample_and_accept_n(lgs[i % ncopy], drafts[i % ncopy])
    torch.cuda.synchronize()
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph, stream=s):
            for i in range(ncopy):
                ctx.sample_and_accept_n(lgs[i], drafts[i])
    torch.cuda.synchronize()
    graph.replay()
    torch.cuda.synchronize()
    rounds = max(1, reps // ncopy)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(rounds):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    ctx.check()
    us = e0.elapsed_time(e1) * 1e3 / (rounds * ncopy)
    nbytes = (k + 1) * V * 4
    return {"us": round(us, 2), "GBps": round(nbytes / (us * 1e-6) / 1e9, 1), "logits_bytes": nbytes, "draft": k}


def step_bytes_27b(cfg, n_past, n):
    """Algorithmic bytes of one verify step: every weight matrix once, the visible KV rows of every layer, the n
    embedding rows and the n x vocab logits."""
    from srhpm_b200 import _lib as L
    row = 2 * 272 if cfg.kv_type == L.Q8_0 else 2 * 512  # K + V bytes per token and KV head
    kv = 0
    for layer in range(cfg.n_layer):
        full = cfg.window <= 0 or layer % cfg.full_every == cfg.full_every - 1
        vis = n_past + n if full else min(n_past + n, cfg.window + n - 1)
        kv += vis * cfg.Hkv * row
    return cfg.weight_bytes() + kv + n * cfg.d * 2 + n * cfg.n_vocab * 4


def measure_step_27b(ctx, dev, peak, ks=(2, 4, 8), kv_type=None, n_past=2048, reps=10, seed=0):
    """A whole verify step of the synthetic 27B-class decoder (64 layers, d 5120, FFN 17408,
    24 / 4 heads of 256, full attention every 4th layer and a 4096-token window elsewhere, vocab 151936; Q4_K attention
    and FFN-down, Q3_K gate / up, Q6_K head; random-init GGUF blocks) over a KV cache of n_past tokens, 1 accepted +
    k drafted tokens, greedy acceptance. CUDA-graph replays; steps/s and bytes / time."""
    import torch
    from srhpm_b200 import _lib as L
    from srhpm_b200 import verify_step as V
    cfg = V.DecoderConfig(kv_type=kv_type if kv_type is not None else L.F16)
    w = V.DeviceWeights.random(cfg, dev, seed)
    cap = n_past + max(ks) + 1
    rowb = 272 if cfg.kv_type == L.Q8_0 else 512
    g = torch.Generator(device=dev)
    g.manual_seed(seed + 1)
    caches = []
    for layer in range(cfg.n_layer):
        pair = []
        for _ in range(2):
            x = torch.randn((cap * cfg.Hkv, cfg.hd), device=dev, generator=g)
            if cfg.kv_type == L.Q8_0:
                pair.append(ctx.quantize_rows_q8_0(x).view(cap, cfg.Hkv, rowb))
            else:
                pair.append(x.half().view(torch.uint8).view(cap, cfg.Hkv, rowb))
            del x
        caches.append(pair)
    kc = [p[0] for p in caches]
    vc = [p[1] for p in caches]
    out = {}
    for k in ks:
        n = k + 1
        step = V.VerifyStep(ctx, cfg, w, kc, vc, n, n_past)
        ids = torch.randint(0, cfg.n_vocab, (n,), generator=g, device=dev)
        step.set_tokens(ids, ids[1:])
        for _ in range(2):
            step.run()
        torch.cuda.synchronize()
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        ctx.launch_count(reset=True)
        with torch.cuda.stream(s):
            with torch.cuda.graph(graph, stream=s):
                step.run(s)
        launches = ctx.launch_count(reset=True)
        for _ in range(2):
            graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        ctx.check()
        ms = e0.elapsed_time(e1) / reps
        nbytes = step_bytes_27b(cfg, n_past, n)
        gbs = nbytes / (ms * 1e-3) / 1e9
        out[f"k{k}"] = {"ms": round(ms, 3), "steps_per_s": round(1e3 / ms, 1), "GBps": round(gbs, 1),
                        "frac": round(gbs / peak, 4), "bytes": nbytes, "launches": launches,
                        "accepted": int(step.out_n.item())}
        del graph, step
    del w, caches, kc, vc
    torch.cuda.empty_cache()
    return out


def main():
    # stdout carries exactly one JSON line: keep a private handle on it and send everything else that libraries
    # write to file descriptor 1 (NCCL prints its version line there) to stderr
    global JSON_OUT
    JSON_OUT = os.fdopen(os.dup(1), "w")
    sys.stdout.flush()
    os.dup2(2, 1)
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="srhpm", choices=["srhpm", "reference"])
    ap.add_argument("--only", default=None, help='one product "TYPE:ROWSxK:N", e.g. q4_K:17408x5120:4')
    ap.add_argument("--eager", action="store_true", help="time eager calls instead of a captured graph")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU time of the CPU-baseline sample")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-attn", action="store_true", help="skip the attention and acceptance measurements")
    ap.add_argument("--attn", type=int, default=None, help="time only the attention at this KV length (profiling)")
    ap.add_argument("--no-step", action="store_true", help="skip the 27B-class verify-step measurements")
    ap.add_argument("--attn-rows", type=int, default=8, help="query tokens of the --attn leg (9: the k = 8 step's)")
    ap.add_argument("--step27b", type=int, default=None, help="time only the 27B-class step with k drafted tokens")
    ap.add_argument("--step27b-long", type=int, default=None,
                    help="time only the long-context 27B-class step (q8_0 KV of 131072 tokens) with k drafted tokens")
    ap.add_argument("--traffic", type=float, default=None, help="ncu dram bytes per launch, when captured")
    args = ap.parse_args()
    if args.step27b:
        import torch
        import srhpm_b200 as S
        ctx = S.Context(0)
        peak, kind = peaks()
        print(json.dumps({"verify_step_27b_f16kv_2048": measure_step_27b(ctx, torch.device("cuda", 0), peak,
                                                                          ks=(args.step27b,)), "peak_kind": kind}),
              file=JSON_OUT, flush=True)
        return 0
    if args.step27b_long:
        import torch
        import srhpm_b200 as S
        from srhpm_b200 import _lib as L
        ctx = S.Context(0)
        peak, kind = peaks()
        print(json.dumps({"verify_step_27b_q8kv_131072": measure_step_27b(ctx, torch.device("cuda", 0), peak,
                                                                           ks=(args.step27b_long,), kv_type=L.Q8_0,
                                                                           n_past=131072, reps=5),
                          "peak_kind": kind}), file=JSON_OUT, flush=True)
        return 0
    if args.attn:
        import torch
        import srhpm_b200 as S
        ctx = S.Context(0)
        peak, kind = peaks()
        print(json.dumps({"attention_q8_0": measure_attention(ctx, torch.device("cuda", 0), peak, lengths=(args.attn,),
                                                              N=args.attn_rows),
                          "rows": args.attn_rows, "peak_kind": kind}), file=JSON_OUT, flush=True)
        return 0
    if args.warmup < 3 and args.impl == "srhpm":
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    return run_gpu(args)


if __name__ == "__main__":
    sys.exit(main())
