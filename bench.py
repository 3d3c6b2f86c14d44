"""Benchmark of the INT4 super-block batched GEMM hot path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl moat|reference]

Workload ("Qwen-3B-like FFN"): INT4 super-block weights
K=3072 x M=8192 quantized from seeded N(0, 0.02), fp16 activations N(0, 1), batch N
swept over 1, 2, 4, 8, 16, 32. With N GPUs the 8192 columns are column-sharded
(group-aligned, 8192/N per rank, re-packed bit-identically) and each output
[N, 8192] is joined with an NCCL all-gather; total work is fixed (strong scaling).

One step = for every batch size in the sweep, the GEMM over each of R distinct copies
of the weight (a ring far larger than the 126 MB L2, so every weight byte comes from
HBM), then the all-gather (N > 1 GPUs). ``value`` = algorithmic HBM bytes all ranks
moved per second (K*M*144/256 + 2*N*K + 2*N*M per call); tokens/s per batch size are
reported beside it. The GEMM launches of a step are replayed from a CUDA graph.

``e2e`` measures the same sweep through the public Python API (``batched_gemm``) as a
host user calls it: per call the activations come from pinned host memory and the
output goes back to pinned host memory (the copies overlap the neighbouring calls'
kernels on the library's copy streams), one host wait per step.

``--impl reference`` times the reference's CPU path (the NumPy oracle port of
src/dequant.py:116-147 + the fp32 CPU GEMM of test_batched_speed.py:39-42) on this
host's cores, on a bounded sample of the same workload; rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

K_DIM, M_DIM = 3072, 8192
SWEEP = (1, 2, 4, 8, 16, 32)
L2_BYTES = 126 * 1024 * 1024
METRIC = "INT4 GEMM achieved HBM GB/s (3072x8192, N=1..32 sweep)"
SEED = 2024


def gemm_bytes(N, K, M):
    return K * M * 144 // 256 + 2 * N * K + 2 * N * M


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def load_traffic():
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if not os.path.exists(p):
        return None
    with open(p) as f:
        return json.load(f)


# ---------------------------------------------------------------------------
# clocks sampling during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.out = None

    def start(self):
        try:
            self.out = open(os.devnull, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=self.out, text=True)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            txt, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            txt, _ = self.proc.communicate()
        rows = []
        for line in txt.strip().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for nm, v in zip(names, r[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(rows)}


# ---------------------------------------------------------------------------
# reference arm / CPU baseline: the oracle port of the reference's CPU path
# ---------------------------------------------------------------------------
def all_cores() -> int:
    """Raise the NumPy BLAS / OpenMP and torch thread limits to every host core
    (torchrun starts its workers with OMP_NUM_THREADS=1) and return the core count."""
    n = os.cpu_count() or 1
    try:
        from threadpoolctl import threadpool_limits
        threadpool_limits(limits=n)
    except Exception:
        pass
    try:
        import torch
        torch.set_num_threads(n)
    except Exception:
        pass
    return n


class CpuReference:
    """The reference's CPU path per call: ``unpack_superblock_weights`` (src/dequant.py:116-147)
    then the fp32 NumPy GEMM (test_batched_speed.py:39-42), via the oracle port.
    Setup (quantize + pack) happens once, outside any timed region."""

    def __init__(self):
        from oracle import int4 as O
        all_cores()
        self.O = O
        self.st = O.quantize_pack_matrix(O.make_weights(K_DIM, M_DIM, SEED))
        self.xs = {n: O.make_activations(n, K_DIM, n) for n in SWEEP}
        O.gemm(self.xs[1], O.unpack_superblock_weights(self.st).reshape(K_DIM, M_DIM))  # warm BLAS threads

    def call(self, n):
        w = self.O.unpack_superblock_weights(self.st).reshape(K_DIM, M_DIM)
        return self.O.gemm(self.xs[n], w)

    def sweep(self):
        for n in SWEEP:
            self.call(n)

    @staticmethod
    def threads():
        threads = os.cpu_count()
        try:
            from threadpoolctl import threadpool_info
            threads = max((i.get("num_threads") or 0) for i in threadpool_info()) or threads
        except Exception:
            pass
        return threads


def cpu_reference(budget_s=10.0):
    """CPU baseline: cycle the batch sweep for about ``budget_s`` seconds."""
    ref = CpuReference()
    total_bytes, total_tok, calls = 0, 0, 0
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < budget_s:
        for n in SWEEP:
            ref.call(n)
            total_bytes += gemm_bytes(n, K_DIM, M_DIM)
            total_tok += n
            calls += 1
    el = time.perf_counter() - t0
    return {"value": total_bytes / el / 1e9, "unit": "GB/s", "tok_per_s": total_tok / el,
            "cores": CpuReference.threads(), "kind": "port",
            "sample": f"{calls} calls ({el:.1f} s) of unpack_superblock_weights + fp32 NumPy GEMM at 3072x8192, "
                      f"cycling N in {list(SWEEP)}"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    ref = CpuReference()
    steps = max(1, args.steps)
    for _ in range(min(args.warmup, 1)):
        ref.sweep()
    t0 = time.perf_counter()
    for _ in range(steps):
        ref.sweep()
    el = time.perf_counter() - t0
    step_bytes = sum(gemm_bytes(n, K_DIM, M_DIM) for n in SWEEP)
    value = step_bytes * steps / el / 1e9
    cores = CpuReference.threads()
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": args.gpus,
        "steps": steps, "warmup": args.warmup, "ms_per_step": el / steps * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f16 x int4 -> f32 acc -> f16", "data": "synthetic",
        "config": {"workload": "BASELINE config 3: INT4 super-block GEMM K=3072 x M=8192, N sweep "
                               + ",".join(map(str, SWEEP)) + " (host CPU, unsharded)",
                   "K": K_DIM, "M": M_DIM, "sweep": list(SWEEP)},
        "tok_per_s": sum(SWEEP) * steps / el,
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": f"{steps} steps x one call per N in {list(SWEEP)} (oracle port of the "
                                   f"reference CPU path: unpack_superblock_weights + fp32 NumPy GEMM)"},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def run_moat(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    from moat_b200 import _lib
    from moat_b200.dequant import extract_columns, quantize_to_superblocks
    from moat_b200.dist import column_bounds
    from moat_b200.gemm import plan

    L = _lib.lib()
    K, M = K_DIM, M_DIM
    bounds = column_bounds(M, world, K)
    c0, c1 = bounds[rank]
    Ms = c1 - c0
    sweep = tuple(int(s) for s in args.sweep.split(","))

    # weights: seeded N(0, 0.02) on the device, GPU quantizer, this rank's columns
    g = torch.Generator(device=dev)
    g.manual_seed(SEED)
    w = torch.randn((K, M), generator=g, device=dev, dtype=torch.float32) * 0.02
    full = quantize_to_superblocks(w.reshape(-1))
    del w
    shard = extract_columns(full, K, M, c0, c1)
    del full
    sb_bytes = shard.numel()
    R = args.ring
    if R <= 0:  # ring >= 4x L2 on every rank at up to 8 GPUs: fixed total work
        R = -(-4 * L2_BYTES * 8 // (K * M * 144 // 256))
    ring = torch.empty((R, sb_bytes), dtype=torch.uint8, device=dev)
    ring[:] = shard
    xs = {n: (torch.randn((n, K), generator=g, device=dev) ).to(torch.float16) for n in sweep}
    ys = {n: torch.empty((R, n, Ms), dtype=torch.float16, device=dev) for n in sweep}
    gath = {n: torch.empty((world, R, n, Ms), dtype=torch.float16, device=dev) for n in sweep} if world > 1 else {}
    yfull = {n: torch.empty((R, n, M), dtype=torch.float16, device=dev) for n in sweep} if world > 1 else {}

    stream = torch.cuda.Stream(device=dev)
    plans = {n: plan(n, K, Ms) for n in sweep}

    def gemm_launches(n):
        st = stream.cuda_stream
        x = xs[n]
        y = ys[n]
        for r in range(R):
            rc = L.mb_int4_gemm(x.data_ptr(), ring[r].data_ptr(), y[r].data_ptr(), n, K, Ms, None, st)
            if rc != 0:
                raise RuntimeError(f"mb_int4_gemm failed: {rc}")

    torch.cuda.synchronize()
    graphs = {}
    with torch.cuda.stream(stream):
        for n in sweep:  # warm the launch path (attributes, occupancy) before capture
            gemm_launches(n)
        stream.synchronize()
        for n in sweep:
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=stream):
                gemm_launches(n)
            graphs[n] = gr
    torch.cuda.synchronize()

    ev = [{n: (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for n in sweep}
          for _ in range(args.steps)]
    gemm_ms = {n: 0.0 for n in sweep}

    def step(record):
        with torch.cuda.stream(stream):
            for n in sweep:
                if record is not None:
                    ev[record][n][0].record(stream)
                graphs[n].replay()
                if record is not None:
                    ev[record][n][1].record(stream)
                if world > 1:
                    dist.all_gather_into_tensor(gath[n].view(-1), ys[n].view(-1))
                    yfull[n].view(R, n, world, Ms).copy_(gath[n].permute(1, 2, 0, 3))

    for _ in range(args.warmup):
        step(None)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = ClockSampler(local)
    clocks.start()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    t_start.record(stream)
    for i in range(args.steps):
        step(i)
    t_end.record(stream)
    torch.cuda.synchronize()
    for i in range(args.steps):
        for n in sweep:
            gemm_ms[n] += ev[i][n][0].elapsed_time(ev[i][n][1])
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    elapsed = t_start.elapsed_time(t_end) / 1e3  # seconds
    el_t = torch.tensor([elapsed], device=dev)
    if world > 1:
        dist.all_reduce(el_t, op=dist.ReduceOp.MAX)
    elapsed = float(el_t.item())

    # per-launch GEMM time (this rank), bytes per launch of this rank's shard
    per_n = {}
    tot_bytes_launch, tot_gemm_s = 0, 0.0
    for n in sweep:
        t_launch = gemm_ms[n] / 1e3 / (args.steps * R)
        b = gemm_bytes(n, K, Ms)
        per_n[str(n)] = {"us_per_call": t_launch * 1e6, "GBps": b / t_launch / 1e9,
                         "tok_per_s": n * world / max(t_launch, 1e-12) if world == 1 else None}
        tot_bytes_launch += b * args.steps * R
        tot_gemm_s += gemm_ms[n] / 1e3
    achieved = tot_bytes_launch / tot_gemm_s / 1e9
    step_bytes = sum(gemm_bytes(n, K, Ms) for n in sweep) * R * world
    value = step_bytes * args.steps / elapsed / 1e9
    tok_per_s = {str(n): n * R * args.steps / elapsed for n in sweep}

    # e2e through the public API with pinned host buffers
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(args, dev, stream, shard, sweep, Ms, world, rank, bounds, R)

    peak, peak_kind = load_peaks()
    traffic = load_traffic()
    tr = None
    if traffic and "k_gemm_int4" in traffic:
        per = traffic["k_gemm_int4"].get("dram_bytes_per_launch", {})
        if all(str(n) in per for n in sweep) and world == 1:
            tr = sum(per[str(n)] for n in sweep) / len(sweep)

    attn = None if args.no_attn else attention_side(dev, peak, peak_kind, with_cpu=not args.no_cpu, rank=rank,
                                                    world=world)
    cfg2 = None if (world > 1 or args.no_config2) else config2_side(dev, peak, peak_kind)
    decode = None if args.no_decode else decode_side(dev, rank, world, with_cpu=not args.no_cpu)
    sampling = None if (world > 1 or args.no_decode) else sampling_side(dev, rows=(16,))

    if rank == 0:
        cpu = None if (world > 1 or args.no_cpu) else cpu_reference(budget_s=args.cpu_seconds)
        line = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": elapsed / args.steps * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f16 x int4 -> f32 acc -> f16",
            "data": "synthetic (seeded N(0,0.02) weights, N(0,1) activations)",
            "config": {"workload": "BASELINE config 3: INT4 super-block GEMM K=3072 x M=8192, N sweep "
                                   + ",".join(map(str, sweep)) + f"; column-sharded over {world} GPU(s)"
                                   + (" + NCCL all-gather" if world > 1 else ""),
                       "K": K, "M": M, "sweep": list(sweep), "ring_copies": R,
                       "ring_bytes_per_rank": R * sb_bytes, "l2": "inputs larger than L2 (weight ring)",
                       "parallelism": f"column-shard M over {world}"},
            "tok_per_s": tok_per_s,
            "per_n": per_n,
            "plans": {str(n): plans[n] for n in sweep},
            "roofline": {"bound": "hbm", "kernel": "k_gemm_int4", "achieved": achieved, "peak": peak,
                         "unit": "GB/s", "frac": achieved / peak, "peak_kind": peak_kind,
                         "traffic": tr, "bytes_per_launch": "K*M*144/256 + 2NK + 2NM (this rank's shard)"},
            "gpu_launches": args.steps * R * len(sweep),
            "clocks": clk,
            "e2e": e2e,
            "cpu_baseline": cpu,
            "attention": attn,
            "config2": cfg2,
            "decode": decode,
            "sampling": sampling,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        graphs.clear()
        dist.destroy_process_group()
    return 0


def config2_side(dev, peak, peak_kind, reps: int = 5):
    """BASELINE config 2 (Qwen-1.5B-like FFN up-projection, INT4 K=2048 x M=5504,
    N = 1, 2, 4, 8, 16, 32, one GPU): per N the GEMM over a ring of weight copies far
    larger than L2, replayed from a CUDA graph, CUDA-event timed; us per call, achieved
    GB/s and the fraction of the measured HBM peak. Reported beside the config-3 line."""
    import torch
    from moat_b200 import _lib
    from moat_b200.dequant import quantize_to_superblocks
    from moat_b200.gemm import plan
    L = _lib.lib()
    K, M = 2048, 5504
    g = torch.Generator(device=dev)
    g.manual_seed(SEED + 2)
    sb = quantize_to_superblocks((torch.randn((K, M), generator=g, device=dev) * 0.02).reshape(-1))
    R = -(-4 * L2_BYTES // sb.numel())
    ring = torch.empty((R, sb.numel()), dtype=torch.uint8, device=dev)
    ring[:] = sb
    st = torch.cuda.Stream(device=dev)
    out = {}
    for n in SWEEP:
        x = torch.randn((n, K), generator=g, device=dev).half()
        y = torch.empty((R, n, M), dtype=torch.float16, device=dev)

        def launches():
            for r in range(R):
                rc = L.mb_int4_gemm(x.data_ptr(), ring[r].data_ptr(), y[r].data_ptr(), n, K, M, None, st.cuda_stream)
                if rc != 0:
                    raise RuntimeError(f"mb_int4_gemm failed: {rc}")

        with torch.cuda.stream(st):
            launches()
            st.synchronize()
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=st):
                launches()
            for _ in range(3):
                gr.replay()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            for _ in range(reps):
                gr.replay()
            e1.record(st)
            st.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / (reps * R)
        b = gemm_bytes(n, K, M)
        out[str(n)] = {"us_per_call": us, "GBps": b / us / 1e3, "frac": b / us / 1e3 / peak,
                       "tok_per_s": n / us * 1e6, "plan": plan(n, K, M)}
        del gr, y
    del ring
    torch.cuda.empty_cache()
    return {"workload": "BASELINE config 2: INT4 super-block GEMM K=2048 x M=5504, N sweep "
                        + ",".join(map(str, SWEEP)) + ", one GPU",
            "ring_copies": R, "l2": "inputs larger than L2 (weight ring)", "peak": peak, "peak_kind": peak_kind,
            "per_n": out}


def attention_side(dev, peak, peak_kind, reps: int = 10, with_cpu: bool = True, rank: int = 0, world: int = 1):
    """BASELINE config 4 decode attention (16 traces x 16 heads, KV length 4096, d 128,
    fp16 KV, 32,768-entry LUT over [-16, 0]) timed with CUDA events, the KV copies
    rotated so each call streams from HBM (together far larger than L2). With ``world``
    > 1 the heads are sharded (rank r computes its head range) and every call ends with
    the NCCL all-gather of the [16, 16, 128] output, the calls replayed from a CUDA
    graph; the time is the maximum over ranks and GB/s counts every head's K and V.
    Reported beside the GEMM line, not part of its value."""
    import torch
    from moat_b200 import _lib
    from moat_b200.attention import ExponentialLUT, attention_bytes
    from moat_b200.dist import gather_heads, head_bounds
    L = _lib.lib()
    T, H, Lk, d = 16, 16, 4096, 128
    bounds = head_bounds(H, world)
    h0, h1 = bounds[rank]
    Hl = h1 - h0
    g = torch.Generator(device=dev)
    g.manual_seed(SEED + 7)
    q = torch.randn((T, H, d), generator=g, device=dev).half()[:, h0:h1].contiguous()
    copy_bytes = 2 * T * Hl * Lk * d * 2
    copies = max(2, -(-4 * L2_BYTES // copy_bytes))
    kv = [(torch.randn((T, Hl, Lk, d), generator=g, device=dev).half(),
           torch.randn((T, Hl, Lk, d), generator=g, device=dev).half()) for _ in range(copies)]
    lut = ExponentialLUT(range_max=16.0)
    tab = lut.device_table(dev)
    out = torch.empty((T, Hl, d), dtype=torch.float16, device=dev)
    nb = int(L.mb_decode_attn_workspace_size(T, Hl, Lk, d))
    ws = torch.zeros(nb, dtype=torch.uint8, device=dev)
    st = torch.cuda.Stream(device=dev)
    scale = 1.0 / float(d) ** 0.5

    def call(i):
        k, v = kv[i % copies]
        rc = L.mb_decode_attn(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), T, Hl, Lk, d, scale,
                              tab.data_ptr(), lut.size, 16.0, ws.data_ptr(), nb, st.cuda_stream)
        assert rc == 0, rc
        if world > 1:
            gather_heads(out, bounds)

    graph = None
    with torch.cuda.stream(st):
        for i in range(4):
            call(i)
        st.synchronize()
        if world > 1:
            # one pass over the KV copies replayed from a CUDA graph (the all-gather
            # included), so the small per-call launches do not leave the GPUs idle
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=st):
                for i in range(copies):
                    call(i)
            graph.replay()
            st.synchronize()
            import torch.distributed as dist
            dist.barrier()
        passes = max(1, -(-reps // copies))
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        if graph is not None:
            for _ in range(passes):
                graph.replay()
        else:
            for i in range(reps):
                call(i)
        e1.record(st)
        st.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (passes * copies if graph is not None else reps)
    del graph  # a graph holding NCCL calls is released before the process group
    if world > 1:
        import torch.distributed as dist
        m = torch.tensor([us], dtype=torch.float64, device=dev)
        dist.all_reduce(m, op=dist.ReduceOp.MAX)
        us = float(m.item())
    b = attention_bytes(T, H, Lk, d)
    gbs = b / us / 1e3
    del kv, ws
    torch.cuda.empty_cache()
    res = {"workload": "BASELINE config 4: LUT-softmax decode attention, 16 traces x 16 heads, L=4096, d=128"
                       + (f"; heads sharded over {world} GPUs + NCCL all-gather" if world > 1 else ""),
           "us_per_call": us, "GBps": gbs, "bytes_per_call": b, "kernels_per_call": 3, "kv_copies": copies,
           "heads_per_rank": [h1_ - h0_ for h0_, h1_ in bounds],
           "roofline": {"bound": "hbm", "achieved": gbs / world, "peak": peak, "unit": "GB/s",
                        "frac": gbs / world / peak, "peak_kind": peak_kind, "per": "GPU"},
           "cpu_baseline": attention_cpu_baseline(T, H, Lk, d) if (with_cpu and world == 1) else None}
    return res


def attention_cpu_baseline(T, H, Lk, d, budget_s: float = 6.0):
    """The reference's CPU composition of decode attention (NumPy einsum scores, LUT
    softmax, einsum with V; oracle port) on the host cores, one full config-4 call per
    sample until the budget is spent."""
    from oracle import attention as OA
    from moat_b200.attention import attention_bytes
    cores = all_cores()
    q, k, v = OA.make_attention_inputs(T, H, Lk, d, SEED + 11)
    tbl = OA.exp_table(32768, 16.0)
    calls, t0 = 0, time.perf_counter()
    while True:
        OA.decode_attention(q, k, v, tbl, 16.0)
        calls += 1
        el = time.perf_counter() - t0
        if el >= budget_s or calls >= 20:
            break
    return {"value": attention_bytes(T, H, Lk, d) * calls / el / 1e9, "unit": "GB/s", "cores": cores,
            "kind": "port", "sample": f"{calls} full config-4 calls ({el:.1f} s) of the NumPy composition "
                                       "(einsum scores, LUT softmax, einsum with V)",
            "us_per_call": el / calls * 1e6}


def decode_side(dev, rank: int = 0, world: int = 1, steps: int = 256, prompt: int = 512, check_steps: int = 16,
                with_cpu: bool = True, profile_step: bool = False):
    """BASELINE config 5 as written: a random-init Qwen-1.5B-like INT4 decoder (24
    layers, hidden 2048, 16 heads x 128, FFN 5504, vocab 151936), N = 16 traces, a
    prompt of 512 seeded random token ids run through the decode step one position at
    a time (the reference engine's prefill loop), then 256 greedy steps replayed from one
    captured CUDA graph and timed with CUDA events (maximum over ranks). With ``world``
    > 1 the decoder is tensor-parallel: heads, FFN and vocabulary split over the ranks,
    two exchanges per layer (peer stores over NVLink, one kernel that joins the partial
    rows with the residual add and RMSNorm) and one for the greedy choice, all inside
    the graph; tokens/s counts the N tokens the whole job makes per step (total work
    fixed: strong scaling).

    Then the decoder is rewound to the end of the prompt and ``check_steps`` greedy
    steps are replayed eagerly, recording each step's input and output ids. On one GPU
    the reference-style CPU forward (oracle port of transformer.py:161-225 with the same
    dequantized weights, fp32, every host core) replays the same inputs from the same
    cache: its time is the decode CPU baseline and its argmax agreement with the GPU's
    ids is reported (exact softmax, the reference's TinyLlamaModel; exp-LUT softmax, the
    reference's batch decode path). On N GPUs every rank also builds the whole model as
    a replica and replays the tensor-parallel inputs: the number of differing ids is
    reported. Reported beside the GEMM line."""
    import torch
    from moat_b200.decode import DecoderConfig, Int4Decoder, timed_decode
    cfg = DecoderConfig(max_len=prompt + steps + 24)
    N = 16
    g = torch.Generator(device=dev)
    g.manual_seed(SEED + 6)
    prompt_ids = torch.randint(0, cfg.vocab, (N, prompt), generator=g, device=dev, dtype=torch.int32)
    dec = Int4Decoder(cfg, N, device=dev, seed=SEED + 5, rank=rank, world=world, exchange_timeout_s=2.0)
    cpu = None
    tp_check = None
    try:
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        dec.prefill(prompt_ids)
        torch.cuda.synchronize()
        prefill_s = time.perf_counter() - t0
        snap = dec.cache_snapshot()
        first = dec.ids.clone()
        try:
            ms = timed_decode(dec, steps, warmup=3, graph=True)
        except RuntimeError as e:  # raised on every rank alike (the check is all-reduced)
            return {"workload": "BASELINE config 5 decode", "error": str(e), "tensor_parallel": world}
        if profile_step:  # one eager step inside an NVTX range, for an ncu launch list of one step
            torch.cuda.nvtx.range_push("decode_step")
            dec.step(dec.ids)
            torch.cuda.synchronize()
            torch.cuda.nvtx.range_pop()
        err = int(dec.err.item())
        wbytes = sum(sum(int(lw[k].numel()) for k in ("wqkv", "wo", "wgu", "wd")) for lw in dec.layers) \
            + int(dec.lm_head.numel()) * dec.Vl // dec.lm_cols  # without the LM head's zero padding
        kv = 2 * cfg.layers * N * dec.Hl * cfg.head_dim * 2 * (prompt + 5 + steps // 2)  # mean cache length
        tot = torch.tensor([float(wbytes + kv), float(err)], dtype=torch.float64, device=dev)
        if world > 1:
            import torch.distributed as dist
            dist.all_reduce(tot)
        step_bytes, err = float(tot[0].item()), int(tot[1].item())
        # rewind to the end of the prompt and record a short greedy trajectory
        dec.restore_cache(snap)
        ids = first.clone()
        ins, outs = [], []
        for _ in range(check_steps):
            ins.append(ids.cpu())
            ids = dec.step(ids).clone()
            outs.append(ids.cpu())
        if world == 1 and with_cpu and rank == 0:
            cpu = decode_cpu_baseline(dec, snap, ins, outs)
    finally:
        dec.close()  # graph and exchange buffers go before the process group
    del dec
    torch.cuda.empty_cache()
    replicas = None
    if world > 1:  # the other way to use N GPUs: every GPU decodes its own 16 traces
        import torch.distributed as dist
        rep = Int4Decoder(cfg, N, device=dev, seed=SEED + 5)
        try:
            rep.prefill(prompt_ids)
            rsnap = rep.cache_snapshot()
            rfirst = rep.ids.clone()
            # the replica replays the tensor-parallel decoder's inputs from its own cache
            bad = 0
            for i, o in zip(ins, outs):
                bad += int((rep.step(i.to(dev)).cpu() != o).sum().item())
            bad += int((rfirst.cpu() != ins[0]).sum().item())
            rep.restore_cache(rsnap)
            rep.ids.copy_(rfirst)
            rms = timed_decode(rep, steps, warmup=3, graph=True)
        finally:
            rep.close()
        m = torch.tensor([rms, float(bad)], dtype=torch.float64, device=dev)
        dist.all_reduce(m, op=dist.ReduceOp.MAX)
        rms, bad = float(m[0].item()), int(m[1].item())
        replicas = {"tok_per_s": world * N / rms * 1e3, "ms_per_step": rms, "traces_per_gpu": N,
                    "scaling": "weak", "note": "independent full-model replicas, no collective; max over ranks"}
        tp_check = {"tp_vs_replica_mismatch": bad, "ids_compared": N * (check_steps + 1),
                    "how": "the one-GPU replica replays the tensor-parallel decoder's greedy inputs from its own "
                           "prefilled cache (first token + %d steps); max over ranks" % check_steps}
        del rep
        torch.cuda.empty_cache()
    return {"workload": "BASELINE config 5: 24-layer INT4 decoder, hidden 2048, 16x128 heads, FFN 5504, "
                        "vocab 151936; 16 traces, 512-token random prompt run through the step, 256 greedy steps",
            "metric": "decode tok/s", "tok_per_s": N / ms * 1e3, "ms_per_step": ms, "steps": steps,
            "prompt": prompt, "prefill_s": prefill_s, "prefill_tok_per_s": N * prompt / prefill_s, "graph": True,
            "tensor_parallel": world, "scaling": "strong" if world > 1 else None,
            "exchange": ("NVLink peer stores from the o_proj / down GEMM epilogues (mb_int4_gemm_peer, "
                         "mb_peer_sum_rmsnorm) and mb_peer_argmax") if world > 1 else None,
            "bytes_per_step": step_bytes, "GBps": step_bytes / ms / 1e6, "device_error_bits": err,
            "replicas": replicas, "tp_check": tp_check, "cpu_baseline": cpu,
            "data": "synthetic (random-init weights quantized to INT4; seeded random prompt ids)"}


def decode_cpu_baseline(dec, snap, ins, outs):
    """The reference-style CPU decoder forward (oracle port of transformer.py:161-225:
    fp32 torch on every host core, the GPU decoder's INT4 weights dequantized) replays
    the GPU's recorded greedy inputs from the prompt's cache; timed with the exact
    softmax (the reference's TinyLlamaModel), then run again with the exp-LUT softmax of
    the reference's batch decode path. Reports tok/s and both argmax agreements."""
    import torch
    from oracle.decoder import CpuDecoder, argmax_agreement
    threads = all_cores()
    cfg = dec.cfg
    dense = dec.dense_weights()
    ks, vs, n = snap
    gpu = np.stack([o.numpy() for o in outs])
    res = {}
    for mode in ("exact", "lut"):
        cpu = CpuDecoder(dense["layers"], dense["final_norm"], dense["lm_head"], dense["embed"], dense["cis"],
                         cfg.heads, dec.N, n + len(ins) + 1, eps=cfg.eps, softmax=mode, lut=dec.lut.lut,
                         lut_range=cfg.lut_range)
        cpu.load_cache(ks, vs, n)
        got = []
        t0 = time.perf_counter()
        with torch.no_grad():
            for i in ins:
                got.append(torch.argmax(cpu.step(i), dim=-1).numpy())
        res[mode] = (argmax_agreement(np.stack(got), gpu), time.perf_counter() - t0)
        del cpu
    el = res["exact"][1]
    return {"value": dec.N * len(ins) / el, "unit": "tok/s", "cores": threads, "kind": "port",
            "ms_per_step": el / len(ins) * 1e3,
            "sample": f"{len(ins)} greedy steps of 16 traces from the 512-token prompt's cache, fp32 torch CPU "
                      "forward (transformer.py semantics, exact softmax) with the dequantized INT4 weights",
            "argmax_agreement_exact_softmax": res["exact"][0], "argmax_agreement_lut_softmax": res["lut"][0],
            "ids_compared": int(gpu.size)}


def sampling_side(dev, rows=(16,), calls: int = 50, vocab: int = 151936, temperature: float = 0.7):
    """Batched sampler speed on the config-5 LM-head output shape: N rows of 151936
    fp16 logits, temperature 0.7, top-50 of the LUT softmax (``mb_sample_tokens``), as
    back-to-back eager calls and as one captured CUDA graph of the same calls,
    CUDA-event timed after warm-up."""
    import torch
    from moat_b200.sampling import BatchSampler
    out = {"workload": f"mb_sample_tokens: N x {vocab} fp16 logits, T={temperature}, top-50, LUT range 10",
           "calls": calls, "rows": {}}
    for N in rows:
        g = torch.Generator(device=dev)
        g.manual_seed(SEED + 9 + N)
        logits = (torch.randn((N, vocab), generator=g, device=dev) * 3.0).half()
        s = BatchSampler(N, vocab, device=dev, seed=SEED)
        for _ in range(5):
            s.sample(logits, temperature)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(calls):
            s.sample(logits, temperature)
        e1.record()
        torch.cuda.synchronize()
        eager = e0.elapsed_time(e1) / calls * 1e3
        graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            with torch.cuda.graph(graph, stream=side):
                for _ in range(calls):
                    s.sample(logits, temperature)
        torch.cuda.current_stream(dev).wait_stream(side)
        graph.replay()
        torch.cuda.synchronize()
        e0.record()
        graph.replay()
        e1.record()
        torch.cuda.synchronize()
        out["rows"][str(N)] = {"us_per_call": eager, "graph_us_per_call": e0.elapsed_time(e1) / calls * 1e3,
                               "device_error_bits": int(s.err.item())}
        del graph
    if len(rows) == 1:
        out["us_per_call"] = out["rows"][str(rows[0])]["us_per_call"]
    return out


def exchange_side(dev, rank: int, world: int, rows: int = 16, hidden: int = 2048, vocab: int = 151936,
                  iters: int = 200):
    """The tensor-parallel decode step's exchanges on ``world`` GPUs (``--part
    exchange`` under torchrun): ``add_rmsnorm`` of [N, D] fp16 partials over NVLink peer
    stores, the greedy ``argmax`` over [N, V/G] logits per rank, and an NCCL
    ``all_reduce`` of the same [N, D] fp16 rows for comparison; CUDA events over
    back-to-back calls after warm-up, the maximum over ranks. Also a row-parallel
    o_proj (``[N, D / world] x [D / world, D]``) with its join: ``o_proj_gemm_join``
    (the GEMM's partial through HBM, the join kernel stores it to the peers) against
    ``o_proj_gemm_join_fused`` (the GEMM's epilogue stores its rows into the exchange
    buffers, ``mb_int4_gemm_peer``), and the o_proj GEMM alone (``o_proj_gemm``), so
    that ``join_after_gemm[_fused]_us`` is what each join adds after its GEMM.
    ``*_us``: the calls replayed from one CUDA graph,
    as in the decode step; ``*_eager_us``: launched one by one from Python
    (host-bound)."""
    import torch
    import torch.distributed as dist
    from moat_b200.peer import PeerExchange
    N, D = rows, hidden
    px = PeerExchange(N, D, dev)
    g = torch.Generator(device=dev)
    g.manual_seed(rank)
    partial = torch.randn((N, D), generator=g, device=dev).half()
    x = torch.zeros((N, D), device=dev)
    w = torch.ones(D, device=dev)
    h = torch.empty((N, D), dtype=torch.float16, device=dev)
    Vl = vocab // world
    logits = torch.randn((N, Vl), generator=g, device=dev).half()
    ids = torch.empty(N, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    red = partial.clone()

    def timed(fn, graph):
        """Microseconds per call, max over ranks: ``iters`` calls replayed from one CUDA
        graph (as the decode step runs them) or launched eagerly from the host."""
        for _ in range(10):
            fn()
        torch.cuda.synchronize()
        g = None
        if graph:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for _ in range(iters):
                    fn()
            g.replay()
            torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        if graph:
            g.replay()
        else:
            for _ in range(iters):
                fn()
        e1.record()
        torch.cuda.synchronize()
        del g  # a graph holding NCCL calls is released before the process group
        m = torch.tensor([e0.elapsed_time(e1) / iters * 1e3], dtype=torch.float64, device=dev)
        dist.all_reduce(m, op=dist.ReduceOp.MAX)
        return float(m.item())

    # a row-parallel o_proj (K = D / world rows of this rank) and its join: the GEMM's
    # partial through HBM into the join kernel, or stored by the GEMM's epilogue
    from moat_b200._lib import lib
    from moat_b200.dequant import quantize_to_superblocks
    Ko = D // world
    wo = quantize_to_superblocks((0.02 * torch.randn((Ko, D), generator=g, device=dev)).reshape(-1))
    act = torch.randn((N, Ko), generator=g, device=dev).half()
    o = torch.empty((N, D), dtype=torch.float16, device=dev)

    def gemm_only():
        st = torch.cuda.current_stream(dev).cuda_stream
        lib().mb_int4_gemm(act.data_ptr(), wo.data_ptr(), o.data_ptr(), N, Ko, D, err.data_ptr(), st)

    def gemm_join():
        st = torch.cuda.current_stream(dev).cuda_stream
        lib().mb_int4_gemm(act.data_ptr(), wo.data_ptr(), o.data_ptr(), N, Ko, D, err.data_ptr(), st)
        px.add_rmsnorm(o, x, w, 1e-6, h, err, st)

    def gemm_join_fused():
        st = torch.cuda.current_stream(dev).cuda_stream
        px.gemm(act, wo, Ko, D, err, st)
        px.sum_rmsnorm(x, w, 1e-6, h, err, st)

    calls = {"add_rmsnorm": lambda: px.add_rmsnorm(partial, x, w, 1e-6, h, err),
             "argmax": lambda: px.argmax(logits, rank * Vl, ids, err),
             "nccl_all_reduce": lambda: dist.all_reduce(red),
             "o_proj_gemm": gemm_only,
             "o_proj_gemm_join": gemm_join,
             "o_proj_gemm_join_fused": gemm_join_fused}
    try:
        out = {"world": world, "rows": N, "hidden": D, "vocab_per_rank": Vl, "iters": iters}
        for name, fn in calls.items():
            out[f"{name}_us"] = timed(fn, graph=True)
        for name, fn in calls.items():
            out[f"{name}_eager_us"] = timed(fn, graph=False)
        # what each join adds to the o_proj GEMM it follows, as the decode step runs them
        out["join_after_gemm_us"] = out["o_proj_gemm_join_us"] - out["o_proj_gemm_us"]
        out["join_after_gemm_fused_us"] = out["o_proj_gemm_join_fused_us"] - out["o_proj_gemm_us"]
        e = err.clone()
        dist.all_reduce(e, op=dist.ReduceOp.MAX)
        out["device_error_bits"] = int(e.item())
    finally:
        px.close()
    return out


def run_part(args):
    """``--part decode|sampling|exchange``: one side measurement alone (rank 0 prints
    its JSON block)."""
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    try:
        if args.part == "decode":
            out = decode_side(dev, rank, world, steps=args.decode_steps, prompt=args.decode_prompt,
                              with_cpu=not args.no_cpu, profile_step=args.decode_profile)
        elif args.part == "sampling":
            out = sampling_side(dev, rows=tuple(int(r) for r in args.sampling_rows.split(",")))
        else:
            if world < 2:
                raise SystemExit("--part exchange needs torchrun with 2 or more ranks")
            out = exchange_side(dev, rank, world)
        if rank == 0:
            print(json.dumps({"part": args.part, args.part: out}), flush=True)
    finally:
        if world > 1:
            dist.destroy_process_group()
    return 0


def run_e2e(args, dev, stream, shard, sweep, Ms, world, rank, bounds, R):
    """Same sweep through ``moat_b200.gemm.batched_gemm``: per call an H2D of the
    activations from pinned memory and a D2H of the output into pinned memory."""
    import torch
    import torch.distributed as dist
    from moat_b200.dist import gather_columns
    from moat_b200.gemm import batched_gemm, host_wait

    K, M = K_DIM, M_DIM
    R_e = min(R, args.e2e_ring)
    ring = [shard.clone() for _ in range(R_e)]
    g = torch.Generator().manual_seed(SEED + 1)
    host_x = {n: torch.randn((n, K), generator=g).to(torch.float16).pin_memory() for n in sweep}
    host_y = {n: torch.empty((R_e, n, M), dtype=torch.float16).pin_memory() for n in sweep}
    dev_x = {n: torch.empty((n, K), dtype=torch.float16, device=dev) for n in sweep}
    h2d = sum(n * K * 2 for n in sweep) * R_e
    d2h = sum(n * M * 2 for n in sweep) * R_e

    def step():
        with torch.cuda.stream(stream):
            for n in sweep:
                for r in range(R_e):
                    if world == 1:
                        # host buffers in and out: one C call copies in, runs, copies back
                        batched_gemm(host_x[n], ring[r], K, Ms, out=host_y[n][r], sync=False)
                        continue
                    dev_x[n].copy_(host_x[n], non_blocking=True)
                    y = gather_columns(batched_gemm(dev_x[n], ring[r], K, Ms), bounds)
                    host_y[n][r].copy_(y, non_blocking=True)
            if world == 1:
                host_wait(dev)  # the copies of the host calls run on the library's copy streams
            stream.synchronize()

    for _ in range(max(1, args.warmup)):
        step()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    steps = max(1, args.e2e_steps)
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    el = time.perf_counter() - t0
    el_t = torch.tensor([el], device=dev)
    if world > 1:
        dist.all_reduce(el_t, op=dist.ReduceOp.MAX)
    el = float(el_t.item())
    step_bytes = sum(gemm_bytes(n, K, Ms) for n in sweep) * R_e * world
    return {"value": step_bytes * steps / el / 1e9, "unit": "GB/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "steps": steps, "calls_per_step": R_e * len(sweep),
            "tok_per_s": sum(sweep) * R_e * steps / el,
            "how": "public API batched_gemm per call with pinned host activations and output (1 GPU: "
                   "one C call per GEMM enqueues the H2D copy, the kernel and the D2H copy, the copies "
                   "on library copy streams so that they overlap the neighbouring calls' kernels; N GPUs: "
                   "H2D, kernel, all-gather, D2H); wall clock around steps, one host wait per step"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="moat", choices=["moat", "reference"])
    ap.add_argument("--ring", type=int, default=0, help="weight copies per rank (0: >= 4x L2 at 8 GPUs)")
    ap.add_argument("--sweep", default=",".join(map(str, SWEEP)))
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-attn", action="store_true", help="skip the config-4 attention side measurement")
    ap.add_argument("--no-decode", action="store_true", help="skip the config-5 decode side measurement")
    ap.add_argument("--no-config2", action="store_true", help="skip the config-2 (2048 x 5504) sweep")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--e2e-ring", type=int, default=36)
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--part", choices=["all", "decode", "sampling", "exchange"], default="all",
                    help="run one side measurement alone (decode: BASELINE config 5; sampling: mb_sample_tokens; "
                         "exchange: the tensor-parallel joins, under torchrun)")
    ap.add_argument("--decode-steps", type=int, default=256)
    ap.add_argument("--decode-prompt", type=int, default=512)
    ap.add_argument("--decode-profile", action="store_true",
                    help="after timing, one eager decode step inside the NVTX range 'decode_step'")
    ap.add_argument("--sampling-rows", default="1,16,32")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "moat":
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    if args.part != "all":
        return run_part(args)
    return run_moat(args)


if __name__ == "__main__":
    sys.exit(main())
