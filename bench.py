"""fp8imma B200 benchmark (one JSON line on rank 0).

Workload (default): the decode-shape GEMM of the benchmark definition,
M=16, N=4096, K=4096, E4M3 weights with per-column scales, fp16 activations
with 1% outlier channels, through the reference-exact int8 path. One step =
one GEMM call over one activation batch. With --gpus N (torchrun, one process
per GPU) the layer is column-parallel: every rank owns a 4096-column shard of
an N*4096-column weight (weak scaling), runs the same local GEMM and the
shards are gathered into every rank's full output, which is part of the
timed step: by default over NVLink with this library's own peer stores and
flags (fp8imma_gemm_allgather, --gather peer), or with the gather fused into
the GEMM epilogue (--gather peer-epilogue) or an NCCL all-gather (--gather
nccl).

value       whole-job algorithmic GB/s (N*K + 4N + 2MK + 2MN bytes per GEMM),
            kernels on device-resident inputs, CUDA-graph replay, L2 defeated
            by rotating > 2x L2 worth of weight copies.
e2e         the same metric through the library's host-buffer entry
            (fp8imma_gemm_host_io via fp8imma_ext.imma_fp8_gemm(a_host=,
            out_host=)): every step reads that step's pinned host
            activations and writes the result to pinned host memory (on the
            decode shape the GEMM's own pre-pass and epilogue do the
            transfers); one GPU: consecutive steps alternate between two
            streams.
metric_points  the metric's other points on one GPU (decode M=1, decode M=16
            with per-row quantisation, square 4096^3), each with its own
            roofline and clock record.
--impl reference: the reference's own arithmetic on the host cores (the CPU
            oracle, all threads; the reference has no CPU implementation of
            its own), same workload, metric and unit.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "cuda-fp8-ampere_b200")
for _p in (ROOT, PKG, os.path.join(ROOT, "tests")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "GEMM TFLOPS & weight GB/s at M=1/16/4096 vs B200 roofline; 1/2/4/8 GPU"
WORKLOADS = {
    "decode_m16": dict(M=16, N=4096, K=4096, sigma_w=0.02, dist="normal", outlier_frac=0.01),
    "decode_m1": dict(M=1, N=4096, K=4096, sigma_w=0.02, dist="normal", outlier_frac=0.01),
    "decode_m4": dict(M=4, N=4096, K=4096, sigma_w=0.02, dist="normal", outlier_frac=0.01),
    "up70b_m1": dict(M=1, N=28672, K=8192, sigma_w=0.015, dist="normal", outlier_frac=0.0),
    "up70b_m32": dict(M=32, N=28672, K=8192, sigma_w=0.015, dist="normal", outlier_frac=0.0),
    # tensor-bound shapes (tcgen05 path); value is reported in TFLOPS for these
    "square4096": dict(M=4096, N=4096, K=4096, sigma_w=0.02, dist="uniform4", outlier_frac=0.0),
    "prefill": dict(M=2048, N=11008, K=4096, sigma_w=0.02, dist="normal", outlier_frac=0.0),
}
LAUNCHES_PER_CALL = {1: 1, 2: 1, 3: 3, 4: 2, 5: 2}  # by kernel path (fp8imma_last_path)


def alg_bytes(M, N, K):
    return N * K + 4 * N + 2 * M * K + 2 * M * N


def sustained_bf16():
    """MEASURED_PEAKS.json's sustained (power-capped) bf16 TFLOP/s, else the
    earlier measurement on this pool (1.4 PFLOP/s)."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        if "bf16_tflops_sustained" in d:
            return float(d["bf16_tflops_sustained"])
    return 1400.0


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d.get("hbm_gbs", 6650.0)), float(d.get("bf16_tflops", 1590.0)), "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.path = os.path.join("/tmp", "fp8imma_clocks_%d_%d.csv" % (os.getpid(), gpu_index))

    def start(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.idx), "--query-gpu=" + self.Q,
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        rows = []
        for line in open(self.path):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), float(parts[3]), parts[4:]))
            except ValueError:
                continue
        os.unlink(self.path)
        if not rows:
            return None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for r in rows:
            for n, v in zip(names, r[3][1:]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        loaded = [r for r in rows if r[2] > 200.0] or rows
        return {"sm_mhz": statistics.median(r[0] for r in loaded), "sm_max_mhz": max(r[1] for r in rows),
                "power_w_max": max(r[2] for r in rows), "samples": len(rows), "reasons": sorted(reasons)}


# ------------------------------------------------------------------ CPU ----

def cpu_oracle_time(w, budget_s=8.0, nthreads=None):
    """Time the CPU oracle (scalar C restatement, all threads) on a bounded
    sample of the workload: full M and K, a column subset sized to the budget;
    returns (GB/s of the workload's algorithmic bytes, threads, sample text)."""
    import numpy as np

    from oracle import oracle as O

    M, N, K = w["M"], w["N"], w["K"]
    nthreads = nthreads or os.cpu_count() or 1
    rng = np.random.default_rng(0)
    A = rng.standard_normal((M, K)).astype(np.float16).view(np.uint16)
    # calibrate on a small column block, then size the sample to the budget
    n_cal = min(N, 256)
    Bc = rng.integers(0, 256, (n_cal, K), dtype=np.uint8)
    sc = np.full(n_cal, np.float16(1.0)).view(np.uint16)
    t0 = time.perf_counter()
    O.imma_fp8("v4_f16", 32, A, Bc, sc, 1.0, 8.0, nthreads=nthreads)
    t_cal = max(time.perf_counter() - t0, 1e-4)
    n_s = int(min(N, max(n_cal, n_cal * budget_s / t_cal / 2)))
    Bs = rng.integers(0, 256, (n_s, K), dtype=np.uint8)
    ss = np.full(n_s, np.float16(1.0)).view(np.uint16)
    reps, t_tot = 0, 0.0
    while t_tot < budget_s / 2 or reps == 0:
        t0 = time.perf_counter()
        O.imma_fp8("v4_f16", 32, A, Bs, ss, 1.0, 8.0, nthreads=nthreads)
        t_tot += time.perf_counter() - t0
        reps += 1
    t_call = t_tot / reps * (N / n_s)  # scaled to all N columns
    gbs = alg_bytes(M, N, K) / t_call / 1e9
    return gbs, nthreads, "M=%d K=%d, %d of %d columns x %d reps, scaled to N" % (M, K, n_s, N, reps), t_call


def run_reference_arm(args, w):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    K_steps, W_steps = args.steps, args.warmup
    gbs, nthr, sample, t_call = cpu_oracle_time(w, budget_s=2.0)
    # each step: one sampled call (column subset) sized so the run ends in minutes
    import numpy as np

    from oracle import oracle as O

    M, N, K = w["M"], w["N"], w["K"]
    per_step_budget = min(1.0, 90.0 / max(1, K_steps + W_steps))
    n_s = int(max(16, min(N, N * per_step_budget / t_call)))
    rng = np.random.default_rng(1)
    A = rng.standard_normal((M, K)).astype(np.float16).view(np.uint16)
    Bs = rng.integers(0, 256, (n_s, K), dtype=np.uint8)
    ss = np.full(n_s, np.float16(1.0)).view(np.uint16)
    for _ in range(W_steps):
        O.imma_fp8("v4_f16", 32, A, Bs, ss, 1.0, 8.0, nthreads=nthr)
    t0 = time.perf_counter()
    for _ in range(K_steps):
        O.imma_fp8("v4_f16", 32, A, Bs, ss, 1.0, 8.0, nthreads=nthr)
    dt = (time.perf_counter() - t0) / K_steps
    t_full = dt * N / n_s
    val = alg_bytes(M, N, K) / t_full / 1e9
    sample = "M=%d K=%d, %d of %d columns per step, time scaled to N=%d" % (M, K, n_s, N, N)
    line = {"impl": "reference", "metric": METRIC, "value": round(val, 4), "unit": "GB/s", "n_gpus": args.gpus,
            "steps": K_steps, "warmup": W_steps, "ms_per_step": round(t_full * 1e3, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "u8", "data": "synthetic",
            "config": {"workload": args.workload, "M": M, "N": N, "K": K, "path": "int8-exact (v4 f16)"},
            "cpu_baseline": {"value": round(val, 4), "unit": "GB/s", "cores": nthr, "kind": "port", "sample": sample},
            "e2e": {"value": round(val, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "reference arithmetic on host cores: the CPU restatement of the reference fp8imma chain "
                    "(the reference ships only GPU kernels)"}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ GPU ----

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=500)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--workload", default="decode_m16", choices=sorted(WORKLOADS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-ref-lib", action="store_true")
    ap.add_argument("--points", action="store_true", help="also time the other decode/70B shapes")
    ap.add_argument("--no-metric-points", action="store_true",
                    help="skip the metric's other M points (decode M=1, square M=4096) on the default line")
    ap.add_argument("--points-only", default="", help="comma-separated subset of the --points shapes")
    ap.add_argument("--no-pdl", action="store_true", help="launch without programmatic dependent launch")
    ap.add_argument("--gather", default="peer", choices=["peer", "peer-epilogue", "nccl"],
                    help="N>1: NVLink gather in a kernel after the GEMM (peer), in the GEMM's epilogue "
                         "(peer-epilogue), or NCCL all-gather")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    w = WORKLOADS[args.workload]
    if args.impl == "reference":
        run_reference_arm(args, w)
        return

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)

    import fp8imma_b200 as F
    from fp8imma_b200 import workloads as WL

    ext = F.ext()
    F.lib().fp8imma_set_pdl(0 if args.no_pdl else 1)
    M, Nl, K = w["M"], w["N"], w["K"]
    N_tot = Nl * world
    B, s16, sig = WL.make_weights(Nl, K, w["sigma_w"], "e4m3", seed=rank, device="cuda")
    A = WL.make_activations(M, K, w["dist"], w.get("outlier_frac", 0.0), seed=1000, device="cuda")
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    wbytes = B.numel()
    copies = max(1, math.ceil(2 * l2 / wbytes)) + 1
    Bs = [B] + [B.clone() for _ in range(copies - 1)]
    D_full = torch.empty(N_tot, M, dtype=torch.float16, device=dev)
    D_loc = D_full.narrow(0, rank * Nl, Nl)
    gs, ainv = 1.0 / 16.0, 16.0

    fused = None
    F.lib().fp8imma_set_fused_gather(1 if args.gather == "peer-epilogue" else 0)
    if world > 1 and args.gather in ("peer", "peer-epilogue") and M <= 64:
        from fp8imma_b200.sharded import FusedGatherFP8Gemm

        fused = FusedGatherFP8Gemm(B, s16, M)

    def step(i):
        if fused is not None:
            fused(A, gs, ainv, B=Bs[i % copies])
            return
        ext.imma_fp8_gemm(A, Bs[i % copies], s16, None, gs, ainv, "tensor", "e4m3", "int8", "float16", "col", False,
                          D_loc)
        if world > 1:
            dist.all_gather_into_tensor(D_full, D_loc)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # warm-up on the stream the graph is captured on (per-stream scratch such as
    # the decode kernel's activation rows is set up outside the capture)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            step(i)
    barrier()
    path_id = ext.last_path()

    # timed region: K steps captured in one CUDA graph (the NCCL all-gather of
    # the sharded layer included); eager launches if capture is refused
    graph = None
    timing = "CUDA graph of K steps"
    try:
        if world > 1 and fused is None:
            # NCCL inside a captured graph did not shorten the step here and
            # made process-group teardown stall; that variant runs eagerly
            raise RuntimeError("eager at N>1")
        barrier()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for i in range(args.steps):
                step(i)
        torch.cuda.synchronize()
        graph.replay()
        barrier()
    except Exception as ex:  # capture not possible here: fall back to eager launches
        graph = None
        timing = "eager launches" if world > 1 else "eager launches (graph capture failed: %s)" % type(ex).__name__
        torch.cuda.synchronize()
        barrier()
    if world > 1:
        timing += ((", NVLink gather in the GEMM epilogue + flag barrier" if args.gather == "peer-epilogue" else
                    ", NVLink gather kernel + flag barrier") if fused is not None else ", NCCL all-gather in step")
    sampler = ClockSampler(local)
    sampler.start()
    # keep the GPU busy ~0.6 s so the clock samples reflect the loaded state
    t_end = time.time() + 0.6
    while time.time() < t_end:
        if graph is not None:
            graph.replay()
        else:
            for i in range(64):
                step(i)
        torch.cuda.synchronize()
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if graph is not None:
        cur = torch.cuda.current_stream()
        ev0.record(cur)
        graph.replay()
        ev1.record(cur)
    else:
        ev0.record()
        for i in range(args.steps):
            step(i)
        ev1.record()
    barrier()
    clocks = sampler.stop()
    t_ms = ev0.elapsed_time(ev1)
    if world > 1:
        tt = torch.tensor([t_ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t_ms = float(tt.item())
    ms_step = t_ms / args.steps
    bytes_step_rank = alg_bytes(M, Nl, K)
    value = world * bytes_step_rank / (ms_step * 1e-3) / 1e9
    tflops = world * 2 * M * Nl * K / (ms_step * 1e-3) / 1e12

    # kernel-only timing (no gather) for the roofline, same stream as the launches
    kern_ms = ms_step
    if world > 1:
        g2 = None
        ev0.record()
        for i in range(args.steps):
            ext.imma_fp8_gemm(A, Bs[i % copies], s16, None, gs, ainv, "tensor", "e4m3", "int8", "float16", "col",
                              False, D_loc)
        ev1.record()
        torch.cuda.synchronize()
        kern_ms = ev0.elapsed_time(ev1) / args.steps
        del g2

    # e2e through the reference plugin API with host buffers
    A_host = [torch.empty(M, K, dtype=torch.float16, pin_memory=True) for _ in range(4)]
    for h in A_host:
        h.copy_(A.cpu())
    D_host = torch.empty(Nl, M, dtype=torch.float16, pin_memory=True)
    A_dev = torch.empty(M, K, dtype=torch.float16, device=dev)
    use_v4 = (M % 16 == 0)

    D_dev = torch.empty(Nl, M, dtype=torch.float16, device=dev)
    # one GPU: consecutive steps alternate between two streams with their own
    # device and pinned result buffers, so the host transfers of one step run
    # beside the GEMM of the other (the order of steps on each stream is kept)
    pipe_streams = [torch.cuda.Stream(device=dev) for _ in range(2)] if world == 1 else []
    pipe_A = [A_dev, torch.empty_like(A_dev)]
    pipe_D = [D_dev, torch.empty_like(D_dev)]
    pipe_Dh = [D_host, torch.empty_like(D_host).pin_memory()]

    def e2e_step(i):
        if world == 1:
            # one call: host activations in, host result out (fp8imma_gemm_host_io)
            j = i & 1
            with torch.cuda.stream(pipe_streams[j]):
                ext.imma_fp8_gemm(pipe_A[j], Bs[i % copies], s16, None, gs, ainv, "tensor", "e4m3", "int8", "float16",
                                  "col", False, pipe_D[j], a_host=A_host[i % 4], out_host=pipe_Dh[j])
            return
        A_dev.copy_(A_host[i % 4], non_blocking=True)
        if fused is not None:
            Df = fused(A_dev, gs, ainv, B=Bs[i % copies])
            D_host.copy_(Df.narrow(0, rank * Nl, Nl), non_blocking=True)
            return
        if use_v4:
            D = ext.imma_fp8_v4_act(A_dev, Bs[i % copies], s16, gs, ainv, 32)
        else:
            D, _ = ext.imma_fp8_gemm(A_dev, Bs[i % copies], s16, None, gs, ainv, "tensor", "e4m3", "int8",
                                     "float16", "col", False, None)
        if world > 1:
            dist.all_gather_into_tensor(D_full, D)
            D_host.copy_(D_full.narrow(0, rank * Nl, Nl), non_blocking=True)
        else:
            D_host.copy_(D, non_blocking=True)

    def fork():
        for s_ in pipe_streams:
            s_.wait_stream(torch.cuda.current_stream())

    def join():
        for s_ in pipe_streams:
            torch.cuda.current_stream().wait_stream(s_)

    with torch.cuda.stream(stream):
        fork()
        for i in range(max(args.warmup, 2)):  # both pipeline streams get their scratch before capture
            e2e_step(i)
        join()
    torch.cuda.synchronize()
    barrier()
    # one GPU: the K steps (copy in, GEMM, copy out each) captured in a CUDA
    # graph like the kernel timing, so host launch overhead is not the clock
    e2e_graph, e2e_timing = None, "eager launches"
    if world == 1 or fused is not None:  # (the NVLink gather counts its calls on the device: replayable)
        try:
            e2e_graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(e2e_graph, stream=stream):
                fork()
                for i in range(args.steps):
                    e2e_step(i)
                join()
            e2e_graph.replay()
            torch.cuda.synchronize()
            e2e_timing = ("CUDA graph of K steps, each reading its activations from page-locked host memory and "
                          "writing its result to page-locked host memory (fp8imma_gemm_host_io: on this decode shape "
                          "the GEMM's own pre-pass and epilogue do the transfers); consecutive steps on two "
                          "streams") if world == 1 else (
                              "CUDA graph of K steps (H2D copy, GEMM, NVLink gather, D2H copy per step)")
        except Exception:
            e2e_graph = None
            torch.cuda.synchronize()
    barrier()
    with torch.cuda.stream(stream):
        ev0.record()
        if e2e_graph is not None:
            e2e_graph.replay()
        else:
            fork()
            for i in range(args.steps):
                e2e_step(i)
            join()
        ev1.record()
    torch.cuda.synchronize()
    barrier()
    e2e_ms = ev0.elapsed_time(ev1)
    if world > 1:
        tt = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e2e_ms = float(tt.item())
    e2e_val = world * bytes_step_rank / (e2e_ms / args.steps * 1e-3) / 1e9

    hbm, bf16, peak_kind = load_peaks()
    tensor_bound = M > 64
    if tensor_bound:
        achieved = 2.0 * M * Nl * K / (kern_ms * 1e-3) / 1e12
        peak = 2.0 * bf16  # dense int8/FP8 = 2x dense bf16 (nominal ratio); bf16 measured
        roof = {"bound": "tensor", "achieved": round(achieved, 2), "peak": peak, "unit": "TFLOP/s",
                "frac": round(achieved / peak, 4),
                "peak_source": "2 x MEASURED_PEAKS.json bf16_tflops (%s); int8/FP8 dense = 2x bf16 nominal" % peak_kind}
    else:
        achieved = bytes_step_rank / (kern_ms * 1e-3) / 1e9
        roof = {"bound": "hbm", "achieved": round(achieved, 2), "peak": hbm, "unit": "GB/s",
                "frac": round(achieved / hbm, 4),
                "peak_source": "MEASURED_PEAKS.json hbm_gbs (%s)" % peak_kind}
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tpath):
        traffic = json.load(open(tpath)).get(args.workload)

    extra = {}
    if rank == 0 and world == 1 and not args.no_ref_lib:
        extra["ref_lib_b200"] = time_reference_lib(A, Bs, s16, M, Nl, K, gs, ainv, args.steps, copies)
    if rank == 0 and world == 1 and not args.no_metric_points:
        extra["metric_points"] = time_metric_points(ext, local, hbm, bf16, peak_kind)
    if rank == 0 and world == 1 and args.points:
        extra["points"] = time_points(ext, args.steps, [x for x in args.points_only.split(",") if x])

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        gbs, nthr, sample, _ = cpu_oracle_time(w, budget_s=8.0)
        cpu = {"value": round(gbs, 4), "unit": "GB/s", "cores": nthr, "kind": "port", "sample": sample}

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(tflops if tensor_bound else value, 2),
            "unit": "TFLOPS" if tensor_bound else "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 6), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u8", "data": "synthetic",
            "config": {"workload": args.workload, "M": M, "N_per_gpu": Nl, "N_total": N_tot, "K": K,
                       "weights": "E4M3 bytes, sigma_w=%g, per-column scales" % w["sigma_w"],
                       "path": "int8-exact (reference v4 semantics)", "parallelism": "column-parallel x%d" % world,
                       "l2": "weights rotated over %d copies (%.0f MB > 2x L2)" % (copies, copies * wbytes / 1e6),
                       "timing": timing,
                       "pdl": not args.no_pdl},
            "tflops": round(tflops, 4),
            "roofline": dict(roof, traffic=traffic),
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_val * (2.0 * M * Nl * K / bytes_step_rank * 1e-3
                                                 if tensor_bound else 1.0), 2), "unit": "TFLOPS" if tensor_bound else "GB/s", "h2d_bytes_per_step": M * K * 2,
                    "d2h_bytes_per_step": Nl * M * 2, "timing": e2e_timing},
            "gpu_launches": args.steps * LAUNCHES_PER_CALL.get(path_id, 1), "kernel_path": path_id, "clocks": clocks,
            "device_error": int(F.lib().fp8imma_device_error(0)),
        }
        line.update(extra)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def time_reference_lib(A, Bs, s16, M, N, K, gs, ainv, steps, copies):
    """The reference's own WMMA kernels (built for sm_100a from its sources)
    on the same device-resident inputs, CUDA-graph timed like ours."""
    import ctypes

    import torch

    import reflib

    if not reflib.available():
        return {"unavailable": "oracle/_ref/libfp8imma_ref.so not built"}
    L = reflib.lib()
    L.fp8imma_init_fp8_e4m3_lut()
    D = torch.empty(N, M, dtype=torch.float16, device=A.device)
    f = L.fp8imma_launch_imma_fp8_actquant_v4_f16

    def call(i):
        st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        return f(32, ctypes.c_void_p(A.data_ptr()), ctypes.c_void_p(Bs[i % copies].data_ptr()),
                 ctypes.c_void_p(s16.data_ptr()), ctypes.c_void_p(D.data_ptr()), M, N, K, gs, ainv, st)

    for i in range(5):
        assert call(i) == 0
    torch.cuda.synchronize()
    n = min(steps, 200)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for i in range(n):
        call(i)
    ev1.record()
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1) / n
    return {"value": round(alg_bytes(M, N, K) / (ms * 1e-3) / 1e9, 2), "unit": "GB/s", "ms_per_call": round(ms, 5),
            "timing": "eager launches, CUDA events"}


def _timed_graph(call, n_calls, gpu_index, min_ms):
    """CUDA graph of n_calls calls (warmed up on the capture stream); the GPU
    is kept busy ~0.6 s while nvidia-smi samples the clocks, then the graph is
    replayed until at least min_ms of device time is timed. Returns
    (ms per call, clocks)."""
    import torch

    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        for i in range(3):
            call(i)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        for i in range(n_calls):
            call(i)
    g.replay()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    g.replay()
    ev1.record()
    torch.cuda.synchronize()
    reps = max(1, int(math.ceil(min_ms / max(ev0.elapsed_time(ev1), 1e-3))))
    sampler = ClockSampler(gpu_index)
    sampler.start()
    t_end = time.time() + 0.6
    while time.time() < t_end:
        g.replay()
        torch.cuda.synchronize()
    ev0.record()
    for _ in range(reps):
        g.replay()
    ev1.record()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    return ev0.elapsed_time(ev1) / (reps * n_calls), clocks


def time_metric_points(ext, gpu_index, hbm, bf16, peak_kind):
    """The metric's other M points on one GPU, each with its own roofline and
    clock record: decode M=1 (N=K=4096, HBM-bound, weights rotated over > 2x
    L2), decode M=16 with per-row activation quantisation, and the square
    M=N=K=4096 GEMM (tensor-bound, >= 50 ms timed)."""
    import torch

    from fp8imma_b200 import workloads as WL

    out = {}
    for name, (M, N, K, dist_, outl, n_calls, min_ms, aq) in {
            "decode_m1": (1, 4096, 4096, "normal", 0.01, 500, 5.0, "tensor"),
            "decode_m16_rowquant": (16, 4096, 4096, "normal", 0.01, 500, 5.0, "row"),
            "square4096": (4096, 4096, 4096, "uniform4", 0.0, 20, 50.0, "tensor")}.items():
        B, s16, _ = WL.make_weights(N, K, 0.02, "e4m3", seed=0)
        A = WL.make_activations(M, K, dist_, outl, seed=1)
        l2 = torch.cuda.get_device_properties(A.device).L2_cache_size
        copies = max(1, math.ceil(2 * l2 / B.numel())) + 1 if B.numel() < 2 * l2 else 1
        Bs = [B] + [B.clone() for _ in range(copies - 1)]
        D = torch.empty(N, M, dtype=torch.float16, device=A.device)

        def call(i):
            ext.imma_fp8_gemm(A, Bs[i % copies], s16, None, 1.0 / 16, 16.0, aq, "e4m3", "int8", "float16",
                              "col", False, D)

        ms, clocks = _timed_graph(call, n_calls, gpu_index, min_ms)
        path = ext.last_path()
        if M > 64:
            # timed for >= 50 ms back to back: the power-capped (sustained)
            # regime, so the sustained peak is the denominator; the burst
            # fraction is reported beside it
            achieved = 2.0 * M * N * K / (ms * 1e-3) / 1e12
            sus = sustained_bf16()
            roof = {"bound": "tensor", "achieved": round(achieved, 2), "peak": round(2.0 * sus, 1),
                    "unit": "TFLOP/s", "frac": round(achieved / (2.0 * sus), 4),
                    "frac_of_burst": round(achieved / (2.0 * bf16), 4),
                    "peak_source": "2 x MEASURED_PEAKS.json bf16_tflops_sustained (%s); int8 dense = 2x bf16 nominal"
                                   % peak_kind}
            val, unit = achieved, "TFLOPS"
        else:
            achieved = alg_bytes(M, N, K) / (ms * 1e-3) / 1e9
            roof = {"bound": "hbm", "achieved": round(achieved, 2), "peak": hbm, "unit": "GB/s",
                    "frac": round(achieved / hbm, 4), "peak_source": "MEASURED_PEAKS.json hbm_gbs (%s)" % peak_kind}
            val, unit = achieved, "GB/s"
        out[name] = {"M": M, "N": N, "K": K, "act_quant": aq, "us": round(ms * 1e3, 3), "value": round(val, 2),
                     "unit": unit,
                     "roofline": roof, "clocks": clocks, "kernel_path": path,
                     "timing": "CUDA graph of %d calls, >= %g ms timed" % (n_calls, min_ms)}
        del Bs, B, A, D
        torch.cuda.empty_cache()
    return out


def time_points(ext, steps, only=None):
    """Other benchmark shapes, all paths (int8-exact, native FP8, and the
    fp8wgt linear where M is a multiple of 16): decode and 70B-style (split-K
    kernels), prefill / square / 70B M=4096 (tcgen05). CUDA-graph timed,
    weights rotated over > 2x L2 where they would fit in it."""
    import torch

    import fp8imma_b200 as F
    from fp8imma_b200 import workloads as WL

    wgt = F.wgt_ext()

    shapes = {"decode_m1": (1, 4096, 4096), "decode_m4": (4, 4096, 4096), "decode_m16": (16, 4096, 4096),
              "up70b_m1": (1, 28672, 8192), "up70b_m32": (32, 28672, 8192), "prefill": (2048, 11008, 4096),
              "square4096": (4096, 4096, 4096), "square8192": (8192, 8192, 8192), "up70b_m4096": (4096, 28672, 8192)}
    out = {}
    for name, (M, N, K) in shapes.items():
        if only and name not in only:
            continue
        w = WL.CONFIGS.get(name, {})
        B, s16, sig = WL.make_weights(N, K, w.get("sigma_w", 0.02), "e4m3", seed=0)
        A = WL.make_activations(M, K, w.get("dist", "normal"), w.get("outlier_frac", 0.0), seed=1)
        l2 = torch.cuda.get_device_properties(A.device).L2_cache_size
        copies = max(1, math.ceil(2 * l2 / B.numel())) + 1 if B.numel() < 2 * l2 else 1
        Bs = [B] + [B.clone() for _ in range(copies - 1)]
        D = torch.empty(N, M, dtype=torch.float16, device=A.device)
        n = min(steps, 200) if M <= 64 else 10
        for path in ("int8", "fp8", "fp8wgt") if M % 16 == 0 else ("int8", "fp8"):
            def call(i):
                if path == "fp8wgt":
                    wgt.fp8_linear_forward(A, Bs[i % copies], 0.05)
                elif path == "int8":
                    ext.imma_fp8_gemm(A, Bs[i % copies], s16, None, 1.0 / 16, 16.0, "tensor", "e4m3", "int8",
                                      "float16", "col", False, D)
                else:
                    ext.imma_fp8_gemm(A, Bs[i % copies], None, sig, 1.0, 1.0, "row", "e4m3", "fp8", "float16", "col",
                                      False, D)
            g = torch.cuda.CUDAGraph()
            st = torch.cuda.Stream()
            with torch.cuda.stream(st):  # per-stream scratch is set up before the capture
                for i in range(3):
                    call(i)
            torch.cuda.synchronize()
            with torch.cuda.graph(g, stream=st):
                for i in range(n):
                    call(i)
            g.replay()
            torch.cuda.synchronize()
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ev0.record()
            g.replay()
            ev1.record()
            torch.cuda.synchronize()
            ms = ev0.elapsed_time(ev1) / n
            nbytes = alg_bytes(M, N, K) + (2 * M * N if path == "fp8wgt" else 0)  # fp32 output
            out["%s_%s" % (name, path)] = {"us": round(ms * 1e3, 3),
                                          "GB/s": round(nbytes / (ms * 1e-3) / 1e9, 1),
                                          "TFLOPS": round(2 * M * N * K / (ms * 1e-3) / 1e12, 3)}
            if path != "fp8wgt":
                out["%s_%s" % (name, path)]["kernel_path"] = ext.last_path()
            del g
        ref = time_reference_lib(A, [B], s16, M, N, K, 1.0 / 16, 16.0, 3 if M > 64 else 50, 1)
        if "ms_per_call" in ref:
            ms = ref["ms_per_call"]
            out["%s_reflib" % name] = {"us": round(ms * 1e3, 3), "GB/s": round(alg_bytes(M, N, K) / (ms * 1e-3) / 1e9, 1),
                                       "TFLOPS": round(2 * M * N * K / (ms * 1e-3) / 1e12, 3)}
        del Bs, B, A
        torch.cuda.empty_cache()
    return out


if __name__ == "__main__":
    main()
