"""Benchmark of the search hot path on B200 (one process per GPU).

Workload: int8 search, top-100, corpus N = 1,000,000 x d = 768 rows drawn
N(0,1), L2-normalised, symmetric per-row int8 quantised (fp32 scale per row); fp32 queries
quantised the same way inside the kernel; scores int32 dot x s_q x s_row. A step is one fused
scan + top-k call over one batch of queries (default batch 1, the HBM-bound streaming case).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl ours|reference]

N > 1 runs under torchrun as query-parallel replicas (the 772 MB corpus fits every GPU; there
is no exchange step, so no collective on the data path): each rank scans its own queries
against its own copy, timing is the max over ranks and `value` is all ranks' queries / time.

--impl reference times the reference's own CPU search path (cpuCosineSimilarity +
cpuTopKIndices from tests/cpp/cpu_reference.hpp, built into oracle/_ref) on all host cores, on
the same corpus dequantised to fp32, each step a bounded sample of queries.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
PKG = ROOT / "zero-copy-gpu-vector-search-re-ranking-engine_b200"
sys.path.insert(0, str(PKG))

N_DOCS = 1_000_000
DIM = 768
TOP_K = 100
NUM_QUERIES = 1024
CORPUS_SEED = 2001
QUERY_SEED = 2002
METRIC = "queries/sec and p50 query latency at 1/2/4/8 B200; scan HBM GB/s vs peak"
UNIT = "queries/s"


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


def dist_env():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("LOCAL_RANK", "0")),
            int(os.environ.get("WORLD_SIZE", "1")))


def make_corpus(torch, device, seed):
    """N(0,1) rows, L2-normalised in fp32, per-row int8: s = max|x|/127, q = clamp(rint(x/s))."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    codes = torch.empty((N_DOCS, DIM), dtype=torch.int8, device=device)
    scales = torch.empty(N_DOCS, dtype=torch.float32, device=device)
    chunk = 100_000
    for start in range(0, N_DOCS, chunk):
        x = torch.randn((min(chunk, N_DOCS - start), DIM), generator=g, device=device, dtype=torch.float32)
        x = x / x.norm(dim=1, keepdim=True)
        s = x.abs().amax(dim=1) / 127.0
        s = torch.where(s > 0, s, torch.ones_like(s))
        q = torch.round(x * (1.0 / s)[:, None]).clamp_(-127, 127).to(torch.int8)
        codes[start:start + q.shape[0]] = q
        scales[start:start + q.shape[0]] = s
    return codes, scales


def make_queries(torch, device, seed, count):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    x = torch.randn((count, DIM), generator=g, device=device, dtype=torch.float32)
    return (x / x.norm(dim=1, keepdim=True)).contiguous()


class ClockSampler:
    """Samples SM clocks and clock-event (throttle) reasons during the timed region.

    Polls NVML from a thread every `interval_s` (a timed region can be only tens of ms long);
    falls back to an `nvidia-smi -lms` subprocess when NVML is unavailable. Read-only: no
    setting of the GPU is changed.
    """

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, cuda_index: int, interval_s: float = 0.002):
        self.cuda_index = cuda_index
        self.interval_s = interval_s
        self.samples = []          # (sm_mhz, reason bitmask)
        self.max_mhz = None
        self.proc = None
        self.thread = None
        self.stop = None
        self.nvml = None

    def _poll(self, handle):
        nv = self.nvml
        while not self.stop.is_set():
            try:
                self.samples.append((float(nv.nvmlDeviceGetClockInfo(handle, nv.NVML_CLOCK_SM)),
                                     int(nv.nvmlDeviceGetCurrentClocksEventReasons(handle))))
            except Exception:  # noqa: BLE001 - a failed read only loses one sample
                pass
            self.stop.wait(self.interval_s)

    def __enter__(self):
        import threading

        try:
            import pynvml as nv
            import torch

            nv.nvmlInit()
            handle = nv.nvmlDeviceGetHandleByIndex(torch.cuda._get_nvml_device_index(self.cuda_index))
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(handle, nv.NVML_CLOCK_SM))
            self.nvml = nv
            self.stop = threading.Event()
            self.thread = threading.Thread(target=self._poll, args=(handle,), daemon=True)
            self.thread.start()
            return self
        except Exception:  # noqa: BLE001 - fall back to nvidia-smi
            self.nvml = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.cuda_index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "20"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.thread is not None:
            self.stop.set()
            self.thread.join()
            return
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            for ln in out.splitlines():
                parts = [p.strip() for p in ln.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    mhz = float(parts[1])
                    self.max_mhz = float(parts[2])
                except ValueError:
                    continue
                mask = sum(1 << i for i, flag in enumerate(parts[5:9]) if flag.lower() == "active")
                self.samples.append((mhz, mask))

    def summary(self):
        reasons = set()
        for _, mask in self.samples:
            if self.nvml is not None:
                for name, const in self.REASONS:
                    if mask & getattr(self.nvml, const):
                        reasons.add(name)
            else:
                for i, (name, _) in enumerate(self.REASONS):
                    if mask & (1 << i):
                        reasons.add(name)
        sm = [mhz for mhz, _ in self.samples]
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(sm),
                "source": "nvml" if self.nvml is not None else "nvidia-smi"}


def measured_peaks():
    try:
        return json.loads((ROOT / "MEASURED_PEAKS.json").read_text()), "measured"
    except (OSError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


def profiled_traffic(workload: str):
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu summary, if any."""
    path = ROOT / "profiles" / "traffic.json"
    try:
        return json.loads(path.read_text()).get(workload)
    except (OSError, ValueError):
        return None


def cpu_baseline(codes_host, scales_host, queries_host, budget_s=12.0):
    """Times the reference CPU path on a bounded query sample; returns the cpu_baseline dict."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import ctypes

    import oracle

    threads = os.cpu_count() or 1
    ref = oracle.ref_lib()
    if ref is None:
        try:
            oracle.build()
        except Exception:  # noqa: BLE001 - building the reference needs its tree
            pass
        ref = oracle.ref_lib()
    if ref is not None:
        corpus = codes_host.astype(np.float32) * scales_host[:, None]
        # Chunks of one query per thread until about `budget_s` of CPU time (or the query set)
        # is used up.
        chunk = max(1, min(len(queries_host), threads))
        out = np.empty((chunk, TOP_K), dtype=np.int32)
        done, elapsed = 0, 0.0
        while done < len(queries_host) and (done == 0 or elapsed < budget_s):
            q = np.ascontiguousarray(queries_host[done:done + chunk])
            elapsed += ref.refcpu_search(corpus.ctypes.data_as(ctypes.c_void_p), N_DOCS, DIM,
                                         q.ctypes.data_as(ctypes.c_void_p), q.shape[0], TOP_K, threads,
                                         out.ctypes.data_as(ctypes.c_void_p))
            done += q.shape[0]
        return {"value": done / elapsed, "unit": UNIT, "cores": min(threads, chunk), "kind": "reference",
                "sample": f"{done} queries x full {N_DOCS}x{DIM} corpus (dequantised fp32), "
                          f"cpuCosineSimilarity + cpuTopKIndices, {min(threads, chunk)} threads",
                "seconds": elapsed}
    # Oracle port fallback (single thread, exact per-row int8 arithmetic).
    sample = 2
    t0 = time.perf_counter()
    oracle.scan_topk(codes_host, oracle.DTYPE_I8_ROW, DIM, queries_host[:sample], TOP_K, row_scales=scales_host)
    elapsed = time.perf_counter() - t0
    return {"value": sample / elapsed, "unit": UNIT, "cores": 1, "kind": "port",
            "sample": f"{sample} queries x full corpus, oracle/oracle.c, 1 thread", "seconds": elapsed}


def run_reference(args):
    rank, _, world = dist_env()
    if rank != 0:
        return
    import torch

    device = "cuda" if torch.cuda.is_available() else "cpu"
    codes, scales = make_corpus(torch, device, CORPUS_SEED)
    queries = make_queries(torch, device, QUERY_SEED, NUM_QUERIES)
    codes_h, scales_h, q_h = codes.cpu().numpy(), scales.cpu().numpy(), queries.cpu().numpy()
    del codes, scales
    sys.path.insert(0, str(ROOT / "oracle"))
    import ctypes

    import oracle

    ref = oracle.ref_lib()
    threads = os.cpu_count() or 1
    if ref is None:
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libzcgvs_refcpu.so was not built"}))
        return
    corpus = codes_h.astype(np.float32) * scales_h[:, None]
    sample = max(1, min(NUM_QUERIES, threads))
    times = []
    out = np.empty((sample, TOP_K), dtype=np.int32)
    for step in range(args.warmup + args.steps):
        q = np.ascontiguousarray(q_h[(step * sample) % NUM_QUERIES:][:sample])
        n = q.shape[0]
        t = ref.refcpu_search(corpus.ctypes.data_as(ctypes.c_void_p), N_DOCS, DIM,
                              q.ctypes.data_as(ctypes.c_void_p), n, TOP_K, threads,
                              out.ctypes.data_as(ctypes.c_void_p))
        if step >= args.warmup:
            times.append((n, t))
    total_q = sum(n for n, _ in times)
    total_t = sum(t for _, t in times)
    value = total_q / total_t
    line = {"metric": METRIC, "value": value, "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total_t / len(times),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": "cfg2_int8_1Mx768_top100", "batch": sample, "docs": N_DOCS, "dim": DIM,
                       "k": TOP_K, "note": "reference CPU path on the corpus dequantised to fp32"},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": min(threads, sample), "kind": "reference",
                             "sample": f"{sample} queries per step over the full corpus"},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


def run_ours(args):
    import torch
    import torch.distributed as dist

    import zcgvs_sm100 as zc

    rank, local_rank, world = dist_env()
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", init_method="env://", device_id=device,
                                timeout=__import__("datetime").timedelta(seconds=120))

    codes, scales = make_corpus(torch, device, CORPUS_SEED)
    queries = make_queries(torch, device, QUERY_SEED + rank, NUM_QUERIES)
    B = args.batch
    k = TOP_K
    stream = torch.cuda.current_stream()
    ws = zc.Workspace(device)
    out_idx = torch.empty((B, k), dtype=torch.int32, device=device)
    out_val = torch.empty((B, k), dtype=torch.float32, device=device)
    nbatches = max(1, NUM_QUERIES // B)

    def step(i):
        q = queries[(i % nbatches) * B:(i % nbatches) * B + B]
        zc.scan_topk(codes, zc.DTYPE_I8_ROW, DIM, q, k, row_scales=scales, workspace=ws,
                     out=(out_idx, out_val), stream=stream)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()

    events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(args.steps)]
    with ClockSampler(local_rank) as clocks:
        t_start = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        t_start.record(stream)
        for i in range(args.steps):
            events[i][0].record(stream)
            step(i)
            events[i][1].record(stream)
        t_end.record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    elapsed_ms = t_start.elapsed_time(t_end)
    per_step = sorted(a.elapsed_time(b) for a, b in events)
    kernel_ms = sum(per_step) / len(per_step)
    if world > 1:
        t = torch.tensor([elapsed_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed_ms = float(t.item())
    status = ws.status()

    # End to end through the public API with host buffers: pinned host queries -> device,
    # fused scan + top-k, results -> pinned host, synchronised every step (what a caller sees).
    h_queries = queries.cpu().pin_memory()
    h_idx = torch.empty((B, k), dtype=torch.int32).pin_memory()
    h_val = torch.empty((B, k), dtype=torch.float32).pin_memory()
    d_q = torch.empty((B, DIM), dtype=torch.float32, device=device)
    e2e_steps = max(10, args.steps // 2)

    def e2e_step(i):
        j = (i % nbatches) * B
        d_q.copy_(h_queries[j:j + B], non_blocking=True)
        zc.scan_topk(codes, zc.DTYPE_I8_ROW, DIM, d_q, k, row_scales=scales, workspace=ws,
                     out=(out_idx, out_val), stream=stream)
        h_idx.copy_(out_idx, non_blocking=True)
        h_val.copy_(out_val, non_blocking=True)
        stream.synchronize()

    for i in range(3):
        e2e_step(i)
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        e2e_step(i)
    e2e_s = time.perf_counter() - t0
    if world > 1:
        t = torch.tensor([e2e_s], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(codes.cpu().numpy(), scales.cpu().numpy(), queries.cpu().numpy())

    if rank == 0:
        peaks, peak_kind = measured_peaks()
        algo_bytes = N_DOCS * (DIM + 4) + B * DIM * 4 + B * k * 8
        achieved_gbs = algo_bytes / (kernel_ms * 1e-3) / 1e9
        peak = float(peaks["hbm_gbs"])
        workload = f"cfg2_int8row_1Mx768_top100_b{B}"
        traffic = profiled_traffic(workload)
        line = {
            "metric": METRIC, "value": world * B * args.steps / (elapsed_ms * 1e-3), "unit": UNIT,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": elapsed_ms / args.steps, "p50_ms": per_step[len(per_step) // 2],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic",
            "config": {"workload": workload, "docs": N_DOCS, "dim": DIM, "k": TOP_K, "batch": B,
                       "storage": "int8 per-row scale", "parallelism": f"replicas{world}",
                       "l2": "inputs larger than L2 (772 MB corpus vs 126 MB L2)"},
            "roofline": {"bound": "hbm", "achieved": achieved_gbs, "peak": peak, "unit": "GB/s",
                         "frac": achieved_gbs / peak, "traffic": traffic,
                         "peak_source": peak_kind,
                         "kernel": "zc::scan_fast_kernel<kModeI8R,3>" if B == 1 else "zc::scan_kernel<kModeI8R,QB>",
                         "algorithmic_bytes_per_launch": algo_bytes},
            "e2e": {"value": world * B * e2e_steps / e2e_s, "unit": UNIT,
                    "h2d_bytes_per_step": B * DIM * 4, "d2h_bytes_per_step": B * k * 8},
            "gpu_launches": args.steps,
            "clocks": clocks.summary(),
            "device_status": status,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
