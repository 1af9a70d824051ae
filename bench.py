"""Benchmark of the search hot path on B200 (one process per GPU).

Default workload (the one its headline metric is quoted on): int8 search,
top-100, corpus N = 1,000,000 x d = 768 rows drawn N(0,1), L2-normalised, symmetric per-row
int8 quantised (fp32 scale per row); fp32 queries quantised the same way inside the kernel;
scores int32 dot x s_q x s_row. A step is one fused scan + top-k call over one batch of
queries (default batch 1, the HBM-bound streaming case).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload cfg2|cfg2_b1024|cfg1|cfg3|cfg4|cfg5] [--batch B]

The other BASELINE configs run the same timing contract through --workload:
  cfg1       exact fp32 inner product, 5,183 x 384, top-10, batch 1 (latency-bound, L2-resident)
  cfg2_b1024 config 2 at batch 1,024 (the tensor-core path)
  cfg3       1-bit codes 10M x 1024 -> Hamming top-1,000 -> fp16 rescore to top-10, batch 64
  cfg4       fp16 50M x 768, batch 4,096, top-100 (tensor cores); N > 1 shards rows
  cfg5       hybrid BM25 + fp16 dense (2M docs, d = 384), top-10, batch 1
All inputs are seeded synthetic data with the BASELINE shapes and distributions (no datasets
are available offline).

N > 1 runs under torchrun, one rank per GPU. Configs whose corpus fits one GPU run
query-parallel replicas (no collective on the data path, "scaling": "weak"); cfg4 shards its
rows across the ranks and merges the per-shard top-k with one NCCL all-gather per step
("scaling": "strong"). Timing is the max over ranks.

--impl reference times the reference's own CPU search path (cpuCosineSimilarity +
cpuTopKIndices from tests/cpp/cpu_reference.hpp, built into oracle/_ref) on all host cores,
on the same corpus dequantised to fp32, each step a bounded sample of queries.
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

METRIC = "queries/sec and p50 query latency at 1/2/4/8 B200; scan HBM GB/s vs peak"
UNIT = "queries/s"


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=None)
    ap.add_argument("--batch", type=int, default=None)
    ap.add_argument("--workload", default="cfg2",
                    choices=["cfg1", "cfg2", "cfg2_b1024", "cfg3", "cfg4", "cfg5"])
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--docs", type=int, default=None,
                    help="corpus rows instead of the workload's (small cases for profiler captures)")
    ap.add_argument("--no-sharded", action="store_true",
                    help="skip the row-sharded config 4 measurement that follows the replica workloads")
    ap.add_argument("--sharded-docs", type=int, default=None,
                    help="corpus rows of the row-sharded measurement (default: config 4's 50,000,000)")
    ap.add_argument("--no-searcher", action="store_true",
                    help="skip the end-to-end rate through the C++ Searcher (one-query workloads, one GPU)")
    return ap.parse_args()


def dist_env():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("LOCAL_RANK", "0")),
            int(os.environ.get("WORLD_SIZE", "1")))


def measured_peaks():
    try:
        return json.loads((ROOT / "MEASURED_PEAKS.json").read_text()), "measured"
    except (OSError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


def profiled_traffic(workload: str):
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu summary, if any."""
    try:
        return json.loads((ROOT / "profiles" / "traffic.json").read_text()).get(workload)
    except (OSError, ValueError):
        return None


def oracle_mod():
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle

    return oracle


def ref_cpu():
    """The reference's own CPU search library (oracle/_ref), building it if the tree is here."""
    oracle = oracle_mod()
    ref = oracle.ref_lib()
    if ref is None:
        try:
            oracle.build()
        except Exception:  # noqa: BLE001 - building the reference needs its tree
            pass
        ref = oracle.ref_lib()
    return ref


def ref_search_rate(corpus_f32, queries, k, budget_s, rows_total=None):
    """Queries/s of the reference CPU path (cpuCosineSimilarity + cpuTopKIndices, all host
    threads) over `corpus_f32`, in chunks of one query per thread until about `budget_s` of CPU
    time. When the corpus is a row prefix of `rows_total` rows the rate is scaled by
    prefix / total (the path is linear in the rows)."""
    import ctypes

    ref = ref_cpu()
    if ref is None:
        return None
    threads = os.cpu_count() or 1
    corpus_f32 = np.ascontiguousarray(corpus_f32, dtype=np.float32)
    n, d = corpus_f32.shape
    chunk = max(1, min(len(queries), threads))
    out = np.empty((chunk, k), dtype=np.int32)
    done, elapsed = 0, 0.0
    while done < len(queries) and (done == 0 or elapsed < budget_s):
        q = np.ascontiguousarray(queries[done:done + chunk], dtype=np.float32)
        elapsed += ref.refcpu_search(corpus_f32.ctypes.data_as(ctypes.c_void_p), n, d,
                                     q.ctypes.data_as(ctypes.c_void_p), q.shape[0], k, threads,
                                     out.ctypes.data_as(ctypes.c_void_p))
        done += q.shape[0]
    rate = done / elapsed
    scale = 1.0 if rows_total is None else n / rows_total
    return {"value": rate * scale, "unit": UNIT, "cores": min(threads, chunk), "kind": "reference",
            "sample": (f"{done} queries x {n}x{d} fp32 corpus, cpuCosineSimilarity + cpuTopKIndices, "
                       f"{min(threads, chunk)} threads" +
                       ("" if rows_total is None else f"; extrapolated to {rows_total} rows (x{scale:.4g})")),
            "seconds": elapsed}


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


def normal_rows(torch, device, rows, dim, seed, dtype, chunk=1 << 20):
    """N(0,1) rows, L2-normalised in fp32, stored as `dtype`; generated chunk by chunk."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    out = torch.empty((rows, dim), dtype=dtype, device=device)
    for start in range(0, rows, chunk):
        x = torch.randn((min(chunk, rows - start), dim), generator=g, device=device, dtype=torch.float32)
        out[start:start + x.shape[0]] = (x / x.norm(dim=1, keepdim=True)).to(dtype)
    return out


def int8_rows(torch, device, rows, dim, seed, chunk=1 << 17):
    """N(0,1) rows, L2-normalised in fp32, per-row int8: s = max|x|/127, q = clamp(rint(x/s))."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    codes = torch.empty((rows, dim), dtype=torch.int8, device=device)
    scales = torch.empty(rows, dtype=torch.float32, device=device)
    for start in range(0, rows, chunk):
        x = torch.randn((min(chunk, rows - start), dim), generator=g, device=device, dtype=torch.float32)
        x = x / x.norm(dim=1, keepdim=True)
        s = x.abs().amax(dim=1) / 127.0
        s = torch.where(s > 0, s, torch.ones_like(s))
        codes[start:start + x.shape[0]] = torch.round(x * (1.0 / s)[:, None]).clamp_(-127, 127).to(torch.int8)
        scales[start:start + x.shape[0]] = s
    return codes, scales


def pack_signs(torch, x):
    """Sign bits of fp rows: bit b of word w = dim 32 w + b, set when x >= 0 (the reference's
    launchPackBinary convention)."""
    rows, dim = x.shape
    bits = (x >= 0).to(torch.int64).reshape(rows, dim // 32, 32)
    weights = torch.ones(32, dtype=torch.int64, device=x.device) << torch.arange(32, device=x.device)
    words = (bits * weights).sum(dim=2)
    return torch.where(words >= 2 ** 31, words - 2 ** 32, words).to(torch.int32).contiguous()


def native_sharded_searcher(torch, zc, world, rank, total_rows):
    """This rank's zcgvs_sharded handle (NCCL communicator of its own); rank 0 makes the NCCL id
    and the process group (when there is one) carries it to the others."""
    nccl_id = zc.ShardedSearcher.unique_id() if rank == 0 else None
    if world > 1:
        import torch.distributed as dist

        box = [nccl_id]
        dist.broadcast_object_list(box, src=0)
        nccl_id = box[0]
    return zc.ShardedSearcher(nccl_id, world, rank, total_rows)


# --------------------------------------------------------------------------------------------
# Workloads
# --------------------------------------------------------------------------------------------
class Workload:
    """A BASELINE configuration: inputs on the device, one step, an end-to-end step through host
    buffers, and the roofline / CPU-baseline bookkeeping of its dominant kernel."""

    scaling = "weak"
    steps, warmup = 200, 10
    # Library kernel-timing tags of the dominant kernel(s), each launched once per step: their
    # CUDA-event durations (a second, instrumented pass over the same steps) divide the
    # roofline's algorithmic work.
    dominant = ("scan",)

    def kernel_ms(self, kern, steps):
        return sum(kern[t][0] for t in self.dominant) / steps

    # Arguments of the package's searcher_e2e program for this workload's shape (one-query
    # workloads), or None: the end-to-end rate through the C++ drop-in Searcher.
    def searcher_args(self):
        return None

    # Batch-1 workloads replay CUDA graphs, as a serving loop does (the reference's Searcher
    # captures its pipeline the same way): one graph per query of a pool for the device-resident
    # steps, and one over the device staging buffers for the end-to-end steps. The graphs hold
    # the same library launches as a direct call; the kernel-timing pass makes direct calls.
    graphs = False
    pool = 64

    def step(self, i, stream):
        g = getattr(self, "g_step", None)
        if g:
            g[i % len(g)].replay()
        else:
            self.step_direct(i, stream)

    def search_staged(self, stream):
        g = getattr(self, "g_e2e", None)
        if g is not None:
            g.replay()
        else:
            self.search_staged_direct(stream)

    # End-to-end step of a batch-1 workload: the pinned host -> device copy of the query and the
    # search, whose last kernel writes the result straight into pinned host memory (device-
    # accessible under unified addressing: no device -> host copy), replayed as one graph per
    # query of the pool; else the copies and the search run one after another.
    def e2e_step(self, i, stream):
        g = getattr(self, "g_e2e_full", None)
        if g:
            g[i % len(g)].replay()
        else:
            self.stage_in(i)
            self.search_staged(stream)
            self.stage_out()
        stream.synchronize()
        return self.e2e_bytes()

    def capture(self, torch):
        if not self.graphs:
            return
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for i in range(self.pool):
                self.step_direct(i, s)
            self.search_staged_direct(s)
        s.synchronize()
        self.g_step = []
        for i in range(self.pool):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                self.step_direct(i, s)
            self.g_step.append(g)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            self.search_staged_direct(s)
        self.g_e2e = g
        torch.cuda.synchronize()
        try:
            with torch.cuda.stream(s):
                self.search_staged_direct(s, out=self.h_out)
            s.synchronize()
            full = []
            for i in range(self.pool):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=s):
                    self.stage_in(i)
                    self.search_staged_direct(s, out=self.h_out)
                full.append(g)
            self.g_e2e_full = full
        except RuntimeError:
            self.g_e2e_full = None
        torch.cuda.synchronize()

    @staticmethod
    def tensor_peak(peaks, kind, sustained=False):
        # The burst figure for a kernel timed on its own, the sustained one (seconds of
        # back-to-back GEMMs under the power cap) for a kernel that runs for seconds; int8 dense
        # = twice bf16 dense on B200.
        key, what = ("bf16_tflops_sustained", "sustained") if sustained and "bf16_tflops_sustained" in peaks else (
            "bf16_tflops", "burst")
        if kind == "i8":
            return 2.0 * float(peaks[key]), f"2 x measured bf16 {what} (int8 dense = 2 x bf16 dense)"
        return float(peaks[key]), f"measured bf16 {what}"


class Cfg2(Workload):
    """per-row int8 1M x 768, top-100."""

    N, D, K, NQ = 1_000_000, 768, 100, 1024
    dtype = "int8"

    @property
    def dominant(self):
        return ("gemm_filter",) if self.B >= 64 else ("scan",)

    def __init__(self, batch):
        self.B = batch
        self.name = f"cfg2_int8row_1Mx768_top100_b{batch}"
        if batch >= 64:
            self.steps, self.warmup = 20, 3

    def searcher_args(self):
        if self.B != 1:
            return None
        return [f"docs={self.N}", f"dim={self.D}", "dtype=4", f"k={self.K}", "metric=0"]

    units = property(lambda self: self.B)
    launches = property(lambda self: 12 if self.B >= 64 else 1)

    def setup(self, torch, zc, device, rank, world):
        self.torch, self.zc = torch, zc
        self.codes, self.scales = int8_rows(torch, device, self.N, self.D, 2001)
        self.queries = normal_rows(torch, device, self.NQ, self.D, 2002 + rank, torch.float32)
        self.ws = zc.Workspace(device)
        self.out = (torch.empty((self.B, self.K), dtype=torch.int32, device=device),
                    torch.empty((self.B, self.K), dtype=torch.float32, device=device))
        self.h_queries = self.queries.cpu().pin_memory()
        self.h_out = (torch.empty((self.B, self.K), dtype=torch.int32).pin_memory(),
                      torch.empty((self.B, self.K), dtype=torch.float32).pin_memory())
        self.d_q = torch.empty((self.B, self.D), dtype=torch.float32, device=device)

    def _q(self, i, src):
        nb = max(1, self.NQ // self.B)
        j = (i % nb) * self.B
        return src[j:j + self.B]

    graphs = property(lambda self: self.B == 1)

    def step_direct(self, i, stream):
        self.zc.scan_topk(self.codes, self.zc.DTYPE_I8_ROW, self.D, self._q(i, self.queries), self.K,
                          row_scales=self.scales, workspace=self.ws, out=self.out, stream=stream)

    def search_staged_direct(self, stream, out=None):
        self.zc.scan_topk(self.codes, self.zc.DTYPE_I8_ROW, self.D, self.d_q, self.K, row_scales=self.scales,
                          workspace=self.ws, out=out or self.out, stream=stream)

    def stage_in(self, i):
        self.d_q.copy_(self._q(i, self.h_queries), non_blocking=True)

    def stage_out(self):
        self.h_out[0].copy_(self.out[0], non_blocking=True)
        self.h_out[1].copy_(self.out[1], non_blocking=True)

    def e2e_bytes(self):
        return self.B * self.D * 4, self.B * self.K * 8

    def config(self, world):
        return {"workload": self.name, "docs": self.N, "dim": self.D, "k": self.K, "batch": self.B,
                "storage": "int8 per-row scale", "parallelism": f"replicas{world}",
                "l2": "inputs larger than L2 (772 MB corpus vs 126 MB L2)"}

    def roofline(self, kernel_ms, peaks, peak_kind):
        if self.B >= 64:
            ops = 2.0 * self.B * self.N * self.D
            achieved = ops / (kernel_ms * 1e-3) / 1e12
            peak, src = self.tensor_peak(peaks, "i8")
            return {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TOP/s", "frac": achieved / peak,
                    "traffic": profiled_traffic(self.name), "peak_source": f"{peak_kind}: {src}",
                    "kernel": "zc::gemm::gemm_scan_kernel<kModeI8R,kFilter>",
                    "algorithmic_ops_per_launch": ops}
        algo = self.N * (self.D + 4) + self.B * self.D * 4 + self.B * self.K * 8
        achieved = algo / (kernel_ms * 1e-3) / 1e9
        peak = float(peaks["hbm_gbs"])
        return {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                "traffic": profiled_traffic(self.name), "peak_source": peak_kind,
                "kernel": "zc::scan_fast_kernel<kModeI8R,3>" if self.B == 1 else "zc::scan_kernel<kModeI8R,QB>",
                "algorithmic_bytes_per_launch": algo}

    def reference_corpus(self):
        return (self.codes.float() * self.scales[:, None]).cpu().numpy()

    def cpu_baseline(self, budget_s):
        return ref_search_rate(self.reference_corpus(), self.queries.cpu().numpy(), self.K, budget_s)


class Cfg1(Workload):
    """exact fp32 inner product, 5,183 x 384, top-10, 300 queries, batch 1."""

    N, D, K, NQ, B = 5183, 384, 10, 300, 1
    name = "cfg1_f32_5183x384_top10_b1"
    dtype = "f32"
    units = 1
    launches = 1
    steps, warmup = 300, 10

    def searcher_args(self):
        return [f"docs={self.N}", f"dim={self.D}", "dtype=0", f"k={self.K}", "metric=0"]

    def setup(self, torch, zc, device, rank, world):
        self.torch, self.zc = torch, zc
        self.corpus = normal_rows(torch, device, self.N, self.D, 1001, torch.float32)
        self.queries = normal_rows(torch, device, self.NQ, self.D, 1002 + rank, torch.float32)
        self.ws = zc.Workspace(device)
        self.out = (torch.empty((1, self.K), dtype=torch.int32, device=device),
                    torch.empty((1, self.K), dtype=torch.float32, device=device))
        self.h_queries = self.queries.cpu().pin_memory()
        self.h_out = (torch.empty((1, self.K), dtype=torch.int32).pin_memory(),
                      torch.empty((1, self.K), dtype=torch.float32).pin_memory())
        self.d_q = torch.empty((1, self.D), dtype=torch.float32, device=device)

    graphs = True

    def step_direct(self, i, stream):
        j = i % self.NQ
        self.zc.scan_topk(self.corpus, self.zc.DTYPE_F32, self.D, self.queries[j:j + 1], self.K,
                          metric=self.zc.METRIC_COSINE, workspace=self.ws, out=self.out, stream=stream)

    def search_staged_direct(self, stream, out=None):
        self.zc.scan_topk(self.corpus, self.zc.DTYPE_F32, self.D, self.d_q, self.K, metric=self.zc.METRIC_COSINE,
                          workspace=self.ws, out=out or self.out, stream=stream)

    def stage_in(self, i):
        j = i % self.NQ
        self.d_q.copy_(self.h_queries[j:j + 1], non_blocking=True)

    def stage_out(self):
        self.h_out[0].copy_(self.out[0], non_blocking=True)
        self.h_out[1].copy_(self.out[1], non_blocking=True)

    def e2e_bytes(self):
        return self.D * 4, self.K * 8

    def config(self, world):
        return {"workload": self.name, "docs": self.N, "dim": self.D, "k": self.K, "batch": 1,
                "storage": "fp32", "metric": "cosine", "parallelism": f"replicas{world}",
                "l2": "corpus (7.96 MB) is L2-resident: latency-bound, no flush between steps"}

    def roofline(self, kernel_ms, peaks, peak_kind):
        algo = self.N * self.D * 4 + self.D * 4 + self.K * 8
        achieved = algo / (kernel_ms * 1e-3) / 1e9
        peak = float(peaks["hbm_gbs"])
        return {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                "traffic": profiled_traffic(self.name), "peak_source": peak_kind,
                "kernel": "zc::scan_fast_kernel<kModeF32,JC>", "algorithmic_bytes_per_launch": algo,
                "note": "L2-resident corpus: the bound is launch latency, the fraction is not an HBM efficiency"}

    def reference_corpus(self):
        return self.corpus.cpu().numpy()

    def cpu_baseline(self, budget_s):
        return ref_search_rate(self.reference_corpus(), self.queries.cpu().numpy(), self.K, budget_s)


class Cfg3(Workload):
    """1-bit codes (128 B/row) of 10M x 1024 fp16 rows, Hamming top-1,000,
    fp16 rescore to top-10, batch 64. With N ranks the rows are split into N shards, each rank
    holding its rows' codes and fp16 rows: per-shard top-1,000 (global ids), an NCCL exchange
    and merge to the global top-1,000, each rank rescoring the candidates it owns, a second
    exchange and merge of the top-10 (sharded.ShardedRescoreSearch, the reference's
    semantics)."""

    N, D, M, K, B, NQ = 10_000_000, 1024, 1000, 10, 64, 4096
    name = "cfg3_bin1024_10M_top1000_f16rescore_top10_b64"
    dtype = "u32 (xor+popc) / f16"
    units = 64
    steps, warmup = 10, 3
    dominant = ("gemm_filter",)
    scaling = "strong"
    # prep, sample, threshold, 3 x (filter, bucket, select), rescore; sharded: two merges more
    # (the two NCCL all-gathers are the library's kernels, not counted)
    launches = property(lambda self: 13 if self.world == 1 else 15)

    def setup(self, torch, zc, device, rank, world):
        import sharded

        self.torch, self.zc, self.world = torch, zc, world
        self.begin, self.end = sharded.shard_bounds(self.N, world, rank)
        rows = self.end - self.begin
        # Each 1M-row block of the global corpus has its own seed, so a shard holds the same rows
        # whatever the number of ranks.
        self.store = torch.empty((rows, self.D), dtype=torch.float16, device=device)
        blk = 1 << 20
        for b0 in range(self.begin // blk * blk, self.end, blk):
            block = normal_rows(torch, device, min(blk, self.N - b0), self.D, 3001 + b0 // blk, torch.float16)
            lo, hi = max(b0, self.begin), min(b0 + block.shape[0], self.end)
            self.store[lo - self.begin:hi - self.begin] = block[lo - b0:hi - b0]
            del block
        self.codes = torch.empty((rows, self.D // 32), dtype=torch.int32, device=device)
        for s in range(0, rows, blk):
            self.codes[s:s + blk] = pack_signs(torch, self.store[s:s + blk])
        self.queries = normal_rows(torch, device, self.NQ, self.D, 3002, torch.float32)
        self.ws = zc.Workspace(device)
        self.cand = (torch.empty((self.B, self.M), dtype=torch.int32, device=device),
                     torch.empty((self.B, self.M), dtype=torch.float32, device=device))
        self.out = (torch.empty((self.B, self.K), dtype=torch.int32, device=device),
                    torch.empty((self.B, self.K), dtype=torch.float32, device=device))
        self.h_queries = self.queries.cpu().pin_memory()
        self.h_out = (torch.empty((self.B, self.K), dtype=torch.int32).pin_memory(),
                      torch.empty((self.B, self.K), dtype=torch.float32).pin_memory())
        self.d_q = torch.empty((self.B, self.D), dtype=torch.float32, device=device)
        self.store_i16 = self.store.view(torch.int16)
        self.search = native_sharded_searcher(torch, zc, world, rank, self.N) if world > 1 else None

    def _run(self, q, stream, graph=True):
        if self.search is not None:
            self.search.rescore_search(self.codes, self.zc.DTYPE_BINARY, self.store_i16, self.zc.DTYPE_F16, self.D, q,
                                       self.M, self.K, metric=self.zc.METRIC_COSINE, graph=graph, out=self.out,
                                       stream=stream)
            return
        self.zc.scan_topk(self.codes, self.zc.DTYPE_BINARY, self.D, q, self.M, workspace=self.ws, out=self.cand,
                          stream=stream)
        self.zc.rescore_topk(self.store_i16, self.zc.DTYPE_F16, self.D, q, self.cand[0], self.K,
                             metric=self.zc.METRIC_COSINE, out=self.out, stream=stream)

    def step(self, i, stream):
        j = (i % (self.NQ // self.B)) * self.B
        self._run(self.queries[j:j + self.B], stream, graph=True)

    def step_direct(self, i, stream):
        j = (i % (self.NQ // self.B)) * self.B
        self._run(self.queries[j:j + self.B], stream, graph=False)

    def e2e_step(self, i, stream):
        j = (i % (self.NQ // self.B)) * self.B
        self.d_q.copy_(self.h_queries[j:j + self.B], non_blocking=True)
        self._run(self.d_q, stream)
        self.h_out[0].copy_(self.out[0], non_blocking=True)
        self.h_out[1].copy_(self.out[1], non_blocking=True)
        stream.synchronize()
        return self.B * self.D * 4, self.B * self.K * 8

    def config(self, world):
        return {"workload": self.name, "docs": self.N, "dim": self.D, "candidates": self.M, "k": self.K,
                "batch": self.B, "storage": "1-bit codes + fp16 rescore store",
                "parallelism": f"rowshard{world}" if world > 1 else "single",
                "l2": "inputs larger than L2 (1.28 GB codes, 20.5 GB rescore store)"}

    def roofline(self, kernel_ms, peaks, peak_kind):
        # Dominant: the filtered tensor-core Hamming scan (1-bit rows expanded to int8 on chip).
        # Its tensor work bounds it before its HBM reads do: 2 B N D int8 ops (0.41 ms at the
        # int8 peak) against N D / 8 bytes of codes (0.20 ms at the HBM peak). Sharded, each
        # rank scans its own rows.
        ops = 2.0 * self.B * (self.end - self.begin) * self.D
        achieved = ops / (kernel_ms * 1e-3) / 1e12
        peak, src = self.tensor_peak(peaks, "i8")
        return {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TOP/s", "frac": achieved / peak,
                "traffic": profiled_traffic(self.name), "peak_source": f"{peak_kind}: {src}",
                "kernel": "zc::gemm::gemm_scan_kernel<kModeBin,kFilter>",
                "algorithmic_ops_per_launch": ops,
                "note": "the MMA runs 128-query blocks: a 64-query batch fills half of each, so frac <= 0.5"}

    def cpu_baseline(self, budget_s):
        # The reference CPU path scans fp32 rows; time it on a 200k-row prefix and scale.
        prefix = 200_000
        corpus = self.store[:prefix].float().cpu().numpy()
        return ref_search_rate(corpus, self.queries[:256].cpu().numpy(), self.K, budget_s, rows_total=self.N)


class Cfg4(Workload):
    """fp16 50M x 768, batch 4,096, top-100 (tensor cores). With N ranks the
    rows are split into N shards; each rank searches its shard (global ids via id_base), one NCCL
    all-gather exchanges the [4096, 100] results and zcgvs_merge_topk merges them."""

    N, D, K, B = 50_000_000, 768, 100, 4096
    name = "cfg4_f16_50Mx768_top100_b4096"
    dtype = "f16"
    units = 4096
    steps, warmup = 6, 3
    scaling = "strong"

    def setup(self, torch, zc, device, rank, world):
        import sharded

        self.torch, self.zc, self.world = torch, zc, world
        self.begin, self.end = sharded.shard_bounds(self.N, world, rank)
        rows = self.end - self.begin
        # Each 1M-row block of the global corpus has its own seed, so a shard holds the same rows
        # whatever the number of ranks.
        self.shard = torch.empty((rows, self.D), dtype=torch.float16, device=device)
        blk = 1 << 20
        for b0 in range(self.begin // blk * blk, self.end, blk):
            block = normal_rows(torch, device, min(blk, self.N - b0), self.D, 4001 + b0 // blk, torch.float16)
            lo, hi = max(b0, self.begin), min(b0 + block.shape[0], self.end)
            self.shard[lo - self.begin:hi - self.begin] = block[lo - b0:hi - b0]
            del block
        self.shard_i16 = self.shard.view(torch.int16)
        self.queries = normal_rows(torch, device, self.B, self.D, 4002, torch.float16).float()
        self.ws = zc.Workspace(device)

        def gemm_local(q, k, id_base):
            return zc.gemm_topk(self.shard_i16, zc.DTYPE_F16, self.D, q, k, metric=zc.METRIC_COSINE,
                                id_base=id_base, workspace=self.ws)

        self.gemm_local = gemm_local
        self.search = native_sharded_searcher(torch, zc, world, rank, self.N) if (world > 1 or self.native) else None
        self.out = (torch.empty((self.B, self.K), dtype=torch.int32, device=device),
                    torch.empty((self.B, self.K), dtype=torch.float32, device=device))
        self.h_queries = self.queries.cpu().pin_memory()
        self.d_q = torch.empty_like(self.queries)

    def __init__(self, native=False):
        # native: search through the row-sharded handle even on one rank (the sharded key's
        # one-GPU point uses the same code path as its N-GPU points).
        self.native = native

    launches = property(lambda self: 12 if self.search is None else 13)
    dominant = ("gemm_filter",)

    def _run(self, q, graph=True):
        if self.search is None:
            return self.gemm_local(q, self.K, 0)
        return self.search.search(self.shard_i16, self.zc.DTYPE_F16, self.D, q, self.K, metric=self.zc.METRIC_COSINE,
                                  tensor_f16=True, graph=graph, out=self.out)

    def step(self, i, stream):
        self._run(self.queries, graph=True)

    def step_direct(self, i, stream):
        self._run(self.queries, graph=False)

    def e2e_step(self, i, stream):
        self.d_q.copy_(self.h_queries, non_blocking=True)
        ids, scores = self._run(self.d_q)
        ids.cpu()
        scores.cpu()
        return self.B * self.D * 4, self.B * self.K * 8

    def config(self, world):
        return {"workload": self.name, "docs": self.N, "dim": self.D, "k": self.K, "batch": self.B,
                "storage": "fp16", "metric": "cosine", "parallelism": f"rowshard{world}",
                "l2": "inputs larger than L2 (77 GB corpus)"}

    def roofline(self, kernel_ms, peaks, peak_kind):
        rows = self.end - self.begin
        flops = 2.0 * self.B * rows * self.D
        achieved = flops / (kernel_ms * 1e-3) / 1e12
        # One filter launch runs for a third of a second and the steps run back to back for
        # seconds under the 1 kW power cap: the sustained GEMM figure is its denominator.
        peak, src = self.tensor_peak(peaks, "f16", sustained=True)
        return {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                "traffic": profiled_traffic(self.name), "peak_source": f"{peak_kind}: {src}",
                "kernel": "zc::gemm::gemm_scan_kernel<kModeF16,kFilter>",
                "algorithmic_flops_per_launch": flops}

    def cpu_baseline(self, budget_s):
        prefix = 200_000
        corpus = self.shard[:prefix].float().cpu().numpy()
        return ref_search_rate(corpus, self.queries[:256].cpu().numpy(), self.K, budget_s, rows_total=self.N)


class Cfg5(Workload):
    """hybrid BM25 + fp16 dense, 2M docs, d = 384, top-10, batch 1. Token
    counts ~ Poisson(200), terms ~ Zipf(1.1) over 30,000, BM25 k1 = 0.9, b = 0.4; queries of
    3-12 Zipf terms, de-duplicated; score = 0.5 * dense + 0.5 * lex / max(lex)."""

    N, D, K, V, NQ = 2_000_000, 384, 10, 30_000, 1000

    def searcher_args(self):
        # The Searcher's hybrid path with a synthetic index of the same statistics (Zipf(1.1)
        # terms, 200 token draws per document, queries of 3-12 terms), built by the program.
        return [f"docs={self.N}", f"dim={self.D}", "dtype=1", f"k={self.K}", "metric=0", f"vocab={self.V}",
                "mean_len=200", "terms=12", "weight=0.5"]
    name = "cfg5_hybrid_bm25_f16_2Mx384_top10_b1"
    dtype = "f16 + f32"
    units = 1
    launches = 2
    steps, warmup = 200, 10
    # One query: the hybrid scan (dense rows and BM25 in one kernel) and the blend + top-k kernel;
    # other shapes: the lexical kernel and the blending scan.
    dominant = ("lexical", "scan", "hybrid_select")

    def kernel_ms(self, kern, steps):
        return sum(kern[t][0] for t in self.dominant if t in kern) / steps

    def setup(self, torch, zc, device, rank, world):
        import lexical_index as li

        self.torch, self.zc = torch, zc
        offsets, docs, weights = li.synthetic_corpus(self.N, self.V, 200.0, 1.1, 5001, device=device, k1=0.9, b=0.4)
        self.index = zc.LexicalIndex(offsets, docs, weights, device=device)
        self.offsets_h = offsets.cpu().numpy()
        self.dense = normal_rows(torch, device, self.N, self.D, 5002, torch.float16)
        self.dense_i16 = self.dense.view(torch.int16)
        self.queries = normal_rows(torch, device, self.NQ, self.D, 5003 + rank, torch.float32)
        self.terms_h = li.synthetic_queries(self.NQ, self.V, 1.1, 5004 + rank)
        self.terms = torch.from_numpy(self.terms_h).to(device)
        self.ws = zc.Workspace(device)
        self.out = (torch.empty((1, self.K), dtype=torch.int32, device=device),
                    torch.empty((1, self.K), dtype=torch.float32, device=device))
        self.h_queries = self.queries.cpu().pin_memory()
        self.h_terms = torch.from_numpy(self.terms_h).pin_memory()
        self.h_out = (torch.empty((1, self.K), dtype=torch.int32).pin_memory(),
                      torch.empty((1, self.K), dtype=torch.float32).pin_memory())
        self.d_q = torch.empty((1, self.D), dtype=torch.float32, device=device)
        self.d_t = torch.empty((1, self.terms_h.shape[1]), dtype=torch.int32, device=device)
        df = np.diff(self.offsets_h)
        self.sum_df = [int(df[t[t >= 0]].sum()) for t in self.terms_h]

    def _run(self, q, t, stream, out=None):
        self.zc.hybrid_topk(self.dense_i16, self.zc.DTYPE_F16, self.D, q, self.K, self.index, t, 0.5,
                            metric=self.zc.METRIC_COSINE, workspace=self.ws, out=out or self.out, stream=stream)

    graphs = True

    def step_direct(self, i, stream):
        j = i % self.NQ
        self._run(self.queries[j:j + 1], self.terms[j:j + 1], stream)

    def search_staged_direct(self, stream, out=None):
        self._run(self.d_q, self.d_t, stream, out)

    def stage_in(self, i):
        j = i % self.NQ
        self.d_q.copy_(self.h_queries[j:j + 1], non_blocking=True)
        self.d_t.copy_(self.h_terms[j:j + 1], non_blocking=True)

    def stage_out(self):
        self.h_out[0].copy_(self.out[0], non_blocking=True)
        self.h_out[1].copy_(self.out[1], non_blocking=True)

    def e2e_bytes(self):
        return self.D * 4 + self.terms_h.shape[1] * 4, self.K * 8

    def config(self, world):
        return {"workload": self.name, "docs": self.N, "dim": self.D, "vocab": self.V, "k": self.K, "batch": 1,
                "storage": "fp16 dense + CSR BM25 (k1 0.9, b 0.4)", "dense_weight": 0.5,
                "mean_sum_df": float(np.mean(self.sum_df)), "parallelism": f"replicas{world}",
                "l2": "inputs larger than L2 (1.54 GB dense)"}

    def roofline(self, kernel_ms, peaks, peak_kind):
        algo = self.N * self.D * 2 + 8 * float(np.mean(self.sum_df)) + self.N * 4 * 2 + self.D * 4
        achieved = algo / (kernel_ms * 1e-3) / 1e9
        peak = float(peaks["hbm_gbs"])
        return {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                "traffic": profiled_traffic(self.name), "peak_source": peak_kind,
                "kernel": "zc::scan_fast_kernel<kModeF16,3,true> (dense rows + BM25 in one kernel) + "
                          "zc::hybrid_select_kernel (blend + top-k), one launch each per step",
                "algorithmic_bytes_per_launch_pair": algo,
                "note": "bytes = dense rows + 8 B per posting of the query's terms + lexical scores written and read"}

    def cpu_baseline(self, budget_s):
        oracle = oracle_mod()
        dense_bits = self.dense.view(self.torch.int16).cpu().numpy().view(np.uint16)
        docs = self.index.docs.cpu().numpy()
        weights = self.index.weights.cpu().numpy()
        queries = self.queries.cpu().numpy()
        from concurrent.futures import ThreadPoolExecutor

        # One query per host thread at a time (the oracle's C loops run outside the GIL).
        threads = os.cpu_count() or 1
        oracle.lib()  # loaded once, before the threads

        def one(i):
            oracle.hybrid_topk(dense_bits, oracle.DTYPE_F16, self.D, queries[i:i + 1], self.K, self.offsets_h,
                               docs, weights, self.V, self.terms_h[i:i + 1], 0.5, metric=oracle.METRIC_COSINE)

        done, t0 = 0, time.perf_counter()
        with ThreadPoolExecutor(max_workers=threads) as pool:
            while done + threads <= len(queries) and (done == 0 or time.perf_counter() - t0 < budget_s):
                list(pool.map(one, range(done, done + threads)))
                done += threads
        elapsed = time.perf_counter() - t0
        return {"value": done / elapsed, "unit": UNIT, "cores": threads, "kind": "port",
                "sample": f"{done} queries over the full corpus, oracle hybrid (reference loops restated), "
                          f"{threads} threads, one query each",
                "seconds": elapsed}


def make_workload(args):
    if args.workload == "cfg2":
        wl = Cfg2(args.batch or 1)
    elif args.workload == "cfg2_b1024":
        wl = Cfg2(args.batch or 1024)
    else:
        wl = {"cfg1": Cfg1, "cfg3": Cfg3, "cfg4": Cfg4, "cfg5": Cfg5}[args.workload]()
    if args.docs:
        wl.N = args.docs
    return wl


# --------------------------------------------------------------------------------------------
# Arms
# --------------------------------------------------------------------------------------------
def run_reference(args):
    """The reference's CPU search path (all host threads) on the workload's corpus, as fp32."""
    rank, _, world = dist_env()
    if rank != 0:
        return
    import ctypes

    import torch

    wl = make_workload(args)
    steps = args.steps if args.steps is not None else wl.steps
    warmup = args.warmup if args.warmup is not None else wl.warmup
    if not isinstance(wl, (Cfg1, Cfg2)):
        run_reference_sampled(args, wl, steps, warmup)
        return
    ref = ref_cpu()
    if ref is None:
        emit(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libzcgvs_refcpu.so was not built"}))
        return
    device = "cuda" if torch.cuda.is_available() else "cpu"
    import zcgvs_sm100 as zc

    wl.setup(torch, zc, device, 0, 1)  # the seeded inputs are generated on the device
    corpus = np.ascontiguousarray(wl.reference_corpus(), dtype=np.float32)
    queries = wl.queries.cpu().numpy()
    threads = os.cpu_count() or 1
    sample = max(1, min(len(queries), threads))
    out = np.empty((sample, wl.K), dtype=np.int32)
    times = []
    for step in range(warmup + steps):
        q = np.ascontiguousarray(np.roll(queries, -step * sample, axis=0)[:sample])
        t = ref.refcpu_search(corpus.ctypes.data_as(ctypes.c_void_p), corpus.shape[0], corpus.shape[1],
                              q.ctypes.data_as(ctypes.c_void_p), q.shape[0], wl.K, threads,
                              out.ctypes.data_as(ctypes.c_void_p))
        if step >= warmup:
            times.append((q.shape[0], t))
    value = sum(n for n, _ in times) / sum(t for _, t in times)
    line = {"metric": METRIC, "value": value, "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
            "steps": steps, "warmup": warmup, "ms_per_step": 1e3 * sum(t for _, t in times) / len(times),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": dict(wl.config(1), note="reference CPU path on the corpus as fp32, all host threads"),
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": min(threads, sample), "kind": "reference",
                             "sample": f"{sample} queries per step over the full corpus"},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    emit(json.dumps(line))


def run_reference_sampled(args, wl, steps, warmup):
    """Reference arm for configs 3, 4 and 5, whose CPU path takes minutes per query over the
    full corpus: every step is the workload's bounded CPU sample (the same code as the ours
    line's cpu_baseline: the reference's CPU search over a row prefix of the corpus, scaled to the
    full row count, for configs 3 and 4; the restated hybrid chain on every host thread for
    config 5), with about 90 s of CPU time over the whole run."""
    import torch

    import zcgvs_sm100 as zc

    if ref_cpu() is None and not isinstance(wl, Cfg5):
        emit(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libzcgvs_refcpu.so was not built"}))
        return
    device = "cuda" if torch.cuda.is_available() else "cpu"
    wl.setup(torch, zc, device, 0, 1)  # the seeded inputs are generated on the device
    budget = max(1.0, 90.0 / (steps + warmup))
    samples = []
    for step in range(warmup + steps):
        cb = wl.cpu_baseline(budget)
        if step >= warmup:
            samples.append(cb)
    value = sum(c["value"] for c in samples) / len(samples)
    last = samples[-1]
    line = {"metric": METRIC, "value": value, "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
            "steps": steps, "warmup": warmup, "ms_per_step": 1e3 * sum(c["seconds"] for c in samples) / len(samples),
            "higher_is_better": True, "scaling": wl.scaling, "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": dict(wl.config(1), note="reference CPU path, a bounded sample per step (see cpu_baseline)"),
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": last["cores"], "kind": last["kind"],
                             "sample": last["sample"]},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    emit(json.dumps(line))


def searcher_e2e(wl):
    """End-to-end rate through the C++ drop-in layer: the package's searcher_e2e program runs
    zcgvs::Searcher::search on a host query + copyResultToHost per query (graph replay once
    captured), on this workload's shape, in its own process on this GPU."""
    argv = wl.searcher_args()
    if argv is None:
        return None
    exe = PKG / "searcher_e2e"
    if not exe.exists():
        return {"unavailable": f"{exe.name} is not built (make -C {PKG.name})"}
    res = subprocess.run([str(exe)] + argv + ["steps=1000", "warmup=30"], capture_output=True, text=True,
                         timeout=600)
    if res.returncode != 0:
        return {"unavailable": (res.stderr.strip().splitlines() or ["exit status %d" % res.returncode])[-1]}
    out = json.loads(res.stdout.strip().splitlines()[-1])
    return {"value": out["queries_per_s"], "unit": UNIT, "h2d_bytes_per_step": out["h2d_bytes_per_step"],
            "d2h_bytes_per_step": out["d2h_bytes_per_step"], "ms_per_query": out["ms_per_query"],
            "search_gpu_ms_mean": out["search_gpu_ms_mean"], "steps": out["steps"], "graph": out["graph"],
            "api": "zcgvs::Searcher::search (host query) + copyResultToHost, C++ (" + exe.name + ")"}


def measure_sharded(args, torch, zc, device, rank, world):
    """Row-sharded config 4 (fp16 50M x 768, batch 4,096, top-100) through the native sharded
    handle, in the processes of the replica run: rank r holds rows shard_bounds(N, P, r), a step
    is its tensor-core search with global ids, an NCCL all-gather of every rank's [4096, 100]
    result and the device merge, replayed as one CUDA graph. Strong scaling (the corpus is fixed;
    each rank scans N / P rows). Timed with CUDA events over the steps, max over ranks; a second,
    direct pass with the library's kernel timing on splits the step into the local search, the
    all-gather and the merge."""
    import torch.distributed as dist

    wl = Cfg4(native=True)
    if args.sharded_docs:
        wl.N = args.sharded_docs
    wl.setup(torch, zc, device, rank, world)
    stream = torch.cuda.current_stream()
    steps, warmup = 5, 3
    for i in range(warmup):  # the first step runs directly and captures the graph the rest replay
        wl.step(i, stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(device.index) as clocks:
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for i in range(steps):
            wl.step(i, stream)
        t1.record(stream)
        torch.cuda.synchronize()
    elapsed_ms = t0.elapsed_time(t1)
    tags = ("gemm_sample", "gemm_threshold", "gemm_filter", "gemm_bucket", "gemm_select", "gemm_retry", "allgather",
            "merge")
    zc.kernel_timing(True)
    for i in range(steps):
        wl.step_direct(i, stream)
    torch.cuda.synchronize()
    zc.kernel_timing(False)
    kern = {t: zc.kernel_timing_read(t)[0] / steps for t in tags}
    word, comm_error = wl.search.status()
    local_ms = sum(v for t, v in kern.items() if t.startswith("gemm_"))
    vals = [elapsed_ms, local_ms, kern["allgather"], kern["merge"], kern["gemm_filter"], float(word | comm_error)]
    if world > 1:
        t = torch.tensor(vals, device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        vals = [float(v) for v in t.tolist()]
    elapsed_ms, local_ms, gather_ms, merge_ms, filter_ms, bad = vals
    rows = wl.end - wl.begin
    result = {
        "workload": wl.name, "docs": wl.N, "rows_per_rank": rows, "dim": wl.D, "k": wl.K, "batch": wl.B,
        "parallelism": f"rowshard{world}", "scaling": "strong", "launch": "one cuda graph per step",
        "value": wl.B * steps / (elapsed_ms * 1e-3), "unit": UNIT, "steps": steps, "warmup": warmup,
        "ms_per_step": elapsed_ms / steps,
        "local_search_ms_per_step": local_ms, "filter_ms_per_step": filter_ms,
        "allgather_ms_per_step": gather_ms, "merge_ms_per_step": merge_ms,
        # the share of a step spent in the rank's own search: strong-scaling efficiency when the
        # local search time is proportional to the rows (the driver's 1 -> N record has the rest)
        "local_fraction": local_ms / (elapsed_ms / steps),
        "filter_tflops": 2.0 * wl.B * rows * wl.D / (filter_ms * 1e-3) / 1e12 if filter_ms > 0 else None,
        "gpu_launches": wl.launches * steps,
        "clocks": clocks.summary(),
        "device_status": int(bad),
        "l2": "inputs larger than L2 (77 GB corpus)",
    }
    wl.search.close()
    return result


def run_ours(args):
    import torch
    import torch.distributed as dist

    import zcgvs_sm100 as zc

    rank, local_rank, world = dist_env()
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", init_method="env://", device_id=device, timeout=timedelta(seconds=300))

    wl = make_workload(args)
    steps = args.steps if args.steps is not None else wl.steps
    warmup = args.warmup if args.warmup is not None else wl.warmup
    wl.setup(torch, zc, device, rank, world)
    wl.capture(torch)
    stream = torch.cuda.current_stream()

    for i in range(warmup):
        wl.step(i, stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()

    events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    with ClockSampler(local_rank) as clocks:
        t_start = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        t_start.record(stream)
        for i in range(steps):
            events[i][0].record(stream)
            wl.step(i, stream)
            events[i][1].record(stream)
        t_end.record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    elapsed_ms = t_start.elapsed_time(t_end)
    per_step = sorted(a.elapsed_time(b) for a, b in events)

    # The same steps again with the library's per-launch CUDA events on (kept out of the timed
    # pass above): the duration of the dominant kernel(s) for the roofline.
    tags = ("scan", "gemm_sample", "gemm_threshold", "gemm_filter", "gemm_bucket", "gemm_select", "gemm_retry",
            "rescore", "lexical", "hybrid_select", "merge")
    zc.kernel_timing(True)
    for i in range(steps):
        wl.step_direct(i, stream)
    torch.cuda.synchronize()
    zc.kernel_timing(False)
    kern = {t: zc.kernel_timing_read(t) for t in tags}
    kernel_ms = wl.kernel_ms(kern, steps)
    if world > 1:
        t = torch.tensor([elapsed_ms, kernel_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed_ms, kernel_ms = float(t[0].item()), float(t[1].item())
    status = wl.ws.status()

    # End to end through the public API with host buffers: pinned host inputs -> device, the
    # search, results -> pinned host, synchronised every step (what a caller sees).
    e2e_steps = max(3, steps // 2)
    for i in range(2):
        wl.e2e_step(i, stream)
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    h2d = d2h = 0
    for i in range(e2e_steps):
        h2d, d2h = wl.e2e_step(i, stream)
    e2e_s = time.perf_counter() - t0
    if world > 1:
        t = torch.tensor([e2e_s], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = wl.cpu_baseline(12.0)
    peaks, peak_kind = measured_peaks()
    e2e_path = ("graph per query: pinned query copied in, result written by the search's last kernel into "
                "pinned host memory" if getattr(wl, "g_e2e_full", None) else "copies and search one after another")
    summary = {"scaling": wl.scaling, "units": wl.units, "dtype": wl.dtype, "config": wl.config(world),
               "graphs": wl.graphs, "roofline": wl.roofline(kernel_ms, peaks, peak_kind),
               "launches": wl.launches}
    e2e_ranks = [e2e_s]
    if world > 1:
        # every rank's end-to-end seconds: shows whether one rank held back the max
        t = torch.zeros(world, device=device)
        t[rank] = e2e_s
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        e2e_ranks = [round(float(v), 4) for v in t.tolist()]
    line_extra = {}
    if rank == 0 and world == 1 and not args.no_searcher:
        line_extra["e2e_searcher"] = searcher_e2e(wl)
    if wl.scaling == "weak" and not args.no_sharded:
        # The replica workloads have no exchange on their data path; the row-sharded search does.
        # Measure it in the same processes (config 4: the corpus split over the ranks).
        wl = None
        torch.cuda.empty_cache()
        line_extra["sharded"] = measure_sharded(args, torch, zc, device, rank, world)

    if rank == 0:
        peaks, peak_kind = measured_peaks()
        total_units = (1 if summary["scaling"] == "strong" else world) * summary["units"]
        line = {
            "metric": METRIC, "value": total_units * steps / (elapsed_ms * 1e-3), "unit": UNIT,
            "n_gpus": world, "steps": steps, "warmup": warmup,
            "ms_per_step": elapsed_ms / steps, "p50_ms": per_step[len(per_step) // 2],
            "higher_is_better": True, "scaling": summary["scaling"], "vs_baseline": None, "dtype": summary["dtype"],
            "data": "synthetic",
            "config": dict(summary["config"], launch="cuda-graph replay per query" if summary["graphs"] else "direct calls"),
            "roofline": dict(summary["roofline"], kernel_ms=kernel_ms),
            "kernels_ms_per_step": {t: v[0] / steps for t, v in kern.items() if v[1]},
            "e2e": {"value": total_units * e2e_steps / e2e_s, "unit": UNIT,
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "path": e2e_path},
            "gpu_launches": summary["launches"] * steps,
            "clocks": clocks.summary(),
            "device_status": status,
            "e2e_seconds_per_rank": e2e_ranks,
            "cpu_baseline": cpu,
        }
        line.update(line_extra)
        emit(json.dumps(line))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


_RESULT_FD = None


def emit(text: str) -> None:
    """Writes the run's one result line to the real standard output."""
    sys.stdout.flush()
    os.write(_RESULT_FD if _RESULT_FD is not None else 1, (text + "\n").encode())


class StdoutToStderr:
    """Sends everything else written to file descriptor 1 (Python prints and the libraries' own,
    such as NCCL's version banner on rank 0) to stderr, so that standard output carries only the
    result line that emit() writes."""

    def __enter__(self):
        global _RESULT_FD
        sys.stdout.flush()
        _RESULT_FD = os.dup(1)
        os.dup2(2, 1)
        return self

    def __exit__(self, *exc):
        global _RESULT_FD
        sys.stdout.flush()
        os.dup2(_RESULT_FD, 1)
        os.close(_RESULT_FD)
        _RESULT_FD = None


def main():
    args = parse_args()
    with StdoutToStderr():
        if args.impl == "reference":
            run_reference(args)
        else:
            run_ours(args)


if __name__ == "__main__":
    main()
