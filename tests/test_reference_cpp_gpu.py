"""GPU tier: the reference's own C++ test programs (tests/cpp/test_*.cu of the reference),
compiled unchanged against this library's C++ interface (include/zcgvs/) by `make -C oracle
reftests`, run on the device. Each program checks the GPU path against the reference's CPU code
and exits 0 on success; together they are the reference's regression suite run through the
drop-in boundary (similarity sweep, masks / L2, int8, batched and large top-k, BM25 / fuse, the
Searcher pipeline with rescoring and CUDA-graph replay)."""

from __future__ import annotations

import subprocess

import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu

BIN = ROOT / "oracle" / "_ref" / "cpp"
PROGRAMS = sorted(p.name for p in BIN.glob("test_*")) if BIN.is_dir() else []


@pytest.mark.parametrize("program", PROGRAMS or ["(not built)"])
def test_reference_program(zc, program):
    if not PROGRAMS:
        pytest.skip("oracle/_ref/cpp was not built (needs the reference tree at build time)")
    result = subprocess.run([str(BIN / program)], capture_output=True, text=True, timeout=600)
    assert result.returncode == 0, f"{program} failed:\n{result.stdout[-3000:]}\n{result.stderr[-3000:]}"


def test_reference_kernel_benchmark_runs(zc):
    """The reference's kernel benchmark (apps/bench_kernels.cu), compiled unchanged against the
    same headers plus the device-context header and the cuBLAS yardstick, runs end to end at its
    smallest settings: storage scans of every dtype, the cuBLAS GEMV, top-k widths and the
    Searcher with and without graphs."""
    exe = BIN / "bench_kernels"
    if not exe.exists():
        pytest.skip("oracle/_ref/cpp/bench_kernels was not built (needs the reference tree at build time)")
    result = subprocess.run([str(exe), "--docs", "20000", "--dim", "128", "--k", "10", "--warmup", "1",
                             "--iterations", "2"], capture_output=True, text=True, timeout=600)
    assert result.returncode == 0, f"bench_kernels failed:\n{result.stdout[-3000:]}\n{result.stderr[-3000:]}"
    out = result.stdout
    assert "NVIDIA B200" in out or "sm_10" in out, out[:500]
    for label in ("similarity scan", "cublas sgemv", "top-k selection", "pipeline (graph)"):
        assert label in out, f"{label!r} missing from:\n{out}"
