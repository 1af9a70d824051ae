"""ctypes binding of libzcgvs_sm100.so, the C ABI declared in include/zcgvs_sm100.h.

This is the host-side mirror of the reference's launcher surface for Python callers (tests,
bench.py, services): device buffers are torch CUDA tensors used as plain memory, and every
call goes straight to the CUDA library. There is no CPU fallback: importing this module on a
machine without the built library raises, and a call without a GPU fails with the CUDA error.
"""

from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libzcgvs_sm100.so"
HEADER_PATH = HERE.parent / "include" / "zcgvs_sm100.h"

OK, ERR_INVALID_ARG, ERR_CUDA, ERR_UNSUPPORTED, ERR_DEVICE_STATUS, ERR_COMM = 0, 1, 2, 3, 4, 5
SHARDED_GRAPH, SHARDED_F16_TENSOR = 1, 2
# Bits of the device status word (the first 4 bytes of a workspace; ZCGVS_DEVICE_* in the header).
DEVICE_TILE_WAIT_TIMEOUT, DEVICE_DRAIN_TIMEOUT, DEVICE_TMEM_WAIT_TIMEOUT, DEVICE_CANDIDATE_OVERFLOW = 1, 2, 4, 8
_DEVICE_STATUS_TEXT = {
    DEVICE_TILE_WAIT_TIMEOUT: "a bounded wait for a corpus tile ran out",
    DEVICE_DRAIN_TIMEOUT: "a bounded wait for in-flight copies ran out",
    DEVICE_TMEM_WAIT_TIMEOUT: "a tensor-memory accumulator hand-off ran out",
    DEVICE_CANDIDATE_OVERFLOW: "a query kept more candidates than its buffer holds (its top-k is incomplete)",
}
DTYPE_F32, DTYPE_F16, DTYPE_I8, DTYPE_BINARY, DTYPE_I8_ROW = 0, 1, 2, 3, 4
METRIC_COSINE, METRIC_DOT, METRIC_L2 = 0, 1, 2
MAX_K = 1024

_P = ctypes.c_void_p
_i32, _i64, _f32, _sz = ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t

# Every exported function: name -> (restype, argtypes). Kept in the order of the header.
SIGNATURES = {
    "zcgvs_version": (_i32, []),
    "zcgvs_last_error_message": (ctypes.c_char_p, []),
    "zcgvs_last_cuda_error": (_i32, []),
    "zcgvs_workspace_init": (_i32, [_P, _sz, _P]),
    "zcgvs_workspace_status": (_i32, [_P, _sz, _P, _P]),
    "zcgvs_test_set_candidate_cap": (_i32, [_i32]),
    "zcgvs_check_bounded_wait": (_i32, [_P, _sz, _P]),
    "zcgvs_kernel_timing": (_i32, [_i32]),
    "zcgvs_kernel_timing_read": (_i32, [ctypes.c_char_p, _P, _P]),
    "zcgvs_scan_topk_workspace_bytes": (_sz, [_i32, _i64, _i32, _i32, _i32]),
    "zcgvs_scan_topk": (_i32, [_P, _i32, _f32, _P, _i64, _i32, _P, _i32, _P, _i32, _i32, _i32,
                               _P, _P, _P, _sz, _P]),
    "zcgvs_scan_topk_noalloc": (_i32, [_P, _i32, _f32, _P, _i64, _i32, _P, _i32, _P, _i32, _i32,
                                       _i32, _P, _P, _P]),
    "zcgvs_scan_topk_noalloc_status": (_i32, [_P, _P]),
    "zcgvs_similarity": (_i32, [_P, _i32, _f32, _P, _i64, _i32, _P, _i32, _P, _i32, _P, _P]),
    "zcgvs_rescore_topk": (_i32, [_P, _i32, _f32, _P, _i64, _i32, _P, _i32, _P, _i32, _i32, _i32,
                                  _P, _P, _P]),
    "zcgvs_gather_rescore": (_i32, [_P, _i32, _f32, _P, _i64, _i32, _P, _i32, _P, _i32, _i32, _P,
                                    _P]),
    "zcgvs_gemm_topk_workspace_bytes": (_sz, [_i32, _i64, _i32, _i32, _i32]),
    "zcgvs_gemm_topk": (_i32, [_P, _i32, _P, _i64, _i32, _P, _i32, _P, _i32, _i32, _i32, _P, _P, _P, _sz, _P]),
    "zcgvs_gemm_similarity_workspace_bytes": (_sz, [_i32, _i64, _i32, _i32]),
    "zcgvs_gemm_similarity": (_i32, [_P, _i32, _P, _i64, _i32, _P, _i32, _P, _i32, _P, _P, _sz, _P]),
    "zcgvs_topk": (_i32, [_P, _i64, _i32, _i32, _P, _P, _P]),
    "zcgvs_convert_f16": (_i32, [_P, _P, _sz, _P]),
    "zcgvs_convert_i8": (_i32, [_P, _P, _sz, _f32, _P]),
    "zcgvs_convert_i8_rows": (_i32, [_P, _P, _P, _i64, _i32, _P]),
    "zcgvs_pack_binary": (_i32, [_P, _P, _i64, _i32, _P]),
    "zcgvs_remap_indices": (_i32, [_P, _P, _i32, _i32, _i32, _P, _P]),
    "zcgvs_merge_topk": (_i32, [_P, _P, _i32, _i32, _i32, _i32, _P, _P, _P]),
    "zcgvs_merge_topk_lists": (_i32, [_P, _P, _i64, _i32, _i32, _i32, _P, _i32, _P, _P, _i32, _i32, _P, _P]),
    "zcgvs_shard_bounds": (_i32, [_i64, _i32, _i32, _P, _P]),
    "zcgvs_nccl_id_bytes": (_sz, []),
    "zcgvs_nccl_unique_id": (_i32, [_P]),
    "zcgvs_sharded_create": (_i32, [_P, _i32, _i32, _i64, _P]),
    "zcgvs_sharded_destroy": (_i32, [_P]),
    "zcgvs_sharded_search": (_i32, [_P, _P, _i32, _f32, _P, _i64, _i32, _P, _i32, _P, _i32, _i32, ctypes.c_uint,
                                    _P, _P, _P]),
    "zcgvs_sharded_rescore_search": (_i32, [_P, _P, _i32, _f32, _P, _P, _i32, _f32, _P, _i64, _i32, _P, _i32, _i32,
                                            _i32, _i32, ctypes.c_uint, _P, _P, _P]),
    "zcgvs_sharded_status": (_i32, [_P, _P, _P, _P]),
    "zcgvs_sharded_clear_status": (_i32, [_P, _P]),
    "zcgvs_hybrid_topk_workspace_bytes": (_sz, [_i32, _i64, _i32, _i32, _i32]),
    "zcgvs_hybrid_topk": (_i32, [_P, _i32, _f32, _P, _i64, _i32, _P, _i32, _P, _i32, _P, _P, _P, _i32,
                                 _P, _i32, _f32, _i32, _P, _P, _P, _sz, _P]),
    "zcgvs_bm25": (_i32, [_P, _P, _P, _P, _i32, _i32, _P, _P]),
    "zcgvs_max_positive": (_i32, [_P, _i32, _P, _P]),
    "zcgvs_fuse_scores": (_i32, [_P, _P, _P, _f32, _i32, _P]),
}


class ZcgvsError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"[status {status}] {message}")
        self.status = status


class InvalidArgument(ZcgvsError, ValueError):
    pass


class DeviceStatusError(ZcgvsError):
    """A search finished with a non-zero device status word: its results may be incomplete."""

    def __init__(self, word: int):
        super().__init__(ERR_DEVICE_STATUS, describe_device_status(word))
        self.word = word


def describe_device_status(word: int) -> str:
    parts = [text for bit, text in _DEVICE_STATUS_TEXT.items() if word & bit]
    unknown = word & ~sum(_DEVICE_STATUS_TEXT)
    if unknown:
        parts.append(f"unknown bits 0x{unknown:x}")
    return f"device status 0x{word:x}: " + "; ".join(parts)


_lib = None


def build() -> None:
    subprocess.run(["make", "-s", "-j8", "-C", str(HERE)], check=True)


def lib():
    """Loads the CUDA library; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is not built; run `make -C {HERE}` or __graft_entry__.build()")
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = handle
    return _lib


def check(status: int) -> None:
    if status == OK:
        return
    message = lib().zcgvs_last_error_message().decode("utf-8", "replace")
    if status == ERR_INVALID_ARG:
        raise InvalidArgument(status, message)
    raise ZcgvsError(status, message)


# ----------------------------------------------------------------------------------------
# torch helpers (torch is plumbing: device memory and streams only)
# ----------------------------------------------------------------------------------------
def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(stream):
    import torch

    s = torch.cuda.current_stream() if stream is None else stream
    return ctypes.c_void_p(s.cuda_stream)


class Workspace:
    """A zero-initialised device workspace that grows on demand (re-zeroed when it grows)."""

    def __init__(self, device=None):
        self.device = device
        self.buffer = None

    def get(self, nbytes: int, stream=None):
        import torch

        if self.buffer is None or self.buffer.numel() < nbytes:
            self.buffer = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=self.device or "cuda")
        return self.buffer

    def status(self, stream=None) -> int:
        """The device status word (synchronises `stream`); 0 when every call completed."""
        if self.buffer is None:
            return 0
        value = ctypes.c_uint32(0)
        check(lib().zcgvs_workspace_status(_ptr(self.buffer), self.buffer.numel(), ctypes.byref(value),
                                           _stream(stream)))
        return int(value.value)

    def clear_status(self, stream=None) -> None:
        if self.buffer is not None:
            check(lib().zcgvs_workspace_init(_ptr(self.buffer), 4, _stream(stream)))

    def raise_on_status(self, stream=None) -> None:
        """Raises DeviceStatusError (after clearing the word) when a call left it non-zero."""
        word = self.status(stream)
        if word:
            self.clear_status(stream)
            raise DeviceStatusError(word)


def _own_workspace(workspace, device):
    """(workspace, owned): a helper that creates its own workspace also checks its status."""
    return (workspace, False) if workspace is not None else (Workspace(device), True)


def set_test_candidate_cap(cap: int) -> None:
    """Test hook: caps the tensor-core path's per-query candidate buffer (0 restores 16384)."""
    check(lib().zcgvs_test_set_candidate_cap(int(cap)))


def check_bounded_wait(workspace: Workspace, stream=None) -> None:
    """Runs the diagnostic whose bounded wait runs out (2 s), setting the timeout bit in the
    workspace's status word."""
    buf = workspace.get(256, stream)
    check(lib().zcgvs_check_bounded_wait(_ptr(buf), buf.numel(), _stream(stream)))


def noalloc_status(stream=None) -> int:
    """Status word of the last zcgvs_scan_topk_noalloc call on the current device."""
    value = ctypes.c_uint32(0)
    check(lib().zcgvs_scan_topk_noalloc_status(ctypes.byref(value), _stream(stream)))
    return int(value.value)


def kernel_timing(enable: bool) -> None:
    """Starts (clearing earlier records) or stops CUDA-event timing of the library's kernels."""
    check(lib().zcgvs_kernel_timing(1 if enable else 0))


def kernel_timing_read(tag: str) -> tuple[float, int]:
    """(summed milliseconds, launches) of the recorded launches tagged `tag`."""
    total = ctypes.c_double(0.0)
    count = ctypes.c_int(0)
    check(lib().zcgvs_kernel_timing_read(tag.encode(), ctypes.byref(total), ctypes.byref(count)))
    return float(total.value), int(count.value)


def scan_topk_workspace_bytes(dtype: int, doc_count: int, dim: int, batch: int, k: int) -> int:
    return int(lib().zcgvs_scan_topk_workspace_bytes(dtype, doc_count, dim, batch, k))


def scan_topk(corpus, dtype: int, dim: int, queries, k: int, *, scale: float = 1.0,
              row_scales=None, mask=None, metric: int = METRIC_DOT, id_base: int = 0,
              workspace: Workspace | None = None, out=None, stream=None):
    """Fused scan + top-k on device tensors. Returns (indices int32 [B,k], scores fp32 [B,k])."""
    import torch

    doc_count = corpus.shape[0]
    queries = queries.reshape(-1, dim)
    batch = queries.shape[0]
    if out is None:
        out = (torch.empty((batch, k), dtype=torch.int32, device=queries.device),
               torch.empty((batch, k), dtype=torch.float32, device=queries.device))
    ws, owned = _own_workspace(workspace, queries.device)
    nbytes = scan_topk_workspace_bytes(dtype, doc_count, dim, batch, k)
    buf = ws.get(nbytes, stream)
    check(lib().zcgvs_scan_topk(_ptr(corpus), dtype, scale, _ptr(row_scales), doc_count, dim,
                                _ptr(queries), batch, _ptr(mask), metric, k, id_base,
                                _ptr(out[0]), _ptr(out[1]), _ptr(buf), buf.numel(), _stream(stream)))
    if owned:
        ws.raise_on_status(stream)
    return out


def scan_topk_noalloc(corpus, dtype: int, dim: int, queries, k: int, *, scale: float = 1.0,
                      row_scales=None, mask=None, metric: int = METRIC_DOT, id_base: int = 0,
                      out=None, stream=None, check_status: bool = True):
    """zcgvs_scan_topk_noalloc: the fused search with the library's static scratch (no
    workspace). Returns (indices int32 [B,k], scores fp32 [B,k]); with check_status (the
    default) it reads the call's device status word and raises DeviceStatusError if non-zero."""
    import torch

    doc_count = corpus.shape[0]
    queries = queries.reshape(-1, dim)
    batch = queries.shape[0]
    if out is None:
        out = (torch.empty((batch, k), dtype=torch.int32, device=queries.device),
               torch.empty((batch, k), dtype=torch.float32, device=queries.device))
    check(lib().zcgvs_scan_topk_noalloc(_ptr(corpus), dtype, scale, _ptr(row_scales), doc_count, dim,
                                        _ptr(queries), batch, _ptr(mask), metric, k, id_base,
                                        _ptr(out[0]), _ptr(out[1]), _stream(stream)))
    if check_status:
        word = noalloc_status(stream)
        if word:
            raise DeviceStatusError(word)
    return out


def similarity(corpus, dtype: int, dim: int, queries, *, scale: float = 1.0, row_scales=None,
               mask=None, metric: int = METRIC_DOT, out=None, stream=None):
    """Score matrix [B, N] (the reference launchSimilarity contract)."""
    import torch

    doc_count = corpus.shape[0]
    batch = queries.shape[0]
    if out is None:
        out = torch.empty((batch, doc_count), dtype=torch.float32, device=queries.device)
    check(lib().zcgvs_similarity(_ptr(corpus), dtype, scale, _ptr(row_scales), doc_count, dim,
                                 _ptr(queries), batch, _ptr(mask), metric, _ptr(out), _stream(stream)))
    return out


def rescore_topk(store, dtype: int, dim: int, queries, candidates, k: int, *, scale: float = 1.0,
                 row_scales=None, metric: int = METRIC_DOT, out=None, stream=None):
    """Fused gather + exact rescore + top-k over candidate ids [B, M]. Returns (ids, scores)."""
    import torch

    queries = queries.reshape(-1, dim)
    batch = queries.shape[0]
    candidates = candidates.reshape(batch, -1)
    if out is None:
        out = (torch.empty((batch, k), dtype=torch.int32, device=queries.device),
               torch.empty((batch, k), dtype=torch.float32, device=queries.device))
    check(lib().zcgvs_rescore_topk(_ptr(store), dtype, scale, _ptr(row_scales), store.shape[0], dim,
                                   _ptr(queries), batch, _ptr(candidates), candidates.shape[1], metric,
                                   k, _ptr(out[0]), _ptr(out[1]), _stream(stream)))
    return out


def gather_rescore(store, dtype: int, dim: int, queries, candidates, *, scale: float = 1.0,
                   row_scales=None, metric: int = METRIC_DOT, out=None, stream=None):
    """Exact scores [B, M] of candidate ids [B, M] (the reference launchGatherRescore)."""
    import torch

    queries = queries.reshape(-1, dim)
    batch = queries.shape[0]
    candidates = candidates.reshape(batch, -1)
    if out is None:
        out = torch.empty(candidates.shape, dtype=torch.float32, device=queries.device)
    check(lib().zcgvs_gather_rescore(_ptr(store), dtype, scale, _ptr(row_scales), store.shape[0], dim,
                                     _ptr(queries), batch, _ptr(candidates), candidates.shape[1],
                                     metric, _ptr(out), _stream(stream)))
    return out


class LexicalIndex:
    """Device copy of a CSR BM25 index (offsets int64, docs int32, weights fp32; torch tensors).
    Posting lists must be sorted by document within each term (lexical_index.sort_postings)."""

    def __init__(self, offsets, docs, weights, device=None):
        import torch

        self.offsets = torch.as_tensor(offsets, dtype=torch.int64, device=device or "cuda")
        self.docs = torch.as_tensor(docs, dtype=torch.int32, device=device or "cuda")
        self.weights = torch.as_tensor(weights, dtype=torch.float32, device=device or "cuda")
        self.vocab = self.offsets.numel() - 1


def hybrid_topk(corpus, dtype: int, dim: int, queries, k: int, index: LexicalIndex, terms,
                dense_weight: float, *, scale: float = 1.0, row_scales=None, mask=None,
                metric: int = METRIC_DOT, workspace: Workspace | None = None, out=None, stream=None):
    """Hybrid BM25 + dense top-k. terms: int32 device tensor [B, stride] (-1 padded)."""
    import torch

    doc_count = corpus.shape[0]
    queries = queries.reshape(-1, dim)
    batch = queries.shape[0]
    if terms.dim() != 2:
        terms = terms.reshape(batch, -1)
    if out is None:
        out = (torch.empty((batch, k), dtype=torch.int32, device=queries.device),
               torch.empty((batch, k), dtype=torch.float32, device=queries.device))
    ws, owned = _own_workspace(workspace, queries.device)
    nbytes = int(lib().zcgvs_hybrid_topk_workspace_bytes(dtype, doc_count, dim, batch, k))
    buf = ws.get(nbytes, stream)
    check(lib().zcgvs_hybrid_topk(_ptr(corpus), dtype, scale, _ptr(row_scales), doc_count, dim, _ptr(queries),
                                  batch, _ptr(mask), metric, _ptr(index.offsets), _ptr(index.docs),
                                  _ptr(index.weights), index.vocab, _ptr(terms), terms.shape[1], dense_weight, k,
                                  _ptr(out[0]), _ptr(out[1]), _ptr(buf), buf.numel(), _stream(stream)))
    if owned:
        ws.raise_on_status(stream)
    return out


def bm25(index: LexicalIndex, terms, scores, stream=None):
    """scores[d] += BM25 weights of one query's terms (the reference launchBm25)."""
    check(lib().zcgvs_bm25(_ptr(index.offsets), _ptr(index.docs), _ptr(index.weights), _ptr(terms),
                           terms.numel(), scores.numel(), _ptr(scores), _stream(stream)))
    return scores


def max_positive(values, out_max, stream=None):
    check(lib().zcgvs_max_positive(_ptr(values), values.numel(), _ptr(out_max), _stream(stream)))
    return out_max


def fuse_scores(dense, lexical, lexical_max, weight: float, stream=None):
    check(lib().zcgvs_fuse_scores(_ptr(dense), _ptr(lexical), _ptr(lexical_max), weight, dense.numel(),
                                  _stream(stream)))
    return dense


def merge_topk(list_indices, list_scores, k: int, out=None, stream=None):
    """Global top-k of per-shard lists [P, B, k_in] (int32 ids, fp32 scores) -> ([B, k], [B, k])."""
    import torch

    lists, batch, k_in = list_indices.shape
    if out is None:
        out = (torch.empty((batch, k), dtype=torch.int32, device=list_indices.device),
               torch.empty((batch, k), dtype=torch.float32, device=list_indices.device))
    check(lib().zcgvs_merge_topk(_ptr(list_indices), _ptr(list_scores), lists, batch, k_in, k, _ptr(out[0]),
                                 _ptr(out[1]), _stream(stream)))
    return out


def merge_topk_lists(list_indices, list_scores, list_stride: int, lists: int, batch: int, k_in: int, k: int, *,
                     list_id_offsets=None, out=None, own_range=None, out_owned=None, stream=None):
    """zcgvs_merge_topk_lists over flat device tensors (see the header for the layout)."""
    check(lib().zcgvs_merge_topk_lists(_ptr(list_indices), _ptr(list_scores), list_stride, lists, batch, k_in,
                                       _ptr(list_id_offsets), k, _ptr(out[0]) if out else None,
                                       _ptr(out[1]) if out else None, own_range[0] if own_range else 0,
                                       own_range[1] if own_range else 0, _ptr(out_owned), _stream(stream)))
    return out, out_owned


def shard_bounds(total_rows: int, world: int, rank: int) -> tuple[int, int]:
    begin, end = ctypes.c_int64(0), ctypes.c_int64(0)
    check(lib().zcgvs_shard_bounds(total_rows, world, rank, ctypes.byref(begin), ctypes.byref(end)))
    return int(begin.value), int(end.value)


class ShardedSearcher:
    """Rank `rank`'s handle of a row-sharded search over `world` GPUs (zcgvs_sharded_*): the
    local fused search, NCCL all-gathers and device merges, the whole step replayed as one CUDA
    graph after the first search of a shape. Every rank must make the same calls in order."""

    def __init__(self, nccl_id: bytes, world: int, rank: int, total_rows: int):
        handle = ctypes.c_void_p()
        buf = ctypes.create_string_buffer(bytes(nccl_id), len(nccl_id))
        check(lib().zcgvs_sharded_create(buf, world, rank, total_rows, ctypes.byref(handle)))
        self.handle = handle
        self.world, self.rank, self.total_rows = world, rank, total_rows
        self.begin, self.end = shard_bounds(total_rows, world, rank)

    @staticmethod
    def unique_id() -> bytes:
        n = int(lib().zcgvs_nccl_id_bytes())
        buf = ctypes.create_string_buffer(n)
        check(lib().zcgvs_nccl_unique_id(buf))
        return buf.raw

    def _out(self, batch, k, device, out):
        import torch

        if out is None:
            out = (torch.empty((batch, k), dtype=torch.int32, device=device),
                   torch.empty((batch, k), dtype=torch.float32, device=device))
        return out

    def search(self, shard, dtype: int, dim: int, queries, k: int, *, scale: float = 1.0, row_scales=None,
               mask=None, metric: int = METRIC_DOT, tensor_f16: bool = False, graph: bool = True, out=None,
               stream=None):
        queries = queries.reshape(-1, dim)
        out = self._out(queries.shape[0], k, queries.device, out)
        flags = (SHARDED_GRAPH if graph else 0) | (SHARDED_F16_TENSOR if tensor_f16 else 0)
        check(lib().zcgvs_sharded_search(self.handle, _ptr(shard), dtype, scale, _ptr(row_scales), shard.shape[0], dim,
                                         _ptr(queries), queries.shape[0], _ptr(mask), metric, k, flags, _ptr(out[0]),
                                         _ptr(out[1]), _stream(stream)))
        return out

    def rescore_search(self, codes, code_dtype: int, store, store_dtype: int, dim: int, queries, candidates: int,
                       k: int, *, code_scale: float = 1.0, code_row_scales=None, store_scale: float = 1.0,
                       store_row_scales=None, metric: int = METRIC_DOT, graph: bool = True, out=None, stream=None):
        queries = queries.reshape(-1, dim)
        out = self._out(queries.shape[0], k, queries.device, out)
        check(lib().zcgvs_sharded_rescore_search(self.handle, _ptr(codes), code_dtype, code_scale,
                                                 _ptr(code_row_scales), _ptr(store), store_dtype, store_scale,
                                                 _ptr(store_row_scales), codes.shape[0], dim, _ptr(queries),
                                                 queries.shape[0], metric, candidates, k,
                                                 SHARDED_GRAPH if graph else 0, _ptr(out[0]), _ptr(out[1]),
                                                 _stream(stream)))
        return out

    def status(self, stream=None) -> tuple[int, int]:
        """(device status word, NCCL asynchronous error) after synchronising `stream`."""
        word, comm = ctypes.c_uint32(0), ctypes.c_int(0)
        check(lib().zcgvs_sharded_status(self.handle, ctypes.byref(word), ctypes.byref(comm), _stream(stream)))
        return int(word.value), int(comm.value)

    def clear_status(self, stream=None) -> None:
        check(lib().zcgvs_sharded_clear_status(self.handle, _stream(stream)))

    def close(self) -> None:
        if self.handle:
            check(lib().zcgvs_sharded_destroy(self.handle))
            self.handle = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass


def gemm_topk(corpus, dtype: int, dim: int, queries, k: int, *, row_scales=None, mask=None,
              metric: int = METRIC_DOT, id_base: int = 0, workspace: Workspace | None = None, out=None,
              stream=None):
    """Tensor-core batched top-k (F16, I8_ROW or BINARY corpora). Returns (ids [B, k], scores [B, k])."""
    import torch

    doc_count = corpus.shape[0]
    queries = queries.reshape(-1, dim)
    batch = queries.shape[0]
    if out is None:
        out = (torch.empty((batch, k), dtype=torch.int32, device=queries.device),
               torch.empty((batch, k), dtype=torch.float32, device=queries.device))
    ws, owned = _own_workspace(workspace, queries.device)
    nbytes = int(lib().zcgvs_gemm_topk_workspace_bytes(dtype, doc_count, dim, batch, k))
    buf = ws.get(nbytes, stream)
    check(lib().zcgvs_gemm_topk(_ptr(corpus), dtype, _ptr(row_scales), doc_count, dim, _ptr(queries), batch,
                                _ptr(mask), metric, k, id_base, _ptr(out[0]), _ptr(out[1]), _ptr(buf), buf.numel(),
                                _stream(stream)))
    if owned:
        ws.raise_on_status(stream)
    return out


def gemm_similarity(corpus, dtype: int, dim: int, queries, *, row_scales=None, mask=None, metric: int = METRIC_DOT,
                    workspace: Workspace | None = None, out=None, stream=None):
    """Tensor-core score matrix [B, N]."""
    import torch

    doc_count = corpus.shape[0]
    queries = queries.reshape(-1, dim)
    batch = queries.shape[0]
    if out is None:
        out = torch.empty((batch, doc_count), dtype=torch.float32, device=queries.device)
    ws, owned = _own_workspace(workspace, queries.device)
    nbytes = int(lib().zcgvs_gemm_similarity_workspace_bytes(dtype, doc_count, dim, batch))
    buf = ws.get(nbytes, stream)
    check(lib().zcgvs_gemm_similarity(_ptr(corpus), dtype, _ptr(row_scales), doc_count, dim, _ptr(queries), batch,
                                      _ptr(mask), metric, _ptr(out), _ptr(buf), buf.numel(), _stream(stream)))
    if owned:
        ws.raise_on_status(stream)
    return out


def topk(scores, k: int, out=None, stream=None):
    """Top-k of every row of a [B, N] fp32 score matrix (the reference launchTopK)."""
    import torch

    batch, n = scores.shape
    if out is None:
        out = (torch.empty((batch, k), dtype=torch.int32, device=scores.device),
               torch.empty((batch, k), dtype=torch.float32, device=scores.device))
    check(lib().zcgvs_topk(_ptr(scores), n, k, batch, _ptr(out[0]), _ptr(out[1]), _stream(stream)))
    return out


# ------------------------------------------------------------------------------------------
# Store converters: fp32 rows on the device -> the stored precisions.
# ------------------------------------------------------------------------------------------
def convert_f16(src, out=None, stream=None):
    """fp32 -> fp16 bits (round to nearest even), any shape. Returns int16 bits of src's shape."""
    import torch

    out = torch.empty(src.shape, dtype=torch.int16, device=src.device) if out is None else out
    check(lib().zcgvs_convert_f16(_ptr(src), _ptr(out), src.numel(), _stream(stream)))
    return out


def convert_i8(src, scale: float, out=None, stream=None):
    """Per-matrix int8: clamp(rint(x * (1 / scale)), +-127), any shape."""
    import torch

    out = torch.empty(src.shape, dtype=torch.int8, device=src.device) if out is None else out
    check(lib().zcgvs_convert_i8(_ptr(src), _ptr(out), src.numel(), scale, _stream(stream)))
    return out


def convert_i8_rows(src, out=None, stream=None):
    """Per-row int8 of fp32 rows [rows, dim] -> (int8 [rows, dim], fp32 scales [rows]), the
    DTYPE_I8_ROW store layout."""
    import torch

    rows, dim = src.shape
    if out is None:
        out = (torch.empty((rows, dim), dtype=torch.int8, device=src.device),
               torch.empty((rows,), dtype=torch.float32, device=src.device))
    check(lib().zcgvs_convert_i8_rows(_ptr(src), _ptr(out[0]), _ptr(out[1]), rows, dim, _stream(stream)))
    return out


def pack_binary(src, out=None, stream=None):
    """Sign bits of fp32 rows [rows, dim] -> int32 words [rows, ceil(dim / 32)] (bit b of word w
    is dimension 32 w + b, set when x >= 0)."""
    import torch

    rows, dim = src.shape
    if out is None:
        out = torch.empty((rows, (dim + 31) // 32), dtype=torch.int32, device=src.device)
    check(lib().zcgvs_pack_binary(_ptr(src), _ptr(out), rows, dim, _stream(stream)))
    return out
