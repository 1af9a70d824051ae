"""CPU tier: the C-ABI library loads, exports every symbol include/*.h declares, and rejects
invalid arguments before touching a device (mirroring the reference's std::invalid_argument
cases, src/cuda/topk.cu:146-153 and src/search/searcher.cpp:91-135)."""

from __future__ import annotations

import ctypes
import re

import pytest

from conftest import ROOT


def declared_functions():
    names = set()
    for header in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
        names.update(re.findall(r"\b(zcgvs_[a-z0-9_]+)\s*\(", text))
    return sorted(names)


def test_header_declares_entry_points():
    names = declared_functions()
    assert "zcgvs_scan_topk" in names and "zcgvs_similarity" in names


def test_library_exports_every_declared_symbol(zc):
    lib = zc.lib()
    for name in declared_functions():
        assert hasattr(lib, name), f"{name} declared in include/ but not exported"
        assert name in zc.SIGNATURES, f"{name} has no ctypes signature"


def test_version(zc):
    assert zc.lib().zcgvs_version() >= 100


@pytest.mark.parametrize("k,n,expect", [(0, 100, "k must be positive"), (1025, 5000, "exceeds kernel capacity"),
                                        (101, 100, "exceeds corpus size")])
def test_scan_topk_rejects_bad_k(zc, k, n, expect):
    fake = ctypes.c_void_p(16)
    status = zc.lib().zcgvs_scan_topk(fake, zc.DTYPE_F32, 1.0, None, n, 8, fake, 1, None, zc.METRIC_DOT, k, 0,
                                      fake, fake, fake, 1 << 20, None)
    assert status == zc.ERR_INVALID_ARG
    assert expect in zc.lib().zcgvs_last_error_message().decode()


def test_zero_sized_problem_is_a_noop(zc):
    assert zc.lib().zcgvs_scan_topk(None, zc.DTYPE_F32, 1.0, None, 0, 8, None, 1, None, 0, 10, 0,
                                    None, None, None, 0, None) == zc.OK
    assert zc.lib().zcgvs_similarity(None, zc.DTYPE_F32, 1.0, None, 10, 8, None, 0, None, 0, None, None) == zc.OK


def test_per_row_int8_needs_scales(zc):
    fake = ctypes.c_void_p(16)
    status = zc.lib().zcgvs_scan_topk(fake, zc.DTYPE_I8_ROW, 1.0, None, 100, 8, fake, 1, None, zc.METRIC_DOT, 10, 0,
                                      fake, fake, fake, 1 << 20, None)
    assert status == zc.ERR_INVALID_ARG


@pytest.mark.parametrize("dtype,m,k,expect", [
    (3, 100, 10, "float32, float16 or int8"),       # binary rescore store (src/cuda/rescore.cu:102-105)
    (0, 100, 0, "k must be in"),
    (0, 100, 1025, "k must be in"),
    (0, 10, 11, "k exceeds candidate_count"),
    (0, 8193, 10, "candidate_count exceeds"),
])
def test_rescore_rejects_bad_arguments(zc, dtype, m, k, expect):
    fake = ctypes.c_void_p(16)
    status = zc.lib().zcgvs_rescore_topk(fake, dtype, 1.0, None, 1000, 8, fake, 1, fake, m, zc.METRIC_DOT, k,
                                         fake, fake, None)
    assert status == zc.ERR_INVALID_ARG
    assert expect in zc.lib().zcgvs_last_error_message().decode()


def test_rescore_zero_sized_is_a_noop(zc):
    assert zc.lib().zcgvs_rescore_topk(None, 0, 1.0, None, 10, 8, None, 1, None, 0, 0, 5, None, None, None) == zc.OK
    assert zc.lib().zcgvs_gather_rescore(None, 0, 1.0, None, 10, 8, None, 0, None, 4, 0, None, None) == zc.OK


def test_converters_check_arguments_before_touching_the_device(zc):
    """Zero-sized conversions are no-ops; null pointers are INVALID_ARG (no device call either
    way, so this runs without a GPU)."""
    lib = zc.lib()
    assert lib.zcgvs_convert_i8_rows(None, None, None, 0, 8, None) == zc.OK
    assert lib.zcgvs_convert_i8_rows(None, None, None, 4, 0, None) == zc.OK
    assert lib.zcgvs_convert_i8_rows(None, None, None, 4, 8, None) == zc.ERR_INVALID_ARG
    assert "zcgvs_convert_i8_rows" in lib.zcgvs_last_error_message().decode()
    assert lib.zcgvs_convert_i8(None, None, 0, 1.0, None) == zc.OK
    assert lib.zcgvs_convert_i8(None, None, 16, 1.0, None) == zc.ERR_INVALID_ARG
    assert lib.zcgvs_pack_binary(None, None, 0, 8, None) == zc.OK
    assert lib.zcgvs_pack_binary(None, None, 3, 8, None) == zc.ERR_INVALID_ARG


def test_status_readers_and_test_hooks_check_arguments(zc):
    """The no-alloc status reader, the candidate-cap test hook and the bounded-wait diagnostic
    reject bad arguments before touching a device."""
    lib = zc.lib()
    assert lib.zcgvs_scan_topk_noalloc_status(None, None) == zc.ERR_INVALID_ARG
    assert "null status pointer" in lib.zcgvs_last_error_message().decode()
    for cap in (-1, 16385):
        assert lib.zcgvs_test_set_candidate_cap(cap) == zc.ERR_INVALID_ARG
    assert lib.zcgvs_test_set_candidate_cap(0) == zc.OK
    assert lib.zcgvs_check_bounded_wait(None, 256, None) == zc.ERR_INVALID_ARG
    assert lib.zcgvs_workspace_status(None, 0, None, None) == zc.ERR_INVALID_ARG


def test_device_status_text_names_every_bit(zc):
    text = zc.describe_device_status(zc.DEVICE_CANDIDATE_OVERFLOW | zc.DEVICE_TILE_WAIT_TIMEOUT)
    assert "0x9" in text and "corpus tile" in text and "more candidates" in text
    assert "unknown bits 0x20" in zc.describe_device_status(0x20)


def test_shard_bounds_match_the_python_split(zc):
    import sharded

    for n, world in ((10, 3), (50_000_000, 8), (7, 7), (140_011, 2)):
        spans = [zc.shard_bounds(n, world, r) for r in range(world)]
        assert spans == [sharded.shard_bounds(n, world, r) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == n
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    lib = zc.lib()
    b, e = ctypes.c_int64(), ctypes.c_int64()
    assert lib.zcgvs_shard_bounds(10, 0, 0, ctypes.byref(b), ctypes.byref(e)) == zc.ERR_INVALID_ARG
    assert lib.zcgvs_shard_bounds(10, 2, 2, ctypes.byref(b), ctypes.byref(e)) == zc.ERR_INVALID_ARG


def test_sharded_entry_points_check_arguments_before_any_device_or_nccl_call(zc):
    lib = zc.lib()
    handle = ctypes.c_void_p()
    nccl_id = ctypes.create_string_buffer(int(lib.zcgvs_nccl_id_bytes()))
    assert lib.zcgvs_nccl_id_bytes() == 128
    for world, rank, rows in ((0, 0, 10), (2, 2, 10), (4, 0, 3), (2, -1, 10)):
        assert lib.zcgvs_sharded_create(nccl_id, world, rank, rows, ctypes.byref(handle)) == zc.ERR_INVALID_ARG
    assert lib.zcgvs_sharded_create(None, 1, 0, 10, ctypes.byref(handle)) == zc.ERR_INVALID_ARG
    fake = ctypes.c_void_p(16)
    assert lib.zcgvs_sharded_search(None, fake, 4, 1.0, fake, 10, 8, fake, 1, None, 1, 5, 0, fake, fake,
                                    None) == zc.ERR_INVALID_ARG
    assert "null handle" in lib.zcgvs_last_error_message().decode()
    assert lib.zcgvs_sharded_destroy(None) == zc.OK
    # The list merge: no output at all, or a stride shorter than one list.
    assert lib.zcgvs_merge_topk_lists(fake, fake, 100, 2, 2, 50, None, 10, None, None, 0, 0, None,
                                      None) == zc.ERR_INVALID_ARG
    assert lib.zcgvs_merge_topk_lists(fake, fake, 99, 2, 2, 50, None, 10, fake, fake, 0, 0, None,
                                      None) == zc.ERR_INVALID_ARG
    assert "list_stride" in lib.zcgvs_last_error_message().decode()
