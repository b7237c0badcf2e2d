"""CPU tests of the C-ABI boundary: the library loads, exports every function
include/qwen_b200.h declares, and rejects bad arguments before touching CUDA."""

import ctypes as C

import pytest

from qwen_fpga_b200 import api


def test_library_exports_every_header_symbol():
    L = api.load()
    syms = api.header_symbols()
    assert len(syms) >= 12
    for s in syms:
        assert hasattr(L, s), s
    assert b"sm_100a" in L.qwen_version()


def test_create_rejects_bad_arguments():
    L = api.load()
    h = C.c_void_p()
    assert L.qwen_create(b"x", b"y", 2, None, 16, 1, C.byref(h)) == api.QWEN_ERR_ARG
    assert b"n_gpus" in L.qwen_last_error(None)
    assert L.qwen_create(b"x", b"y", 1, None, 16, 0, C.byref(h)) == api.QWEN_ERR_ARG
    assert L.qwen_create(b"x", b"y", 1, None, 16, 65, C.byref(h)) == api.QWEN_ERR_ARG
    assert b"max_batch" in L.qwen_last_error(None)
    assert L.qwen_create_tp(b"x", b"y", 0, 0, 2, 16, 2, C.byref(h)) == api.QWEN_ERR_ARG
    assert L.qwen_create(b"x", b"y", 1, None, 0, 1, C.byref(h)) == api.QWEN_ERR_ARG
    assert L.qwen_create(None, b"y", 1, None, 16, 1, C.byref(h)) == api.QWEN_ERR_ARG
    assert L.qwen_create(b"x", b"y", 1, None, 16, 1, None) == api.QWEN_ERR_ARG


def test_operators_reject_bad_arguments():
    L = api.load()
    assert L.qwen_gemv_i8_f32(None, None, None, None, 4, 1024, None) == api.QWEN_ERR_ARG
    fake = C.c_void_p(64)     # never dereferenced: the K check fails first
    assert L.qwen_gemv_i8_f32(fake, fake, fake, fake, 4, 48, None) == api.QWEN_ERR_ARG
    assert L.qwen_gemv_i8_f32(fake, fake, fake, fake, 4, 4096, None) == api.QWEN_ERR_ARG
    assert L.qwen_gemv_i8_f32(fake, fake, fake, fake, 0, 1024, None) == api.QWEN_ERR_ARG
    assert L.qwen_gemv_i8_i8(None, None, fake, fake, fake, 1.0, 4, 1024, None) == api.QWEN_ERR_ARG
    odd = C.c_void_p(64 + 16)  # 16- but not 32-byte aligned weights
    assert L.qwen_gemv_i8_i8(fake, fake, odd, fake, fake, 1.0, 4, 1024, None) == api.QWEN_ERR_ARG
    assert L.qwen_delta_rule_layer(None, None, None, None, None, None, None, None) == api.QWEN_ERR_ARG
    # batched GEMM: N a multiple of 128, K of 128 in [128, 4096], B in [1, 64], 16-byte alignment
    assert L.qwen_gemm_i8_i8(None, None, fake, fake, fake, fake, 128, 128, 1, None) == api.QWEN_ERR_ARG
    assert L.qwen_gemm_i8_i8(fake, None, fake, fake, fake, fake, 100, 128, 1, None) == api.QWEN_ERR_ARG
    assert L.qwen_gemm_i8_i8(fake, None, fake, fake, fake, fake, 128, 4224, 1, None) == api.QWEN_ERR_ARG
    assert L.qwen_gemm_i8_i8(fake, None, fake, fake, fake, fake, 128, 128, 65, None) == api.QWEN_ERR_ARG
    assert L.qwen_gemm_i8_i8(fake, None, C.c_void_p(72), fake, fake, fake, 128, 128, 1, None) == api.QWEN_ERR_ARG


def test_null_context_is_an_error():
    L = api.load()
    assert L.qwen_reset(None, 0) == api.QWEN_ERR_ARG
    assert L.qwen_set_act_int8(None, 1) == api.QWEN_ERR_ARG
    assert L.qwen_decode_timed(None, 1, 1, None) == api.QWEN_ERR_ARG
    assert L.qwen_destroy(None) == api.QWEN_OK


def test_index_parsers_roundtrip(tmp_path, blob_path):
    """The manifest JSON and the flat index describe the same layout (CPU-side check
    of what qwen_create parses)."""
    import json
    from qwen_fpga_b200 import synth
    man = json.load(open(synth.manifest_path(blob_path)))
    idx = open(synth.index_path(blob_path)).read().splitlines()
    assert synth.index_lines(man) == idx
