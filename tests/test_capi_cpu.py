"""Host-side checks of the C ABI that need no GPU: the library loads, exports
every symbol include/mla_b200.h declares, rejects bad arguments before any
launch, and plans splits sensibly."""
import ctypes
import os
import re

import pytest

from ada_mla import capi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_functions():
    names = []
    for fn in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if fn.endswith(".h"):
            src = open(os.path.join(ROOT, "include", fn)).read()
            src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
            names += re.findall(r"\b(mla_b200_\w+)\s*\(", src)
    return sorted(set(names))


def test_header_declares_entry_points():
    names = _declared_functions()
    assert "mla_b200_decode_split_f16" in names
    assert "mla_b200_combine_f32" in names
    assert len(names) >= 10


@pytest.mark.parametrize("name", _declared_functions())
def test_library_exports_declared_symbol(name):
    lib = ctypes.CDLL(capi.LIB_PATH)
    assert hasattr(lib, name), f"{name} declared in include/ but not exported"


def test_binding_signatures_cover_header():
    assert set(_declared_functions()) == set(capi.SIGNATURES)


def test_constants_and_strings():
    assert capi.constant("HEAD_DIM_K") == 576
    assert capi.constant("HEAD_DIM_V") == 512
    assert capi.constant("HEAD_DIM_ROPE") == 64
    assert capi.constant("NUM_HEADS") == 128
    assert capi.constant("nope") == -1
    assert capi.status_string(0) == "ok"
    assert "workspace" in capi.status_string(capi.ERR_WORKSPACE)


def test_invalid_arguments_rejected_before_launch():
    lib = capi.lib()
    # null query
    assert lib.mla_b200_decode_split_f16(None, None, None, 128, 64, 0, None, 0, None) == capi.ERR_INVALID_ARG
    # negative sizes
    assert lib.mla_b200_decode_batched_f16(16, 16, None, -1, 128, 0, 0, 1.0, 0, 16, 0, None, None, 0,
                                           None) == capi.ERR_INVALID_ARG
    # misaligned pointers
    assert lib.mla_b200_decode_split_f16(18, 16, 16, 128, 64, 0, None, 0, None) == capi.ERR_INVALID_ARG
    # dense batch whose total does not match batch * max_seq_len
    assert lib.mla_b200_decode_batched_f16(16, 16, None, 2, 128, 100, 64, 1.0, 0, 16, 0, None, None, 0,
                                           None) == capi.ERR_INVALID_ARG
    # bad output dtype and bad scale
    assert lib.mla_b200_decode_batched_f16(16, 16, None, 1, 128, 64, 64, 1.0, 0, 16, 7, None, None, 0,
                                           None) == capi.ERR_INVALID_ARG
    assert lib.mla_b200_decode_batched_f16(16, 16, None, 1, 128, 64, 64, float("nan"), 0, 16, 0, None,
                                           None, 0, None) == capi.ERR_INVALID_ARG
    # bf16 entry: fp16 output is not a bf16 output dtype; more than 128 heads unsupported
    assert lib.mla_b200_decode_batched_bf16(16, 16, None, 1, 128, 64, 64, 1.0, 0, 16, capi.OUT_F16,
                                            None, None, 0, None) == capi.ERR_INVALID_ARG
    assert lib.mla_b200_decode_batched_bf16(16, 16, None, 1, 256, 64, 64, 1.0, 0, 16, capi.OUT_BF16,
                                            None, None, 0, None) == capi.ERR_UNSUPPORTED
    # paged: page size not a multiple of 32; max_seq_len beyond the block table;
    # fp16 entry with a bf16 output dtype
    assert lib.mla_b200_decode_paged_f16(16, 16, 16, 16, 1, 128, 4, 48, 4, 64, 1.0, 0, 16, capi.OUT_F16,
                                         None, None, 0, None) == capi.ERR_UNSUPPORTED
    assert lib.mla_b200_decode_paged_f16(16, 16, 16, 16, 1, 128, 4, 64, 2, 200, 1.0, 0, 16, capi.OUT_F16,
                                         None, None, 0, None) == capi.ERR_INVALID_ARG
    assert lib.mla_b200_decode_paged_f16(16, 16, 16, 16, 1, 128, 4, 64, 4, 64, 1.0, 0, 16, capi.OUT_BF16,
                                         None, None, 0, None) == capi.ERR_INVALID_ARG
    assert lib.mla_b200_decode_paged_bf16(16, 16, None, 16, 1, 128, 4, 64, 4, 64, 1.0, 0, 16,
                                          capi.OUT_BF16, None, None, 0, None) == capi.ERR_INVALID_ARG
    # fp8: bad kv scale; bf16 output is not offered
    assert lib.mla_b200_decode_batched_fp8(16, 16, 0.0, None, 1, 128, 64, 64, 1.0, 0, 16, capi.OUT_F16,
                                           None, None, 0, None) == capi.ERR_INVALID_ARG
    assert lib.mla_b200_decode_batched_fp8(16, 16, 1.0, None, 1, 128, 64, 64, 1.0, 0, 16, capi.OUT_BF16,
                                           None, None, 0, None) == capi.ERR_INVALID_ARG
    assert lib.mla_b200_workspace_size_fp8(2, 128, 200, 100, 1) >= \
        lib.mla_b200_workspace_size(2, 128, 200, 100, 1) + 2 * 2 * 128 * 576
    # multi-token: more than 128 heads, zero tokens
    assert lib.mla_b200_decode_mtp_f16(16, 16, None, 1, 2, 256, 64, 64, 1.0, 0, 16, capi.OUT_F16,
                                       None, None, 0, None) == capi.ERR_UNSUPPORTED
    # multi-token workspace: k x n_h <= 128 shares tiles (one sequence of k x n_h rows);
    # above, one sequence of n_h rows per draft token
    assert lib.mla_b200_workspace_size_mtp(3, 8, 16, 3000, 1000, -1) == \
        lib.mla_b200_workspace_size(3, 128, 3000, 1000, -1)
    assert lib.mla_b200_workspace_size_mtp(3, 4, 128, 3000, 1000, -1) == \
        lib.mla_b200_workspace_size(12, 128, 12000, 1000, -1)
    assert lib.mla_b200_decode_mtp_f16(16, 16, None, 1, 0, 16, 64, 64, 1.0, 0, 16, capi.OUT_F16,
                                       None, None, 0, None) == capi.ERR_INVALID_ARG
    # fused fp32 requires head_dim_c = 576
    assert lib.mla_b200_decode_fused_f32(16, 16, 16, 128, 512, 64, None, 0, None) == capi.ERR_UNSUPPORTED
    # naive needs all buffers
    assert lib.mla_b200_decode_naive_f32(16, 16, None, 16, 128, 576, 64, None) == capi.ERR_INVALID_ARG
    # combine: negative parts
    assert lib.mla_b200_combine_f32(16, 16, -1, 4, 16, 0, None, None) == capi.ERR_INVALID_ARG


def test_no_device_reported_without_gpu():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    code = ctypes.c_int(0)
    # A well-formed call on a machine without an sm_100 device reports it instead of crashing.
    st = capi.lib().mla_b200_decode_batched_f16(16, 16, None, 1, 128, 64, 64, 1.0, 0, 16, 0, None,
                                                16, 1 << 30, None)
    assert st == capi.ERR_NO_DEVICE
    assert capi.lib().mla_b200_get_device_error(ctypes.byref(code), None) == capi.ERR_CUDA
    # ... and names the CUDA error behind that status
    assert capi.lib().mla_b200_last_cuda_error() != 0


@pytest.mark.parametrize("batch,total,maxlen", [(1, 4096, 4096), (1, 131072, 131072),
                                                (128, 589824, 8192), (256, 524288, 2048),
                                                (1, 1, 1), (3, 17 * 3, 17), (1, 0, 0)])
def test_plan_properties(batch, total, maxlen):
    chunk, splits = capi.plan(batch, 128, total, maxlen, 148)
    assert chunk >= 1
    if maxlen > 0:
        assert chunk % 96 == 0 or chunk >= maxlen
        assert chunk <= -(-maxlen // 96) * 96
        assert splits == -(-maxlen // chunk)
    if total:
        # a chunk is never shorter than an even share of the tokens over the 74 SM pairs
        # (unless the chunk is already a whole sequence)
        assert -(-total // chunk) <= 74 or chunk == -(-maxlen // 96) * 96
    if maxlen and total == batch * maxlen:
        items = batch * -(-maxlen // chunk)
        assert items <= max(74, batch)


def test_workspace_size_monotone():
    a = capi.workspace_size(1, 128, 4096, 4096, 4)
    b = capi.workspace_size(1, 128, 4096, 4096, 8)
    assert 0 < a < b
    assert capi.workspace_size(1, 128, 4096, 4096, 4) >= 4 * 128 * 512 * 4
    assert capi.workspace_size(-1, 128, 4096, 4096, 4) == 0
