"""The C ABI library on the CPU host: it loads, exports every symbol include/ebr_attn.h declares, and rejects bad
arguments with the documented status codes before touching a device (no compute without a GPU)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from ebr_b200 import _native
from ebr_b200.build import OUT, build

HEADER = Path(__file__).resolve().parent.parent / "include" / "ebr_attn.h"
LAYERS_HEADER = HEADER.with_name("ebr_layers.h")


@pytest.fixture(scope="module")
def lib():
    build()
    return _native.lib()


def declared_functions(header: Path = HEADER) -> list[str]:
    text = header.read_text()
    return sorted(set(re.findall(r"^\s*(?:int|size_t|const char\*|uint64_t)\s+(ebr_\w+)\s*\(", text, re.M)))


def test_header_declares_the_reference_entry_points():
    names = declared_functions()
    for n in ("ebr_attn_fwd", "ebr_attn_bwd", "ebr_attn_bwd_bwd"):
        assert n in names
    assert set(_native.EXPORTED) <= set(names)


def test_library_exports_every_declared_symbol(lib):
    assert OUT.exists()
    for name in declared_functions() + declared_functions(LAYERS_HEADER):
        assert hasattr(lib, name), name
    assert set(_native.EXPORTED_LAYERS) == set(declared_functions(LAYERS_HEADER))


def test_layer_entry_points_reject_bad_arguments_before_device(lib):
    r = ctypes.byref
    op = _op()
    t = 0x1000
    # RoPE: head dim not a multiple of 4, unknown dtype, NULL tables
    assert lib.ebr_rope_split(_native.BFLOAT16, 1, 4, 2, 6, t, 0, 36, t, t, None, t, t, t, None) == _native.ERR_SHAPE
    assert lib.ebr_rope_split(9, 1, 4, 2, 8, t, 0, 48, t, t, None, t, t, t, None) == _native.ERR_DTYPE
    assert lib.ebr_rope_split(_native.BFLOAT16, 1, 4, 2, 8, t, 0, 48, None, t, None, t, t, t, None) == _native.ERR_NULL
    assert lib.ebr_rope_merge(_native.BFLOAT16, 1, 4, 2, 8, None, r(op), r(op), t, t, None, t, None) == _native.ERR_NULL
    # row kernels: float64 is not a layer dtype; bad row length; NULL output
    assert lib.ebr_add_rms_norm(_native.FLOAT64, 4, 8, 1e-5, t, None, None, t, None, None, 0.0, None) == _native.ERR_DTYPE
    assert lib.ebr_add_rms_norm(_native.BFLOAT16, 4, 0, 1e-5, t, None, None, t, None, None, 0.0, None) == _native.ERR_SHAPE
    assert lib.ebr_swiglu_fwd(_native.BFLOAT16, 4, 8, t, None, None) == _native.ERR_NULL
    assert lib.ebr_rms_norm_bwd(_native.BFLOAT16, 4, 8, t, None, t, t, None) == _native.ERR_NULL
    # descent step: scratch too small
    need = lib.ebr_descent_step_scratch_floats(4, 460800)
    assert need == 4 * ((460800 + 8191) // 8192)
    assert lib.ebr_descent_step(_native.BFLOAT16, 4, 460800, 1.0, 1e-5, t, t, t, t, need - 1, None) == _native.ERR_SCRATCH
    # empty problems are no-ops
    assert lib.ebr_rope_split(_native.BFLOAT16, 0, 4, 2, 8, None, 0, 48, None, None, None, None, None, None, None) == 0
    # The fused projection: 16-bit only, D = 64 / 128 with H D % 256 == 0 and C % 64 == 0, aligned row strides.
    q = lib.ebr_qkv_rope_split
    assert q(_native.FLOAT32, 1, 4, 4, 64, 64, t, 64, t, t, t, None, t, t, t, None) == _native.ERR_DTYPE
    assert q(_native.BFLOAT16, 1, 4, 2, 64, 64, t, 64, t, t, t, None, t, t, t, None) == _native.ERR_SHAPE
    assert q(_native.BFLOAT16, 1, 4, 4, 32, 64, t, 64, t, t, t, None, t, t, t, None) == _native.ERR_SHAPE
    assert q(_native.BFLOAT16, 1, 4, 4, 64, 96, t, 96, t, t, t, None, t, t, t, None) == _native.ERR_SHAPE
    assert q(_native.BFLOAT16, 1, 4, 4, 64, 64, None, 64, t, t, t, None, t, t, t, None) == _native.ERR_NULL
    assert q(_native.BFLOAT16, 1, 4, 4, 64, 64, t, 60, t, t, t, None, t, t, t, None) == _native.ERR_STRIDE
    assert q(_native.BFLOAT16, 0, 4, 4, 64, 64, None, 64, None, None, None, None, None, None, None, None) == 0
    # The o projection: 16-bit only, D = 64 / 128, C_out a multiple of 256, aligned operand and pointers.
    p = lib.ebr_o_proj
    good = _op()
    assert p(_native.FLOAT32, 1, 4, 8, 64, 256, r(good), t, t, None) == _native.ERR_DTYPE
    assert p(_native.BFLOAT16, 1, 4, 8, 32, 256, r(good), t, t, None) == _native.ERR_SHAPE
    assert p(_native.BFLOAT16, 1, 4, 8, 64, 128, r(good), t, t, None) == _native.ERR_SHAPE
    assert p(_native.BFLOAT16, 1, 4, 8, 64, 256, None, t, t, None) == _native.ERR_NULL
    assert p(_native.BFLOAT16, 1, 4, 8, 64, 256, r(good), None, t, None) == _native.ERR_NULL
    assert p(_native.BFLOAT16, 1, 4, 8, 64, 256, r(good), t + 2, t, None) == _native.ERR_STRIDE
    assert p(_native.BFLOAT16, 0, 4, 8, 64, 256, None, None, None, None) == 0
    # The gate / up projection: 16-bit only, C % 64 == 0, I % 128 == 0, aligned row stride.
    gu = lib.ebr_gate_up_swiglu
    assert gu(_native.FLOAT32, 4, 64, 128, t, 64, t, t, t, None) == _native.ERR_DTYPE
    assert gu(_native.BFLOAT16, 4, 96, 128, t, 96, t, t, t, None) == _native.ERR_SHAPE
    assert gu(_native.BFLOAT16, 4, 64, 192, t, 64, t, t, t, None) == _native.ERR_SHAPE
    assert gu(_native.BFLOAT16, 4, 64, 128, t, 64, None, t, t, None) == _native.ERR_NULL
    assert gu(_native.BFLOAT16, 4, 64, 128, t, 60, t, t, t, None) == _native.ERR_STRIDE
    assert gu(_native.BFLOAT16, 0, 64, 128, None, 64, None, None, None, None) == 0
    assert lib.ebr_add_rms_norm(_native.BFLOAT16, 0, 8, 1e-5, None, None, None, None, None, None, 0.0, None) == 0
    # The qkv input gradient with the merge in the GEMM: 16-bit only, D = 64 and C = 512, aligned operands.
    md = lib.ebr_qkv_rope_merge_dx
    g8 = _op(t, 8 * 4 * 64, 4 * 64, 64)  # [1, 8, 4, 64] contiguous
    assert md(_native.FLOAT32, 1, 4, 8, 64, 512, r(g8), r(g8), r(g8), t, t, t, None, None, t, None) == _native.ERR_DTYPE
    assert md(_native.BFLOAT16, 1, 4, 8, 128, 512, r(g8), r(g8), r(g8), t, t, t, None, None, t, None) == _native.ERR_SHAPE
    assert md(_native.BFLOAT16, 1, 4, 8, 64, 256, r(g8), r(g8), r(g8), t, t, t, None, None, t, None) == _native.ERR_SHAPE
    assert md(_native.BFLOAT16, 1, 4, 8, 64, 512, r(g8), r(g8), r(g8), None, t, t, None, None, t, None) == _native.ERR_NULL
    assert md(_native.BFLOAT16, 1, 4, 8, 64, 512, r(g8), r(g8), r(g8), t + 2, t, t, None, None, t, None) == _native.ERR_STRIDE
    assert md(_native.BFLOAT16, 0, 4, 8, 64, 512, None, None, None, None, None, None, None, None, None, None) == 0
    # The double backwards of rms_norm and SwiGLU: layer dtypes only, a row length, every buffer.
    assert lib.ebr_rms_norm_bwd2(_native.FLOAT64, 4, 8, t, t, t, t, t, t, None) == _native.ERR_DTYPE
    assert lib.ebr_rms_norm_bwd2(_native.BFLOAT16, 4, 0, t, t, t, t, t, t, None) == _native.ERR_SHAPE
    assert lib.ebr_rms_norm_bwd2(_native.BFLOAT16, 4, 8, t, t, t, None, t, t, None) == _native.ERR_NULL
    assert lib.ebr_rms_norm_bwd2(_native.BFLOAT16, 0, 8, None, None, None, None, None, None, None) == 0
    assert lib.ebr_swiglu_bwd2(_native.BFLOAT16, 4, 0, t, t, t, t, t, None) == _native.ERR_SHAPE
    assert lib.ebr_swiglu_bwd2(_native.BFLOAT16, 4, 8, t, t, t, t, None, None) == _native.ERR_NULL
    assert lib.ebr_swiglu_bwd2(_native.BFLOAT16, 0, 8, None, None, None, None, None, None) == 0


def _op(ptr=0x1000, sb=0, sh=0, sn=64):
    return _native.Operand(ptr, sb, sh, sn)


def test_argument_errors_before_device(lib):
    q = _op()
    r = ctypes.byref
    # D out of range
    assert lib.ebr_attn_fwd(_native.BFLOAT16, 1, 1, 4, 0, 0.1, r(q), r(q), r(q), 0x2000, 0x3000, None) == _native.ERR_SHAPE
    assert lib.ebr_attn_fwd(_native.BFLOAT16, 1, 1, 4, 300, 0.1, r(q), r(q), r(q), 0x2000, 0x3000, None) == _native.ERR_SHAPE
    # unknown dtype
    assert lib.ebr_attn_fwd(9, 1, 1, 4, 64, 0.1, r(q), r(q), r(q), 0x2000, 0x3000, None) == _native.ERR_DTYPE
    # null operand / output
    assert lib.ebr_attn_fwd(_native.BFLOAT16, 1, 1, 4, 64, 0.1, None, r(q), r(q), 0x2000, 0x3000, None) == _native.ERR_NULL
    assert lib.ebr_attn_fwd(_native.BFLOAT16, 1, 1, 4, 64, 0.1, r(q), r(q), r(q), None, 0x3000, None) == _native.ERR_NULL
    # negative stride
    bad = _op(sn=-64)
    assert lib.ebr_attn_fwd(_native.BFLOAT16, 1, 1, 4, 64, 0.1, r(q), r(bad), r(q), 0x2000, 0x3000, None) == _native.ERR_STRIDE
    # negative size
    assert lib.ebr_attn_fwd(_native.BFLOAT16, -1, 1, 4, 64, 0.1, r(q), r(q), r(q), 0x2000, 0x3000, None) == _native.ERR_SHAPE
    assert lib.ebr_attn_last_error()  # a message was recorded


def test_empty_problem_is_a_no_op(lib):
    q = _op()
    r = ctypes.byref
    assert lib.ebr_attn_fwd(_native.BFLOAT16, 0, 8, 81, 64, 0.125, r(q), r(q), r(q), 0x2000, 0x3000, None) == _native.OK
    assert lib.ebr_attn_bwd(_native.FLOAT32, 2, 8, 0, 64, 0.125, r(q), r(q), r(q), 0x2, 0x3, r(q), 0x4, 0x5, 0x6,
                            None, 0, None) == _native.OK  # fmt: skip
    assert lib.ebr_attn_bwd_bwd(_native.FLOAT32, 2, 0, 5, 64, 0.125, r(q), r(q), r(q), 0x2, 0x3, r(q), None,
                                None, None, None, 0x4, 0x5, 0x6, 0x7, None, 0, None) == _native.OK  # fmt: skip


def test_scratch_sizes(lib):
    assert lib.ebr_attn_bwd_scratch_bytes(_native.BFLOAT16, 2, 8, 81, 64) == 2 * 8 * 81 * 4
    assert lib.ebr_attn_bwd_scratch_bytes(_native.FLOAT64, 2, 8, 81, 64) == 2 * 8 * 81 * 8
    assert lib.ebr_attn_bwd_bwd_scratch_bytes(_native.BFLOAT16, 2, 8, 81, 64) == 3 * 2 * 8 * 81 * 4


def test_kernel_family_choice(lib):
    r = ctypes.byref
    ok = _op(0x1000, 81 * 64 * 8, 81 * 64, 64)
    assert lib.ebr_attn_uses_tensor_cores(_native.BFLOAT16, 64, r(ok), r(ok), r(ok)) == 1
    assert lib.ebr_attn_uses_tensor_cores(_native.FLOAT16, 128, r(ok), r(ok), r(ok)) == 1
    assert lib.ebr_attn_uses_tensor_cores(_native.FLOAT32, 64, r(ok), r(ok), r(ok)) == 0
    assert lib.ebr_attn_uses_tensor_cores(_native.BFLOAT16, 32, r(ok), r(ok), r(ok)) == 0
    odd = _op(0x1000, 81 * 65, 81 * 65, 65)  # token stride not a 16-byte multiple: CUDA-core kernels
    assert lib.ebr_attn_uses_tensor_cores(_native.BFLOAT16, 64, r(odd), r(ok), r(ok)) == 0
    misaligned = _op(0x1002, 0, 0, 64)
    assert lib.ebr_attn_uses_tensor_cores(_native.BFLOAT16, 64, r(misaligned), r(ok), r(ok)) == 0


def test_status_strings(lib):
    assert lib.ebr_attn_status_string(0) == b"ok"
    assert lib.ebr_attn_status_string(_native.ERR_DEVICE_TIMEOUT) == b"device wait timed out"


def test_size_products_are_bounded_before_any_arithmetic(lib):
    """B * H >= 2^31 or B * H * N >= 2^40 is refused on the host (each factor alone is within [0, 2^30])."""
    q = _op()
    r = ctypes.byref
    big = 1 << 30
    assert lib.ebr_attn_fwd(_native.BFLOAT16, big, 4, 8, 64, 0.1, r(q), r(q), r(q), 0x2000, 0x3000, None) == _native.ERR_SHAPE
    assert lib.ebr_attn_fwd(_native.BFLOAT16, 1 << 20, 1 << 10, 1 << 10, 64, 0.1, r(q), r(q), r(q), 0x2000, 0x3000,
                            None) == _native.ERR_SHAPE  # fmt: skip
    # the allocation-free backward refuses them too, before sizing its scratch (no wrap below the buffer size)
    assert lib.ebr_attn_bwd_noalloc(_native.BFLOAT16, 1 << 20, 1 << 10, 1 << 10, 64, 0.1, r(q), r(q), r(q), 0x2,
                                    0x3, r(q), 0x4, 0x5, 0x6, None) == _native.ERR_SHAPE  # fmt: skip
    assert lib.ebr_attn_test_bounded_wait(10, None) == _native.ERR_SHAPE  # limit outside [1 us, 1 s]


@pytest.mark.gpu
def test_bounded_wait_reports_a_timeout_and_the_context_survives(lib):
    """The device error path: a wait that nothing completes runs out after its limit (50 ms), the host reads
    EBR_ERR_DEVICE_TIMEOUT once (the word is then cleared), and the context keeps working."""
    import torch

    torch.cuda.synchronize()
    assert lib.ebr_attn_device_status() == _native.OK
    assert lib.ebr_attn_test_bounded_wait(50_000_000, None) == _native.OK
    assert lib.ebr_attn_device_status() == _native.ERR_DEVICE_TIMEOUT
    assert b"9001" in lib.ebr_attn_last_error()
    assert lib.ebr_attn_device_status() == _native.OK
    x = torch.arange(1024, device="cuda", dtype=torch.float32)
    assert float(x.sum()) == 1023 * 1024 / 2

