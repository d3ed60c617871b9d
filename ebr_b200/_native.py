"""ctypes binding of the C ABI in ``include/ebr_attn.h`` (``libebr_attn.so``, built in-tree by ``ebr_b200.build``).

There is no fallback: if the shared library is missing or cannot be loaded, every op raises.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

LIB_NAME = "libebr_attn.so"
LIB_PATH = Path(__file__).resolve().parent / LIB_NAME

# ebr_dtype / ebr_status (include/ebr_attn.h)
FLOAT32, FLOAT16, BFLOAT16, FLOAT64 = 0, 1, 2, 3
OK = 0
ERR_NULL, ERR_SHAPE, ERR_DTYPE, ERR_STRIDE, ERR_SCRATCH, ERR_CUDA, ERR_DEVICE, ERR_DEVICE_TIMEOUT = range(1, 9)

EXPORTED = (
    "ebr_attn_fwd",
    "ebr_attn_bwd",
    "ebr_attn_bwd_bwd",
    "ebr_attn_bwd_scratch_bytes",
    "ebr_attn_bwd_bwd_scratch_bytes",
    "ebr_attn_uses_tensor_cores",
    "ebr_attn_device_status",
    "ebr_attn_status_string",
    "ebr_attn_last_error",
    "ebr_attn_launch_count",
    "ebr_attn_bwd_noalloc",
    "ebr_attn_test_bounded_wait",
)

# include/ebr_layers.h: the fused kernels on either side of the attention.
EXPORTED_LAYERS = (
    "ebr_rope_split",
    "ebr_rope_merge",
    "ebr_qkv_rope_split",
    "ebr_o_proj",
    "ebr_qkv_rope_merge_dx",
    "ebr_add_rms_norm",
    "ebr_rms_norm_bwd",
    "ebr_swiglu_fwd",
    "ebr_swiglu_bwd",
    "ebr_swiglu_bwd2",
    "ebr_rms_norm_bwd2",
    "ebr_gate_up_swiglu",
    "ebr_descent_step",
    "ebr_descent_step_scratch_floats",
)


class Operand(ctypes.Structure):
    """``ebr_operand``: a strided [B, H, N, D] operand (strides in elements, unit head-dim stride)."""

    _fields_ = [
        ("data", ctypes.c_void_p),
        ("stride_b", ctypes.c_int64),
        ("stride_h", ctypes.c_int64),
        ("stride_n", ctypes.c_int64),
    ]


class AttnError(RuntimeError):
    """A non-zero ``ebr_status`` from the native library."""

    def __init__(self, status: int, what: str, detail: str) -> None:
        super().__init__(f"{what} failed: {detail} (status {status})")
        self.status = status


_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def _declare(lib: ctypes.CDLL) -> None:
    i64, vp, sz = ctypes.c_int64, ctypes.c_void_p, ctypes.c_size_t
    op = ctypes.POINTER(Operand)
    dims = [ctypes.c_int, i64, i64, i64, i64]
    lib.ebr_attn_fwd.argtypes = dims + [ctypes.c_double, op, op, op, vp, vp, vp]
    lib.ebr_attn_bwd.argtypes = dims + [ctypes.c_double, op, op, op, vp, vp, op, vp, vp, vp, vp, sz, vp]
    lib.ebr_attn_bwd_bwd.argtypes = dims + [ctypes.c_double, op, op, op, vp, vp, op, vp, op, op, op] + [vp] * 5 + [
        sz,
        vp,
    ]
    lib.ebr_attn_bwd_noalloc.argtypes = dims + [ctypes.c_double, op, op, op, vp, vp, op, vp, vp, vp, vp]
    lib.ebr_attn_bwd_noalloc.restype = ctypes.c_int
    lib.ebr_attn_bwd_scratch_bytes.argtypes = dims
    lib.ebr_attn_bwd_scratch_bytes.restype = sz
    lib.ebr_attn_bwd_bwd_scratch_bytes.argtypes = dims
    lib.ebr_attn_bwd_bwd_scratch_bytes.restype = sz
    lib.ebr_attn_uses_tensor_cores.argtypes = [ctypes.c_int, i64, op, op, op]
    lib.ebr_attn_device_status.argtypes = []
    lib.ebr_attn_status_string.argtypes = [ctypes.c_int]
    lib.ebr_attn_status_string.restype = ctypes.c_char_p
    lib.ebr_attn_last_error.argtypes = []
    lib.ebr_attn_last_error.restype = ctypes.c_char_p
    lib.ebr_attn_launch_count.argtypes = []
    lib.ebr_attn_launch_count.restype = ctypes.c_uint64
    lib.ebr_attn_test_bounded_wait.argtypes = [i64, vp]
    for name in ("ebr_attn_fwd", "ebr_attn_bwd", "ebr_attn_bwd_bwd", "ebr_attn_uses_tensor_cores",
                 "ebr_attn_device_status", "ebr_attn_test_bounded_wait"):  # fmt: skip
        getattr(lib, name).restype = ctypes.c_int
    dbl, fp = ctypes.c_double, ctypes.c_void_p
    lib.ebr_rope_split.argtypes = dims + [vp, i64, i64, fp, fp, fp, vp, vp, vp, vp]
    lib.ebr_rope_merge.argtypes = dims + [op, op, op, fp, fp, fp, vp, vp]
    lib.ebr_qkv_rope_split.argtypes = dims + [i64, vp, i64, vp, fp, fp, fp, vp, vp, vp, vp]
    lib.ebr_o_proj.argtypes = dims + [i64, op, vp, vp, vp]
    lib.ebr_qkv_rope_merge_dx.argtypes = dims + [i64, op, op, op, vp, fp, fp, fp, vp, vp, vp]
    lib.ebr_add_rms_norm.argtypes = [ctypes.c_int, i64, i64, dbl, vp, vp, vp, vp, fp, vp, dbl, vp]
    lib.ebr_rms_norm_bwd.argtypes = [ctypes.c_int, i64, i64, vp, fp, vp, vp, vp]
    lib.ebr_swiglu_fwd.argtypes = [ctypes.c_int, i64, i64, vp, vp, vp]
    lib.ebr_swiglu_bwd.argtypes = [ctypes.c_int, i64, i64, vp, vp, vp, vp]
    lib.ebr_swiglu_bwd2.argtypes = [ctypes.c_int, i64, i64, vp, vp, vp, vp, vp, vp]
    lib.ebr_rms_norm_bwd2.argtypes = [ctypes.c_int, i64, i64, vp, fp, vp, vp, vp, vp, vp]
    lib.ebr_gate_up_swiglu.argtypes = [ctypes.c_int, i64, i64, i64, vp, i64, vp, vp, vp, vp]
    lib.ebr_descent_step.argtypes = [ctypes.c_int, i64, i64, dbl, dbl, vp, vp, vp, fp, sz, vp]
    lib.ebr_descent_step_scratch_floats.argtypes = [i64, i64]
    lib.ebr_descent_step_scratch_floats.restype = sz
    for name in EXPORTED_LAYERS[:-1]:
        getattr(lib, name).restype = ctypes.c_int


def lib() -> ctypes.CDLL:
    """The loaded native library. Raises ``RuntimeError`` when it is not built: there is no other implementation."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            path = Path(os.environ.get("EBR_ATTN_LIB", LIB_PATH))
            if not path.exists():
                raise RuntimeError(
                    f"ebr_b200: native library {path} is not built; run `python -c 'import __graft_entry__ as g; "
                    "g.build()'` or `python -m ebr_b200.build` (needs nvcc for sm_100a)"
                )
            handle = ctypes.CDLL(str(path))
            _declare(handle)
            _lib = handle
    return _lib


def check(status: int, what: str) -> None:
    if status != OK:
        l = lib()
        detail = l.ebr_attn_last_error().decode() or l.ebr_attn_status_string(status).decode()
        if status in (ERR_SHAPE, ERR_DTYPE, ERR_STRIDE, ERR_NULL):
            raise ValueError(f"{what}: {detail} (status {status})")
        raise AttnError(status, what, detail)


def device_status() -> None:
    """Synchronize and raise if a bounded device-side wait ran out since the last check."""
    check(lib().ebr_attn_device_status(), "device status")


def launch_count() -> int:
    return int(lib().ebr_attn_launch_count())
