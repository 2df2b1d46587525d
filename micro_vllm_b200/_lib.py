"""ctypes binding of ``libmvb200.so``, the C-ABI library in include/mvb200.h.

The library is built in-tree by ``python -m micro_vllm_b200.build``.  There
is no fallback: loading fails loudly when the library is missing.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libmvb200.so"

MVB_OK = 0
MVB_ERR_INVALID_ARGUMENT = -1
MVB_ERR_UNSUPPORTED_DTYPE = -2
MVB_ERR_UNSUPPORTED_SHAPE = -3
MVB_ERR_WORKSPACE_TOO_SMALL = -4
MVB_ERR_CUDA = -5

MVB_DTYPE_F16 = 0
MVB_DTYPE_BF16 = 1
MVB_DTYPE_F32 = 2

MVB_STATUS_SLOT_OUT_OF_RANGE = 1
MVB_STATUS_BLOCK_OUT_OF_RANGE = 2
MVB_STATUS_POSITION_PAST_TABLE = 4
MVB_STATUS_INCONSISTENT_COUNTS = 8
MVB_STATUS_WAIT_TIMEOUT = 16

MVB_SPEC_FULL = 0
MVB_SPEC_SLIDING_WINDOW = 1
MVB_SPEC_CHUNKED_LOCAL = 2

# Every symbol include/mvb200.h declares, with its ctypes signature.
_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I32 = ctypes.c_int32
_F32 = ctypes.c_float
_SZ = ctypes.c_size_t
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "mvb_version": (ctypes.c_int, []),
    "mvb_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "mvb_last_cuda_error": (ctypes.c_int, []),
    "mvb_reshape_and_cache": (
        ctypes.c_int,
        [_P, _P, _P, _P, _P, _I64, _I32, _I32, _I32, _P, _I64, _I32, _P, _P],
    ),
    "mvb_paged_attention_workspace_size": (_SZ, [_I64, _I64, _I32, _I32, _I32]),
    "mvb_debug_arm_decode_stall": (ctypes.c_int, [_I32, _I32, _I32]),
    "mvb_paged_attention": (
        ctypes.c_int,
        [
            _P, _I64, _I64,  # query, token stride, head stride
            _P,  # output
            _P, _I64, _I32, _I32, _I32,  # cache, num_blocks, block_size, Hkv, D
            _P, _P, _P, _P, _P, _I64, _I64,  # metadata, table stride/width
            _I64, _I64, _I32, _F32, _I32,  # T, R, Hq, scale, dtype
            _P, _SZ, _P, _P,  # workspace, bytes, status, stream
        ],
    ),
    "mvb_paged_attention_no_alloc": (
        ctypes.c_int,
        [
            _P, _I64, _I64,  # query, token stride, head stride
            _P,  # output
            _P, _I64, _I32, _I32, _I32,  # cache, num_blocks, block_size, Hkv, D
            _P, _P, _P, _P, _P, _I64, _I64,  # metadata, table stride/width
            _I64, _I64, _I32, _F32, _I32,  # T, R, Hq, scale, dtype
            _P, _P,  # status, stream
        ],
    ),
    "mvb_qk_norm_rope_and_cache": (
        ctypes.c_int,
        [
            _P, _P, _P, _P, _P, _P,  # query, strides, key, strides, value, strides
            _P, _P, _P, _F32, _P, _P,  # q_out, q_weight, k_weight, eps, inv_freq, positions
            _P, _I64, _I32, _I32, _I32,  # cache, NB, bs, Hkv, D
            _P, _I64, _I32, _I32, _P, _P,  # slots, T, Hq, dtype, status, stream
        ],
    ),
    "mvb_sample": (
        ctypes.c_int,
        [_P, _I64, _I64, _I64, _I32, _P, _P, _P, _P, _P, _P, _P],
    ),
    "mvb_rms_norm": (
        ctypes.c_int,
        [_P, _I64, _P, _I64, _P, _P, _P, _F32, _I64, _I32, _I32, _P],
    ),
    "mvb_silu_mul": (
        ctypes.c_int,
        [_P, _I64, _P, _I64, _I32, _I32, _P],
    ),
    "mvb_sample_with_noise": (
        ctypes.c_int,
        [_P, _I64, _I64, _I64, _I32, _P, _P, _P, _P, _P, _P, _I64, _I64, _P, _P, _P],
    ),
    "mvb_build_metadata": (
        ctypes.c_int,
        [
            _P, _P, _P, _P, _P, _P,  # computed, scheduled, block counts, block ids, flags, token ids
            _I64, _I64, _I64, _I64,  # requests, tokens, block ids, sampled
            _I64, _I64, _I64, _I64,  # request / token capacity, table width / stride
            _I32, _I64, _I32, _I64,  # block size, null block, spec kind / param
            _P, _P, _P, _P, _P, _P, _P, _P,  # outputs
            _P, _P,  # status, stream
        ],
    ),
    "mvb_attention_forward": (
        ctypes.c_int,
        [
            _P, _I64, _I64,  # query
            _P, _P, _P, _P,  # key, key strides, value, value strides
            _P, _P, _I64, _I32, _I32, _I32,  # output, cache, NB, bs, Hkv, D
            _P, _P, _P, _P, _P, _I64, _I64,  # metadata
            _P, _I64, _I64, _I32, _F32, _I32,  # slots, T, R, Hq, scale, dtype
            _P, _SZ, _P, _P,  # workspace, bytes, status, stream
        ],
    ),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class MVBError(RuntimeError):
    """A non-zero status from the CUDA library."""


def load() -> ctypes.CDLL:
    """Load the library once and declare every exported signature."""

    global _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH.name} is not built; run `python -m micro_vllm_b200.build` "
                    "(the b200_paged backend has no CPU fallback)"
                )
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (restype, argtypes) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = restype
                fn.argtypes = argtypes
            _lib = lib
        return _lib


def check(status: int, what: str) -> None:
    """Raise the exception the reference backends raise for this status."""

    if status == MVB_OK:
        return
    lib = load()
    text = lib.mvb_status_string(status).decode()
    if status in (MVB_ERR_UNSUPPORTED_DTYPE, MVB_ERR_UNSUPPORTED_SHAPE, MVB_ERR_INVALID_ARGUMENT):
        raise ValueError(f"{what}: {text}")
    if status == MVB_ERR_CUDA:
        raise MVBError(f"{what}: CUDA error {lib.mvb_last_cuda_error()}")
    raise MVBError(f"{what}: {text}")


def strides3(strides: tuple[int, ...]) -> ctypes.Array:
    return (ctypes.c_int64 * 3)(*strides)
