"""ctypes binding of ``libasterq.so`` (declared in ``include/asterq.h``).

The package calls the CUDA kernels only through this C ABI, with raw device
pointers taken from torch tensors and torch's current CUDA stream.  There is no
CPU fallback: if the library is missing every entry point raises.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

_LIB_PATH = Path(__file__).resolve().parent / "libasterq.so"

ASTERQ_OK = 0
ASTERQ_ERR_INVALID_ARGUMENT = -1
ASTERQ_ERR_UNSUPPORTED = -2
ASTERQ_ERR_MISALIGNED = -3
ASTERQ_ERR_WORKSPACE = -4
ASTERQ_ERR_CUDA = -5

DTYPE_F32 = 0
DTYPE_BF16 = 1
DTYPE_F16 = 2


def dtype_code(dtype) -> int:
    """The C ABI's element-type code of a torch dtype (float32, bfloat16, float16)."""
    import torch

    codes = {torch.float32: DTYPE_F32, torch.bfloat16: DTYPE_BF16, torch.float16: DTYPE_F16}
    if dtype not in codes:
        raise TypeError(f"dtype {dtype}: the kernels read float32, bfloat16 or float16")
    return codes[dtype]

SCHEME_HADAMARD_INT4 = 0
SCHEME_INT4 = 1
SCHEME_INT8 = 2
SCHEME_FLOAT8 = 3
ROPE_BF16 = 0  # cold RoPE keys stored as bf16
ROPE_QUANTIZED = 1  # cold RoPE keys stored as INT4 codes of the cold scheme + one fp16 scale a token

TILE_COLD = 0
TILE_HOT = 1
TILE_NEW = 2
TILE_HOLD = 3  # failure-detection test hook (see include/asterq.h)

IPC_HANDLE_BYTES = 64

# entry points declared in include/asterq.h
EXPORTED_SYMBOLS = (
    "asterq_version",
    "asterq_last_error",
    "asterq_quantize",
    "asterq_dequantize",
    "asterq_fwht",
    "asterq_codec_status",
    "asterq_decode_workspace_bytes",
    "asterq_latent_decode",
    "asterq_latent_decode_noalloc",
    "asterq_splitkv_combine",
    "asterq_splitkv_merge",
    "asterq_splitkv_combine_ranks",
    "asterq_mailbox_bytes",
    "asterq_mailbox_create",
    "asterq_mailbox_open",
    "asterq_mailbox_close",
    "asterq_mailbox_destroy",
    "asterq_cp_merge_push",
    "asterq_cp_combine_wait",
    "asterq_plan_scratch_bytes",
    "asterq_plan_batch",
    "asterq_batch_append",
)


class DecodeParams(ctypes.Structure):
    """Mirror of ``asterq_decode_params``."""

    _fields_ = [
        ("n_heads", ctypes.c_int32),
        ("latent_dim", ctypes.c_int32),
        ("rope_dim", ctypes.c_int32),
        ("group_size", ctypes.c_int32),
        ("page_tokens", ctypes.c_int32),
        ("out_dtype", ctypes.c_int32),
        ("softmax_scale", ctypes.c_float),
        ("logit_softcap", ctypes.c_float),
        ("n_cold_pages", ctypes.c_int64),
        ("n_hot_pages", ctypes.c_int64),
        ("total_q", ctypes.c_int64),
        ("n_tiles", ctypes.c_int32),
        ("n_items", ctypes.c_int32),
        ("n_combine", ctypes.c_int32),
        ("n_slots", ctypes.c_int32),
        ("q_lat", ctypes.c_void_p),
        ("q_rope", ctypes.c_void_p),
        ("new_latent", ctypes.c_void_p),
        ("new_rope", ctypes.c_void_p),
        ("cold_codes", ctypes.c_void_p),
        ("cold_scales", ctypes.c_void_p),
        ("cold_rope", ctypes.c_void_p),
        ("hot_latent", ctypes.c_void_p),
        ("hot_rope", ctypes.c_void_p),
        ("tiles", ctypes.c_void_p),
        ("items", ctypes.c_void_p),
        ("combine", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_int64),
        ("device_status", ctypes.c_void_p),
        ("units", ctypes.c_void_p),
        ("n_units", ctypes.c_int32),
        ("cold_scheme", ctypes.c_int32),
        ("workers", ctypes.c_void_p),
        ("n_workers", ctypes.c_int32),
        ("n_combine_total", ctypes.c_int32),
        ("unit_jobs", ctypes.c_void_p),
        ("wait_limit_cycles", ctypes.c_int64),
        ("plan_counts", ctypes.c_void_p),
        ("rope_scheme", ctypes.c_int32),
        ("cold_rope_scales", ctypes.c_void_p),
    ]


class BatchDesc(ctypes.Structure):
    """Mirror of ``asterq_batch_desc`` (device page tables and lengths of a ragged batch)."""

    _fields_ = [
        ("n_seqs", ctypes.c_int32),
        ("n_heads", ctypes.c_int32),
        ("page_tokens", ctypes.c_int32),
        ("max_cold_pages", ctypes.c_int32),
        ("max_hot_pages", ctypes.c_int32),
        ("n_workers", ctypes.c_int32),
        ("n_cold_pages", ctypes.c_void_p),
        ("cold_pages", ctypes.c_void_p),
        ("cold_page_tokens", ctypes.c_void_p),
        ("hot_tokens", ctypes.c_void_p),
        ("hot_pages", ctypes.c_void_p),
        ("q_len", ctypes.c_void_p),
        ("q_start", ctypes.c_void_p),
        ("cold_tile_tokens", ctypes.c_int32),
    ]


class PlanBuffers(ctypes.Structure):
    """Mirror of ``asterq_plan_buffers`` (the tables ``asterq_plan_batch`` writes)."""

    _fields_ = [
        ("cap_tiles", ctypes.c_int32),
        ("cap_units", ctypes.c_int32),
        ("cap_items", ctypes.c_int32),
        ("tiles", ctypes.c_void_p),
        ("units", ctypes.c_void_p),
        ("items", ctypes.c_void_p),
        ("combine", ctypes.c_void_p),
        ("unit_jobs", ctypes.c_void_p),
        ("workers", ctypes.c_void_p),
        ("counts", ctypes.c_void_p),
        ("scratch", ctypes.c_void_p),
    ]


class AsterqError(RuntimeError):
    """A failed ``asterq_*`` call (status and message from ``asterq_last_error``)."""

    def __init__(self, status: int, message: str):
        super().__init__(f"asterq error {status}: {message}")
        self.status = status


_lib = None


def lib_path() -> Path:
    override = os.environ.get("ASTERQ_LIB")
    return Path(override) if override else _LIB_PATH


def load() -> ctypes.CDLL:
    """Load the shared library once and declare every entry point's signature."""
    global _lib
    if _lib is not None:
        return _lib
    path = lib_path()
    if not path.exists():
        raise RuntimeError(
            f"{path} is missing: build the CUDA library first (__graft_entry__.build() or python -m asterq.build)"
        )
    lib = ctypes.CDLL(str(path))
    vp, i32, i64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64
    lib.asterq_version.restype = ctypes.c_int
    lib.asterq_version.argtypes = []
    lib.asterq_last_error.restype = ctypes.c_char_p
    lib.asterq_last_error.argtypes = []
    lib.asterq_quantize.restype = ctypes.c_int
    lib.asterq_quantize.argtypes = [vp, ctypes.c_int, i64, ctypes.c_int, i64, ctypes.c_int, ctypes.c_int, vp, vp, vp]
    lib.asterq_dequantize.restype = ctypes.c_int
    lib.asterq_dequantize.argtypes = [vp, vp, i64, ctypes.c_int, ctypes.c_int, ctypes.c_int, vp, ctypes.c_int, i64, vp]
    lib.asterq_fwht.restype = ctypes.c_int
    lib.asterq_fwht.argtypes = [vp, vp, i64, ctypes.c_int, vp]
    lib.asterq_codec_status.restype = ctypes.c_int
    lib.asterq_codec_status.argtypes = [ctypes.POINTER(ctypes.c_int32)]
    lib.asterq_decode_workspace_bytes.restype = i64
    lib.asterq_decode_workspace_bytes.argtypes = [ctypes.POINTER(DecodeParams)]
    lib.asterq_latent_decode.restype = ctypes.c_int
    lib.asterq_latent_decode.argtypes = [ctypes.POINTER(DecodeParams), vp]
    lib.asterq_latent_decode_noalloc.restype = ctypes.c_int
    lib.asterq_latent_decode_noalloc.argtypes = [ctypes.POINTER(DecodeParams), vp]
    lib.asterq_splitkv_combine.restype = ctypes.c_int
    lib.asterq_splitkv_combine.argtypes = [vp, i32, vp, i32, i32, vp, i32, vp]
    lib.asterq_splitkv_merge.restype = ctypes.c_int
    lib.asterq_splitkv_merge.argtypes = [vp, i32, vp, i32, i32, vp, vp]
    lib.asterq_splitkv_combine_ranks.restype = ctypes.c_int
    lib.asterq_splitkv_combine_ranks.argtypes = [vp, i32, i32, vp, i32, vp, i32, vp]
    lib.asterq_mailbox_bytes.restype = i64
    lib.asterq_mailbox_bytes.argtypes = [i32, i32, i32]
    lib.asterq_mailbox_create.restype = ctypes.c_int
    lib.asterq_mailbox_create.argtypes = [i64, ctypes.POINTER(ctypes.c_void_p), vp]
    lib.asterq_mailbox_open.restype = ctypes.c_int
    lib.asterq_mailbox_open.argtypes = [vp, ctypes.POINTER(ctypes.c_void_p)]
    lib.asterq_mailbox_close.restype = ctypes.c_int
    lib.asterq_mailbox_close.argtypes = [vp]
    lib.asterq_mailbox_destroy.restype = ctypes.c_int
    lib.asterq_mailbox_destroy.argtypes = [vp]
    lib.asterq_cp_merge_push.restype = ctypes.c_int
    lib.asterq_cp_merge_push.argtypes = [vp, i32, vp, i32, i32, vp, i32, i32, vp]
    lib.asterq_cp_combine_wait.restype = ctypes.c_int
    lib.asterq_cp_combine_wait.argtypes = [vp, i32, i32, vp, i32, vp, i32, i64, vp, vp]
    lib.asterq_plan_scratch_bytes.restype = i64
    lib.asterq_plan_scratch_bytes.argtypes = [ctypes.POINTER(BatchDesc), i32, i32, i32]
    lib.asterq_plan_batch.restype = ctypes.c_int
    lib.asterq_plan_batch.argtypes = [ctypes.POINTER(BatchDesc), ctypes.POINTER(PlanBuffers), vp]
    lib.asterq_batch_append.restype = ctypes.c_int
    lib.asterq_batch_append.argtypes = [ctypes.POINTER(BatchDesc), vp, vp, vp, i64, vp, vp, i64, vp, vp]
    _lib = lib
    return lib


def check(status: int) -> None:
    if status != ASTERQ_OK:
        msg = load().asterq_last_error().decode(errors="replace")
        if status in (ASTERQ_ERR_INVALID_ARGUMENT, ASTERQ_ERR_MISALIGNED, ASTERQ_ERR_WORKSPACE):
            raise ValueError(f"asterq error {status}: {msg}")
        raise AsterqError(status, msg)


def ptr(t) -> int | None:
    """Device pointer of a torch tensor (None for None)."""
    return None if t is None else t.data_ptr()


def stream_handle(device=None) -> int:
    import torch

    return torch.cuda.current_stream(device).cuda_stream
