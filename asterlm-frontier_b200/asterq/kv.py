"""Drop-in for AsterLM's ``quantization/kv.py`` backed by the sm_100a kernels.

Same names, arguments, result types and error behaviour as the reference
(src/asterlm/quantization/kv.py); the integer schemes run on the GPU through
the C ABI and are bit-identical to the reference's CPU float32 arithmetic:

* ``normalized_fwht``   kv.py:13-32   -> ``asterq_fwht``
* ``quantize_tensor``   kv.py:76-118  -> ``asterq_quantize``
* ``dequantize_tensor`` kv.py:121-134 -> ``asterq_dequantize``

The ``bfloat16`` / ``float8`` schemes are plain dtype casts in the reference
(kv.py:82-89) and stay casts here.  Integer schemes need CUDA tensors: there is
no CPU path.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import _lib

_SCHEME_IDS = {
    "hadamard_int4": _lib.SCHEME_HADAMARD_INT4,
    "int4": _lib.SCHEME_INT4,
    "int8": _lib.SCHEME_INT8,
}
_DTYPE_IDS = {torch.float32: _lib.DTYPE_F32, torch.bfloat16: _lib.DTYPE_BF16, torch.float16: _lib.DTYPE_F16}


def _next_power_of_two(value: int) -> int:
    """kv.py:9-10."""
    return 1 if value <= 1 else 1 << (value - 1).bit_length()


def _require_cuda(t: torch.Tensor, what: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{what}: asterq kernels need CUDA tensors (got device {t.device}); there is no CPU path")


@dataclass(slots=True)
class QuantizedTensor:
    """Same fields as the reference record (kv.py:58-73)."""

    data: torch.Tensor
    scale: torch.Tensor | None
    original_shape: tuple[int, ...]
    padded_dim: int
    group_size: int
    scheme: str
    source_dtype: torch.dtype

    @property
    def num_bytes(self) -> int:
        total = self.data.numel() * self.data.element_size()
        if self.scale is not None:
            total += self.scale.numel() * self.scale.element_size()
        return int(total)


def normalized_fwht(x: torch.Tensor) -> torch.Tensor:
    """Normalized Walsh-Hadamard transform over the last dimension (kv.py:13-32).

    Bit-identical to the reference for float32 input.  Other floating dtypes
    are transformed in float32 and rounded back once (the reference would
    round after every butterfly stage in that dtype).
    """
    n = x.shape[-1]
    if n & (n - 1):
        raise ValueError("FWHT length must be a power of two")
    _require_cuda(x, "normalized_fwht")
    src = x.to(torch.float32).reshape(-1, n).contiguous()
    out = torch.empty_like(src)
    lib = _lib.load()
    _lib.check(lib.asterq_fwht(src.data_ptr(), out.data_ptr(), src.shape[0], n, _lib.stream_handle(x.device)))
    return out.reshape(x.shape).to(x.dtype)


def _rows_view(x: torch.Tensor) -> tuple[torch.Tensor, int]:
    """[N, dim] view with unit stride on the last axis (copies only if needed)."""
    if x.dtype not in _DTYPE_IDS:
        x = x.float()
    dim = x.shape[-1]
    flat = x.reshape(-1, dim) if x.dim() != 2 else x
    if flat.stride(-1) != 1 or (flat.shape[0] > 1 and flat.stride(0) < dim):
        flat = flat.contiguous()
    stride = flat.stride(0) if flat.shape[0] > 1 else dim
    if (flat.data_ptr() % 16) or ((stride * flat.element_size()) % 16):
        flat = flat.contiguous()
        stride = dim
    return flat, stride


def quantize_tensor(x: torch.Tensor, scheme: str, *, group_size: int = 64) -> QuantizedTensor:
    """Quantize along the last dimension (kv.py:76-118)."""
    if scheme == "bfloat16":
        data = x.to(torch.bfloat16)
        return QuantizedTensor(data, None, tuple(x.shape), x.shape[-1], group_size, scheme, x.dtype)
    if scheme == "float8":
        if not hasattr(torch, "float8_e4m3fn"):
            raise RuntimeError("this PyTorch build does not expose float8_e4m3fn")
        data = x.to(torch.float8_e4m3fn)
        return QuantizedTensor(data, None, tuple(x.shape), x.shape[-1], group_size, scheme, x.dtype)
    if scheme not in _SCHEME_IDS:
        raise ValueError(f"unsupported quantization scheme: {scheme}")
    if group_size <= 0:
        raise ValueError("group_size must be positive")
    _require_cuda(x, "quantize_tensor")
    original_shape = tuple(x.shape)
    dim = x.shape[-1]
    if scheme == "hadamard_int4":
        padded_dim = _next_power_of_two(dim)
        width = math.ceil(padded_dim / group_size) * group_size
    else:
        padded_dim = dim
        width = math.ceil(dim / group_size) * group_size
    lead = original_shape[:-1]
    if scheme == "int8":
        codes = torch.empty(*lead, width, dtype=torch.int8, device=x.device)
    else:
        codes = torch.empty(*lead, width // 2, dtype=torch.uint8, device=x.device)
    scales = torch.empty(*lead, width // group_size, 1, dtype=torch.float16, device=x.device)
    n = int(math.prod(lead))
    if n:
        flat, stride = _rows_view(x)
        lib = _lib.load()
        _lib.check(
            lib.asterq_quantize(
                flat.data_ptr(),
                _DTYPE_IDS[flat.dtype],
                n,
                dim,
                stride,
                _SCHEME_IDS[scheme],
                group_size,
                codes.data_ptr(),
                scales.data_ptr(),
                _lib.stream_handle(x.device),
            )
        )
    return QuantizedTensor(
        data=codes,
        scale=scales,
        original_shape=original_shape,
        padded_dim=padded_dim,
        group_size=group_size,
        scheme=scheme,
        source_dtype=x.dtype,
    )


def dequantize_tensor(q: QuantizedTensor, *, dtype: torch.dtype | None = None) -> torch.Tensor:
    """Inverse of ``quantize_tensor`` (kv.py:121-134)."""
    target_dtype = q.source_dtype if dtype is None else dtype
    if q.scheme in {"bfloat16", "float8"}:
        return q.data.to(target_dtype).reshape(q.original_shape)
    if q.scale is None:
        raise RuntimeError("integer quantized tensor is missing scales")
    if q.scheme not in _SCHEME_IDS:
        raise ValueError(f"unsupported quantization scheme: {q.scheme}")
    _require_cuda(q.data, "dequantize_tensor")
    dim = q.original_shape[-1]
    lead = q.original_shape[:-1]
    kernel_dtype = target_dtype if target_dtype in _DTYPE_IDS else torch.float32
    out = torch.empty(*lead, dim, dtype=kernel_dtype, device=q.data.device)
    n = int(math.prod(lead))
    if n:
        codes = q.data.reshape(n, -1).contiguous()
        scales = q.scale.reshape(n, -1).contiguous()
        lib = _lib.load()
        _lib.check(
            lib.asterq_dequantize(
                codes.data_ptr(),
                scales.data_ptr(),
                n,
                dim,
                _SCHEME_IDS[q.scheme],
                q.group_size,
                out.data_ptr(),
                _DTYPE_IDS[kernel_dtype],
                dim,
                _lib.stream_handle(q.data.device),
            )
        )
    return out.to(target_dtype).reshape(q.original_shape)
