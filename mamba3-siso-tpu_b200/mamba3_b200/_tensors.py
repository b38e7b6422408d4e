"""Tensor -> C-ABI plumbing shared by the kernel wrappers."""

from __future__ import annotations

import weakref

import torch

from . import _capi as C


def ptr(t):
    return None if t is None else t.data_ptr()


def stream_handle(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("the Mamba-3 SISO kernels run on CUDA tensors only (no CPU path)")


def io_dtype(dt: torch.dtype) -> int:
    if dt == torch.bfloat16:
        return C.M3_DTYPE_BF16
    if dt == torch.float32:
        return C.M3_DTYPE_F32
    raise ValueError(f"unsupported dtype {dt}; want bfloat16 or float32")


def policy_code(name) -> int:
    key = str(name).strip().lower()  # a name or a layout.DtypePolicy
    if key in ("bf16", "bfloat16", "default"):
        return C.M3_POLICY_BF16
    if key in ("f32", "fp32", "float32", "highest"):
        return C.M3_POLICY_F32
    raise ValueError(f"Unknown dtype policy {name!r}; want 'bf16' or 'f32'")


def f32c(t):
    """fp32, innermost-contiguous (outer strides are passed through)."""
    if t is None:
        return None
    if t.dtype != torch.float32:
        t = t.float()
    if t.dim() and t.stride(-1) != 1:
        t = t.contiguous()
    return t


_F32_CACHE = {}  # id(tensor) -> (weakref to it, its version, fp32 copy); tensors compare elementwise, so no WeakKeyDictionary


def f32dense(t):
    """fp32, dense.  Small tensors that need a conversion (per-head parameters held in bf16)
    are converted once and reused while their version is unchanged, so a decode step does
    not re-convert every layer's biases on every token."""
    if t is None:
        return None
    if t.dtype == torch.float32 and t.is_contiguous():
        return t
    if t.numel() <= (1 << 16) and not t.requires_grad:
        key = id(t)
        hit = _F32_CACHE.get(key)
        if hit is not None and hit[0]() is t and hit[1] == t._version:
            return hit[2]
        c = t.float().contiguous()
        if not (t.is_cuda and torch.cuda.is_current_stream_capturing()):
            _F32_CACHE[key] = (weakref.ref(t, lambda _r, k=key: _F32_CACHE.pop(k, None)), t._version, c)
        return c
    return t.float().contiguous()


def inner_contig(t, dtype):
    if t is None:
        return None
    if t.dtype != dtype:
        t = t.to(dtype)
    if t.stride(-1) != 1:
        t = t.contiguous()
    return t


def st_bln(t) -> C.M3Strides:
    """(B, L, X) with contiguous X."""
    return C.M3Strides(t.stride(0), 0, t.stride(1))


def st_bhlp(t) -> C.M3Strides:
    return C.M3Strides(t.stride(0), t.stride(1), t.stride(2))


def st_blh(t) -> C.M3Strides:
    return C.M3Strides(t.stride(0), t.stride(2), t.stride(1))
