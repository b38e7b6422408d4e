"""Projections of the decode step: ``m3_gemv_bf16`` at batch 1, ``m3_gemm_bf16`` up to 256 rows.

At batch 1 (`train.generate`) each projection of `model.lm_decode_step` (``model.py:244-296``)
is a stream of its bf16 weight; `small_proj` reads it near HBM speed and folds in the
elementwise work next to it: the RMS norm before in_proj and fc1, ``value * silu(gate)``
before fc2, and the residual add after out_proj and fc2.  The kernel accepts up to 8 rows,
but from 2 rows on cuBLAS is faster (measured), so the model uses it for batch 1 only.
"""

from __future__ import annotations

from typing import Optional

import torch

from . import _capi as C
from . import _tensors as T

MAX_ROWS = 1  # rows the model routes here (the kernel itself takes up to 8)
_WS = {}  # device index -> (scratch fp32, tickets int32); one stream per device at a time


def _workspace(dev: torch.device, floats: int, tickets: int):
    key = dev.index if dev.index is not None else torch.cuda.current_device()
    ws = _WS.get(key)
    if ws is None or ws[0].numel() < floats or ws[1].numel() < tickets:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("small_proj: run the step once before capturing it (workspace growth)")
        f = max(floats, ws[0].numel() if ws else 0)
        t = max(tickets, ws[1].numel() if ws else 0)
        ws = (torch.empty(f, dtype=torch.float32, device=dev), torch.zeros(t, dtype=torch.int32, device=dev))
        _WS[key] = ws
    return ws


def eligible(x: torch.Tensor, w: torch.Tensor) -> bool:
    return (x.dim() == 2 and x.shape[0] <= MAX_ROWS and x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16
            and w.shape[1] % 8 == 0 and w.stride(1) == 1 and w.stride(0) % 8 == 0 and x.stride(1) == 1)


def small_proj(x: torch.Tensor, w: torch.Tensor, *, norm_w: Optional[torch.Tensor] = None, eps: float = 1e-5,
               silu_gate: bool = False, residual: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``f(x) @ w (+ residual)`` for ``x (m, k)`` (``(m, 2k)`` with ``silu_gate``), ``w (k, n)``,
    all bf16, ``m <= 8``; f = RMS norm times ``norm_w`` if given, ``value * silu(gate)`` if
    ``silu_gate``.  Returns a new ``(m, n)`` bf16 tensor."""
    m = x.shape[0]
    k, n = w.shape
    if residual is not None and (residual.dtype != torch.bfloat16 or residual.stride(1) != 1):
        residual = residual.to(torch.bfloat16).contiguous()
    out = torch.empty(m, n, dtype=torch.bfloat16, device=x.device)
    lib = C.lib()
    scratch, tickets = _workspace(x.device, lib.m3_gemv_scratch_floats(m, k, n), (n + 255) // 256)
    a = C.M3GemvArgs()
    a.m, a.k, a.n = m, k, n
    a.x_mode = 2 if silu_gate else (1 if norm_w is not None else 0)
    a.x, a.x_ld = T.ptr(x), x.stride(0)
    nw = T.f32dense(norm_w) if norm_w is not None else None
    a.norm_w, a.eps = T.ptr(nw), eps
    a.w, a.w_ld = T.ptr(w), w.stride(0)
    if residual is not None:
        a.residual, a.r_ld = T.ptr(residual), residual.stride(0)
    a.out, a.out_ld = T.ptr(out), out.stride(0)
    a.scratch, a.tickets = T.ptr(scratch), T.ptr(tickets)
    C.check(lib.m3_gemv_bf16(a, T.stream_handle(x.device)))
    return out


def gated_act(h: torch.Tensor) -> torch.Tensor:
    """``value * silu(gate)`` of ``h (m, 2k)`` (``model.py:125-137``) in one kernel for bf16
    rows (``m3_gated_act_bf16``; the same two roundings as the torch ops); the torch ops
    otherwise."""
    k = h.shape[-1] // 2
    if (h.dim() == 2 and h.shape[-1] == 2 * k and h.dtype == torch.bfloat16 and h.is_cuda and h.stride(1) == 1
            and k % 8 == 0 and h.stride(0) % 8 == 0 and h.data_ptr() % 16 == 0):
        out = torch.empty(h.shape[0], k, dtype=h.dtype, device=h.device)
        C.check(C.lib().m3_gated_act_bf16(T.ptr(h), h.stride(0), T.ptr(out), out.stride(0), h.shape[0], k,
                                          T.stream_handle(h.device)))
        return out
    value, gate = h.chunk(2, dim=-1)
    return value * torch.nn.functional.silu(gate)


GEMM_MAX_ROWS = 256


def gemm_eligible(x: torch.Tensor, w: torch.Tensor, w_kmajor: bool = False) -> bool:
    """Whether `gemm` takes ``x (m, k) @ w`` (bf16, m <= 256, k % 64 == 0, n % 8 == 0,
    16-byte rows).  ``w`` is ``(k, n)`` with n contiguous, or with ``w_kmajor`` a ``(k, n)``
    view of an ``(n, k)`` tensor with k contiguous (``embed.t()``)."""
    if not (x.is_cuda and x.dim() == 2 and w.dim() == 2 and x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16):
        return False
    m, k = x.shape
    n = w.shape[1]
    if not (0 < m <= GEMM_MAX_ROWS and w.shape[0] == k and k % 64 == 0 and n % 8 == 0 and x.stride(1) == 1):
        return False
    ldw = w.stride(1) if w_kmajor else w.stride(0)
    inner = w.stride(0) if w_kmajor else w.stride(1)
    return (inner == 1 and ldw % 8 == 0 and x.stride(0) % 8 == 0 and x.data_ptr() % 16 == 0
            and w.data_ptr() % 16 == 0)


def gemm(x: torch.Tensor, w: torch.Tensor, *, residual: Optional[torch.Tensor] = None, w_kmajor: bool = False,
         out: Optional[torch.Tensor] = None, ksplit: int = 0) -> torch.Tensor:
    """``[residual +] x @ w`` for bf16 ``x (m, k)``, ``m <= 256`` (`gemm_eligible`), through the
    skinny tcgen05 GEMM (``m3_gemm_bf16``): fp32 accumulation, one bf16 rounding, the same
    result every call.  ``w_kmajor``: ``w`` is ``embed.t()``-like (k contiguous)."""
    m, k = x.shape
    n = w.shape[1]
    if residual is not None and (residual.dtype != torch.bfloat16 or residual.stride(1) != 1
                                 or residual.stride(0) % 4 or residual.data_ptr() % 8):
        residual = residual.to(torch.bfloat16).contiguous()
    if out is None:
        out = torch.empty(m, n, dtype=torch.bfloat16, device=x.device)
    a = C.M3GemmArgs()
    a.m, a.n, a.k, a.w_kmajor, a.ksplit = m, n, k, int(w_kmajor), ksplit
    a.a, a.lda = T.ptr(x), x.stride(0)
    a.w, a.ldw = T.ptr(w), (w.stride(1) if w_kmajor else w.stride(0))
    if residual is not None:
        a.residual, a.ldr = T.ptr(residual), residual.stride(0)
    a.out, a.ldo = T.ptr(out), out.stride(0)
    C.check(C.lib().m3_gemm_bf16(a, T.stream_handle(x.device)))
    return out
