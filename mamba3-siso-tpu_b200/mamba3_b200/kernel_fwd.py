"""Forward chunked scan through libm3siso.so.

`siso_forward` keeps the signature and return convention of
``mamba3_pallas/kernel_fwd.py:204-388`` (preprocessed boundary).  `siso_forward_raw` is
the fused boundary of ``siso.py:154-216``: raw in_proj streams in, preprocessing done
inside the kernel.
"""

from __future__ import annotations

import ctypes

from typing import NamedTuple, Optional

import torch

from . import _capi as C
from . import _tensors as T
from . import layout as L


class ForwardResiduals(NamedTuple):
    """``kernel_fwd.py:41-52``: ybar ``(B,H,L,P)`` f32, chunk_states ``(B,H,nc,P,N)``."""

    ybar: torch.Tensor
    chunk_states: torch.Tensor


def _kernel_code(kernel: str) -> int:
    """``"auto"`` (tensor cores where they apply), ``"generic"``, ``"tensorcore"`` or
    ``"tensorcore_v1"`` (the two-sequence tensor-core forward, kept for comparison)."""
    codes = {"auto": C.M3_KERNEL_AUTO, "generic": C.M3_KERNEL_GENERIC, "tensorcore": C.M3_KERNEL_TENSORCORE,
             "tensorcore_v1": C.M3_KERNEL_TENSORCORE_V1}
    if kernel not in codes:
        raise ValueError(f"kernel must be one of {sorted(codes)}, got {kernel!r}")
    return codes[kernel]


def _dims(q, v, n_angles, chunk) -> C.M3Dims:
    b, l, n = q.shape
    return C.M3Dims(b, l, v.shape[1], n, v.shape[3], n_angles, chunk)


def _check_shapes(q, k, v, z):
    if q.dim() != 3 or q.shape != k.shape:
        raise ValueError(f"q {tuple(q.shape)} and k {tuple(k.shape)} must match and be (B, L, N)")
    b, l, _ = q.shape
    if v.dim() != 4 or v.shape[0] != b or v.shape[2] != l:
        raise ValueError(f"unexpected v shape {tuple(v.shape)}")
    if z is not None and z.shape != v.shape:
        raise ValueError(f"z {tuple(z.shape)} must match v {tuple(v.shape)}")


def siso_forward(q, k, v, adt, gamma, scale, phi, q_bias, k_bias, d_skip=None, z=None,
                 seed_ssm=None, seed_k=None, seed_v=None, seed_coef=None, chunk: int = 128,
                 dtype_policy: str = "bf16", save_residuals: bool = False, out_y=None, kernel: str = "auto",
                 interpret=False, device_kind=None):
    """Chunked forward at the preprocessed boundary.  ``interpret`` / ``device_kind`` are
    the reference's TPU options (Pallas interpret mode, TPU generation); they are accepted
    and have no effect here.

    Returns ``(y, final_ssm, final_k, final_v)`` and `ForwardResiduals` when
    ``save_residuals`` (``kernel_fwd.py:245-248``).  ``final_k`` is rotated but unscaled.
    """
    L.validate_chunk(chunk)
    T.require_cuda(q, k, v)
    _check_shapes(q, k, v, z)
    b, l, n = q.shape
    h, p = v.shape[1], v.shape[3]
    nr = phi.shape[-1]
    nc = L.num_chunks(l, chunk)
    for name, t in (("adt", adt), ("gamma", gamma), ("scale", scale)):
        if tuple(t.shape) != (b, h, l):
            raise ValueError(f"{name} must be (B, H, L) = {(b, h, l)}, got {tuple(t.shape)}")
    if tuple(phi.shape) != (b, h, l, nr):
        raise ValueError(f"phi must be (B, H, L, Nr) = {(b, h, l, nr)}, got {tuple(phi.shape)}")
    seeds = (seed_ssm, seed_k, seed_v, seed_coef)
    if any(s is not None for s in seeds) and not all(s is not None for s in seeds):
        raise ValueError("seed_ssm, seed_k, seed_v and seed_coef must be given together")
    dt_io = v.dtype if v.dtype in (torch.bfloat16, torch.float32) else torch.float32
    q, k, v, z = (T.inner_contig(t, dt_io) for t in (q, k, v, z))
    adt, gamma, scale, phi = (T.f32dense(t) for t in (adt, gamma, scale, phi))
    qb, kb, dsk = T.f32dense(q_bias), T.f32dense(k_bias), T.f32dense(d_skip)
    s_ssm, s_k, s_v, s_c = (T.f32dense(t) for t in seeds)
    dev = q.device
    y = out_y if out_y is not None else torch.empty(b, h, l, p, dtype=dt_io, device=dev)
    fs = torch.empty(b, h, p, n, dtype=torch.float32, device=dev)
    fk = torch.empty(b, h, n, dtype=torch.float32, device=dev)
    fv = torch.empty(b, h, p, dtype=torch.float32, device=dev)
    ybar = states = None
    if save_residuals:
        ybar = torch.empty(b, h, l, p, dtype=torch.float32, device=dev)
        sdt = L.policy(dtype_policy).saved_state
        states = torch.empty(b, h, nc, p, n, dtype=sdt, device=dev)
    a = C.M3FwdArgs()
    a.dims = _dims(q, v, nr, chunk)
    a.io_dtype = T.io_dtype(dt_io)
    a.policy = T.policy_code(dtype_policy)
    a.raw = 0
    a.q, a.k, a.v, a.z = T.ptr(q), T.ptr(k), T.ptr(v), T.ptr(z)
    a.q_st, a.k_st, a.v_st = T.st_bln(q), T.st_bln(k), T.st_bhlp(v)
    if z is not None:
        a.z_st = T.st_bhlp(z)
    a.adt, a.gamma, a.scale, a.phi = T.ptr(adt), T.ptr(gamma), T.ptr(scale), T.ptr(phi)
    a.q_bias, a.k_bias, a.d_skip = T.ptr(qb), T.ptr(kb), T.ptr(dsk)
    a.seed_ssm, a.seed_k, a.seed_v, a.seed_coef = T.ptr(s_ssm), T.ptr(s_k), T.ptr(s_v), T.ptr(s_c)
    a.y, a.y_st = T.ptr(y), T.st_bhlp(y)
    a.final_ssm, a.final_k, a.final_v = T.ptr(fs), T.ptr(fk), T.ptr(fv)
    if save_residuals:
        a.ybar, a.chunk_states = T.ptr(ybar), T.ptr(states)
        a.chunk_states_dtype = T.io_dtype(states.dtype)
    a.kernel = _kernel_code(kernel)
    C.check(C.lib().m3_siso_fwd(a, T.stream_handle(dev)))
    if save_residuals:
        return y, fs, fk, fv, ForwardResiduals(ybar=ybar, chunk_states=states)
    return y, fs, fk, fv


def siso_forward_raw(q, k, v, dt_raw, a_raw, trap_raw, angles, dt_bias, q_bias, k_bias,
                     d_skip=None, z=None, seed_ssm=None, seed_k=None, seed_v=None, seed_phi=None,
                     a_floor: float = 1e-4, chunk: int = 128, dtype_policy: str = "bf16",
                     y_out: Optional[torch.Tensor] = None, kernel: str = "auto",
                     bwd_states: Optional[torch.Tensor] = None, return_saved: bool = False,
                     states_only: bool = False):
    """Fused boundary: raw ``(B, L, H)`` dt/A/trap streams and head-shared ``(B, L, Nr)``
    angles (all may be strided views of an in_proj output).  Returns
    ``(y, final_ssm, final_k, final_v, final_phi)``.  ``y_out`` may be a strided
    ``(B, H, L, P)`` view to write into (e.g. a permuted ``(B, L, H, P)`` buffer).

    ``bwd_states``: the workspace of a later `kernel_bwd.siso_backward_raw` on the same
    inputs; when this forward runs on tensor cores it stores the chunk-start states there
    and that backward can pass ``states_ready=True``.  ``return_saved`` appends whether it
    did.  ``states_only``: no y (returned as None), only the final state -- the states-only
    variant of the tensor-core kernel; see `final_state_supported`."""
    L.validate_chunk(chunk)
    T.require_cuda(q, k, v)
    _check_shapes(q, k, v, z)
    b, l, n = q.shape
    h, p = v.shape[1], v.shape[3]
    nr = angles.shape[-1]
    L.num_chunks(l, chunk)
    seeds = (seed_ssm, seed_k, seed_v)
    if any(s is not None for s in seeds) and not all(s is not None for s in seeds):
        raise ValueError("seed_ssm, seed_k and seed_v must be given together")
    dt_io = v.dtype if v.dtype in (torch.bfloat16, torch.float32) else torch.float32
    q, k, v, z = (T.inner_contig(t, dt_io) for t in (q, k, v, z))
    dt_raw, a_raw, trap_raw, angles = (T.f32c(t) for t in (dt_raw, a_raw, trap_raw, angles))
    dtb, qb, kb, dsk = (T.f32dense(t) for t in (dt_bias, q_bias, k_bias, d_skip))
    s_ssm, s_k, s_v, s_phi = (T.f32dense(t) for t in (seed_ssm, seed_k, seed_v, seed_phi))
    dev = q.device
    y = None if states_only else (y_out if y_out is not None else torch.empty(b, h, l, p, dtype=dt_io, device=dev))
    fs = torch.empty(b, h, p, n, dtype=torch.float32, device=dev)
    fk = torch.empty(b, h, n, dtype=torch.float32, device=dev)
    fv = torch.empty(b, h, p, dtype=torch.float32, device=dev)
    fphi = torch.empty(b, h, nr, dtype=torch.float32, device=dev)
    a = C.M3FwdArgs()
    a.dims = _dims(q, v, nr, chunk)
    a.io_dtype = T.io_dtype(dt_io)
    a.policy = T.policy_code(dtype_policy)
    a.raw = 1
    a.a_floor = a_floor
    a.q, a.k, a.v, a.z = T.ptr(q), T.ptr(k), T.ptr(v), T.ptr(z)
    a.q_st, a.k_st, a.v_st = T.st_bln(q), T.st_bln(k), T.st_bhlp(v)
    if z is not None:
        a.z_st = T.st_bhlp(z)
    a.dt_raw, a.a_raw, a.trap_raw = T.ptr(dt_raw), T.ptr(a_raw), T.ptr(trap_raw)
    if dt_raw.stride() != a_raw.stride() or dt_raw.stride() != trap_raw.stride():
        dt_raw, a_raw, trap_raw = dt_raw.contiguous(), a_raw.contiguous(), trap_raw.contiguous()
        a.dt_raw, a.a_raw, a.trap_raw = T.ptr(dt_raw), T.ptr(a_raw), T.ptr(trap_raw)
    a.raw_st = T.st_blh(dt_raw)
    a.angles, a.ang_st, a.dt_bias = T.ptr(angles), T.st_bln(angles), T.ptr(dtb)
    a.q_bias, a.k_bias, a.d_skip = T.ptr(qb), T.ptr(kb), T.ptr(dsk)
    a.seed_ssm, a.seed_k, a.seed_v, a.seed_phi = T.ptr(s_ssm), T.ptr(s_k), T.ptr(s_v), T.ptr(s_phi)
    if y is not None:
        a.y, a.y_st = T.ptr(y), T.st_bhlp(y)
    a.final_ssm, a.final_k, a.final_v, a.final_phi = T.ptr(fs), T.ptr(fk), T.ptr(fv), T.ptr(fphi)
    a.kernel = _kernel_code(kernel)
    # head-shared rotary rates, computed once per (b, t, angle) by the tensor-core forward
    wsz = C.lib().m3_siso_fwd_workspace_size(ctypes.byref(a.dims))
    fws = torch.empty(wsz, dtype=torch.uint8, device=dev)
    a.fwd_workspace, a.fwd_workspace_bytes = T.ptr(fws), wsz
    saved = False
    if bwd_states is not None and C.lib().m3_siso_fwd_saves_states(a):
        a.bwd_states, a.bwd_states_bytes = T.ptr(bwd_states), bwd_states.numel() * bwd_states.element_size()
        saved = True
    C.check(C.lib().m3_siso_fwd(a, T.stream_handle(dev)))
    if return_saved:
        return (y, fs, fk, fv, fphi), saved
    return y, fs, fk, fv, fphi


def final_state_supported(q, v, angles, chunk: int, dtype_policy: str = "bf16") -> bool:
    """Whether `siso_forward_raw(..., states_only=True)` has a kernel for these shapes
    (the tensor-core ones: bf16 I/O and policy, N = 128, P = 64, chunk % 128 == 0)."""
    n, p, nr = q.shape[-1], v.shape[-1], angles.shape[-1]
    return (v.dtype == torch.bfloat16 and T.policy_code(dtype_policy) == C.M3_POLICY_BF16 and n == 128
            and p == 64 and chunk % 128 == 0 and nr % 8 == 0 and nr <= 64 and q.shape[1] % 128 == 0)
