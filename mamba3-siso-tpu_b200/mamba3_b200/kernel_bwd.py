"""Backward through libm3siso.so.

`siso_backward` mirrors ``mamba3_pallas/kernel_bwd.py:534-669`` (kernel + epilogue) at
the preprocessed boundary and returns the same `SISOGrads`.  The forward residuals
(``ybar``, ``chunk_states``) are accepted for signature compatibility but not read: the
kernel recomputes the chunk states (and ybar) itself into a workspace.
`siso_backward_raw` differentiates the fused raw boundary, preprocessing included.
"""

from __future__ import annotations

from typing import NamedTuple, Optional

import torch

from . import _capi as C
from . import _tensors as T
from . import layout as L


class SISOGrads(NamedTuple):
    """``kernel_bwd.py:514-531``."""

    dq: torch.Tensor
    dk: torch.Tensor
    dv: torch.Tensor
    dadt: torch.Tensor
    dgamma: torch.Tensor
    dscale: torch.Tensor
    dphi: torch.Tensor
    dq_bias: torch.Tensor
    dk_bias: torch.Tensor
    dd_skip: Optional[torch.Tensor]
    dz: Optional[torch.Tensor]
    dseed_ssm: Optional[torch.Tensor]
    dseed_k: Optional[torch.Tensor]
    dseed_v: Optional[torch.Tensor]
    dseed_coef: Optional[torch.Tensor]


class RawGrads(NamedTuple):
    """Gradients of the fused raw boundary (the inputs of ``siso.siso_segment``)."""

    dq: torch.Tensor
    dk: torch.Tensor
    dv: torch.Tensor
    dz: Optional[torch.Tensor]
    ddt_raw: torch.Tensor      # (B, L, H)
    da_raw: torch.Tensor       # (B, L, H)
    dtrap_raw: torch.Tensor    # (B, L, H)
    dangles: torch.Tensor      # (B, L, Nr)
    ddt_bias: torch.Tensor
    dq_bias: torch.Tensor
    dk_bias: torch.Tensor
    dd_skip: Optional[torch.Tensor]
    dseed_ssm: Optional[torch.Tensor]
    dseed_k: Optional[torch.Tensor]
    dseed_v: Optional[torch.Tensor]
    dseed_phi: Optional[torch.Tensor]


def workspace_bytes(batch, seqlen, nheads, state_dim, headdim, n_angles, chunk) -> int:
    d = C.M3Dims(batch, seqlen, nheads, state_dim, headdim, n_angles, chunk)
    return int(C.lib().m3_siso_bwd_workspace_size(d))


def _workspace(dims: C.M3Dims, device, workspace=None):
    need = int(C.lib().m3_siso_bwd_workspace_size(dims))
    if workspace is not None and workspace.numel() * workspace.element_size() >= need:
        return workspace, need
    return torch.empty(need, dtype=torch.uint8, device=device), need


def _common(a, q, k, v, z, dy, dt_io):
    a.q, a.k, a.v, a.z, a.dy = T.ptr(q), T.ptr(k), T.ptr(v), T.ptr(z), T.ptr(dy)
    a.q_st, a.k_st, a.v_st, a.dy_st = T.st_bln(q), T.st_bln(k), T.st_bhlp(v), T.st_bhlp(dy)
    if z is not None:
        a.z_st = T.st_bhlp(z)
    a.io_dtype = T.io_dtype(dt_io)


def siso_backward(dy, q, k, v, adt, gamma, scale, phi, q_bias, k_bias, ybar=None, chunk_states=None,
                  d_skip=None, z=None, seed_ssm=None, seed_k=None, seed_v=None, seed_coef=None,
                  dfinal_ssm=None, dfinal_k=None, dfinal_v=None, chunk: int = 128,
                  dtype_policy: str = "bf16", workspace=None, kernel: str = "auto", interpret=False,
                  device_kind=None) -> SISOGrads:
    L.validate_chunk(chunk)
    T.require_cuda(q, k, v, dy)
    b, l, n = q.shape
    h, p = v.shape[1], v.shape[3]
    nr = phi.shape[-1]
    dt_io = v.dtype if v.dtype in (torch.bfloat16, torch.float32) else torch.float32
    q, k, v, z, dy = (T.inner_contig(t, dt_io) for t in (q, k, v, z, dy))
    adt, gamma, scale, phi = (T.f32dense(t) for t in (adt, gamma, scale, phi))
    qb, kb, dsk = T.f32dense(q_bias), T.f32dense(k_bias), T.f32dense(d_skip)
    s_ssm, s_k, s_v, s_c = (T.f32dense(t) for t in (seed_ssm, seed_k, seed_v, seed_coef))
    dfs, dfk, dfv = (T.f32dense(t) for t in (dfinal_ssm, dfinal_k, dfinal_v))
    dev, f32 = q.device, torch.float32
    dq = torch.empty(b, l, n, dtype=f32, device=dev)
    dk = torch.empty(b, l, n, dtype=f32, device=dev)
    dv = torch.empty(b, h, l, p, dtype=f32, device=dev)
    dz = torch.empty(b, h, l, p, dtype=f32, device=dev) if z is not None else None
    dadt = torch.empty(b, h, l, dtype=f32, device=dev)
    dgamma = torch.empty_like(dadt)
    dscale = torch.empty_like(dadt)
    dphi = torch.empty(b, h, l, nr, dtype=f32, device=dev)
    dqb = torch.empty(h, n, dtype=f32, device=dev)
    dkb = torch.empty(h, n, dtype=f32, device=dev)
    ddsk = torch.empty(h, dtype=f32, device=dev) if d_skip is not None else None
    has_seed = seed_ssm is not None
    dss = torch.empty(b, h, p, n, dtype=f32, device=dev) if has_seed else None
    dsk_ = torch.empty(b, h, n, dtype=f32, device=dev) if has_seed else None
    dsv = torch.empty(b, h, p, dtype=f32, device=dev) if has_seed else None
    dsc = torch.empty(b, h, dtype=f32, device=dev) if has_seed else None
    a = C.M3BwdArgs()
    a.dims = C.M3Dims(b, l, h, n, p, nr, chunk)
    _common(a, q, k, v, z, dy, dt_io)
    a.policy = T.policy_code(dtype_policy)
    a.raw = 0
    a.adt, a.gamma, a.scale, a.phi = T.ptr(adt), T.ptr(gamma), T.ptr(scale), T.ptr(phi)
    a.q_bias, a.k_bias, a.d_skip = T.ptr(qb), T.ptr(kb), T.ptr(dsk)
    a.seed_ssm, a.seed_k, a.seed_v, a.seed_coef = T.ptr(s_ssm), T.ptr(s_k), T.ptr(s_v), T.ptr(s_c)
    a.dfinal_ssm, a.dfinal_k, a.dfinal_v = T.ptr(dfs), T.ptr(dfk), T.ptr(dfv)
    a.dq, a.dk, a.dv, a.dz = T.ptr(dq), T.ptr(dk), T.ptr(dv), T.ptr(dz)
    a.dadt, a.dgamma, a.dscale, a.dphi = T.ptr(dadt), T.ptr(dgamma), T.ptr(dscale), T.ptr(dphi)
    a.dq_bias, a.dk_bias, a.dd_skip = T.ptr(dqb), T.ptr(dkb), T.ptr(ddsk)
    a.dseed_ssm, a.dseed_k, a.dseed_v, a.dseed_coef = T.ptr(dss), T.ptr(dsk_), T.ptr(dsv), T.ptr(dsc)
    ws, need = _workspace(a.dims, dev, workspace)
    a.workspace, a.workspace_bytes = T.ptr(ws), need
    a.kernel = {"auto": C.M3_KERNEL_AUTO, "generic": C.M3_KERNEL_GENERIC, "tensorcore": C.M3_KERNEL_TENSORCORE}[kernel]
    C.check(C.lib().m3_siso_bwd(a, T.stream_handle(dev)))
    return SISOGrads(dq=dq, dk=dk, dv=dv, dadt=dadt, dgamma=dgamma, dscale=dscale, dphi=dphi,
                     dq_bias=dqb, dk_bias=dkb, dd_skip=ddsk, dz=dz, dseed_ssm=dss, dseed_k=dsk_,
                     dseed_v=dsv, dseed_coef=dsc)


def siso_backward_raw(dy, q, k, v, dt_raw, a_raw, trap_raw, angles, dt_bias, q_bias, k_bias,
                      d_skip=None, z=None, seed_ssm=None, seed_k=None, seed_v=None, seed_phi=None,
                      dfinal_ssm=None, dfinal_k=None, dfinal_v=None, dfinal_phi=None,
                      a_floor: float = 1e-4, chunk: int = 128, dtype_policy: str = "bf16",
                      workspace=None, kernel: str = "auto", states_ready: bool = False,
                      grad_dtype: torch.dtype = torch.float32, dv_out=None, dz_out=None) -> RawGrads:
    """Gradients of the fused raw boundary.  ``states_ready``: ``workspace`` was given as
    ``bwd_states`` to the forward on these same inputs and it saved the chunk-start states
    (``return_saved``), so the tensor-core backward skips its recompute sweep.
    ``grad_dtype`` (float32 or bfloat16): the dtype of dv and dz.  ``dv_out`` / ``dz_out``:
    ``(B, H, L, P)`` views (P contiguous, e.g. of a ``(B, L, H, P)`` buffer) to write them into."""
    L.validate_chunk(chunk)
    T.require_cuda(q, k, v, dy)
    b, l, n = q.shape
    h, p = v.shape[1], v.shape[3]
    nr = angles.shape[-1]
    dt_io = v.dtype if v.dtype in (torch.bfloat16, torch.float32) else torch.float32
    q, k, v, z, dy = (T.inner_contig(t, dt_io) for t in (q, k, v, z, dy))
    dt_raw, a_raw, trap_raw, angles = (T.f32c(t) for t in (dt_raw, a_raw, trap_raw, angles))
    if dt_raw.stride() != a_raw.stride() or dt_raw.stride() != trap_raw.stride():
        dt_raw, a_raw, trap_raw = dt_raw.contiguous(), a_raw.contiguous(), trap_raw.contiguous()
    dtb, qb, kb, dsk = (T.f32dense(t) for t in (dt_bias, q_bias, k_bias, d_skip))
    s_ssm, s_k, s_v, s_phi = (T.f32dense(t) for t in (seed_ssm, seed_k, seed_v, seed_phi))
    dfs, dfk, dfv, dfp = (T.f32dense(t) for t in (dfinal_ssm, dfinal_k, dfinal_v, dfinal_phi))
    dev, f32 = q.device, torch.float32
    dq = torch.empty(b, l, n, dtype=f32, device=dev)
    dk = torch.empty(b, l, n, dtype=f32, device=dev)
    gdt = grad_dtype if grad_dtype in (torch.float32, torch.bfloat16) else torch.float32
    dv = dv_out if dv_out is not None else torch.empty(b, h, l, p, dtype=gdt, device=dev)
    dz = (dz_out if dz_out is not None else torch.empty(b, h, l, p, dtype=gdt, device=dev)) if z is not None else None
    for t in (dv, dz):
        if t is not None and (t.dtype != gdt or t.stride(-1) != 1 or tuple(t.shape) != (b, h, l, p)):
            raise ValueError("dv_out / dz_out must be (B, H, L, P) views in grad_dtype with P contiguous")
    ddt = torch.empty(b, l, h, dtype=f32, device=dev)
    da = torch.empty_like(ddt)
    dtr = torch.empty_like(ddt)
    dang = torch.empty(b, l, nr, dtype=f32, device=dev)
    ddtb = torch.empty(h, dtype=f32, device=dev)
    dqb = torch.empty(h, n, dtype=f32, device=dev)
    dkb = torch.empty(h, n, dtype=f32, device=dev)
    ddsk = torch.empty(h, dtype=f32, device=dev) if d_skip is not None else None
    has_seed = seed_ssm is not None
    dss = torch.empty(b, h, p, n, dtype=f32, device=dev) if has_seed else None
    dsk_ = torch.empty(b, h, n, dtype=f32, device=dev) if has_seed else None
    dsv = torch.empty(b, h, p, dtype=f32, device=dev) if has_seed else None
    dsp = torch.empty(b, h, nr, dtype=f32, device=dev) if seed_phi is not None else None
    a = C.M3BwdArgs()
    a.dims = C.M3Dims(b, l, h, n, p, nr, chunk)
    _common(a, q, k, v, z, dy, dt_io)
    a.policy = T.policy_code(dtype_policy)
    a.raw = 1
    a.a_floor = a_floor
    a.dt_raw, a.a_raw, a.trap_raw, a.raw_st = T.ptr(dt_raw), T.ptr(a_raw), T.ptr(trap_raw), T.st_blh(dt_raw)
    a.angles, a.ang_st, a.dt_bias = T.ptr(angles), T.st_bln(angles), T.ptr(dtb)
    a.q_bias, a.k_bias, a.d_skip = T.ptr(qb), T.ptr(kb), T.ptr(dsk)
    a.seed_ssm, a.seed_k, a.seed_v, a.seed_phi = T.ptr(s_ssm), T.ptr(s_k), T.ptr(s_v), T.ptr(s_phi)
    a.dfinal_ssm, a.dfinal_k, a.dfinal_v, a.dfinal_phi = T.ptr(dfs), T.ptr(dfk), T.ptr(dfv), T.ptr(dfp)
    a.dq, a.dk, a.dv, a.dz = T.ptr(dq), T.ptr(dk), T.ptr(dv), T.ptr(dz)
    a.ddt_raw, a.da_raw, a.dtrap_raw, a.dangles, a.ddt_bias = T.ptr(ddt), T.ptr(da), T.ptr(dtr), T.ptr(dang), T.ptr(ddtb)
    a.dq_bias, a.dk_bias, a.dd_skip = T.ptr(dqb), T.ptr(dkb), T.ptr(ddsk)
    a.dseed_ssm, a.dseed_k, a.dseed_v, a.dseed_phi = T.ptr(dss), T.ptr(dsk_), T.ptr(dsv), T.ptr(dsp)
    a.kernel = {"auto": C.M3_KERNEL_AUTO, "generic": C.M3_KERNEL_GENERIC, "tensorcore": C.M3_KERNEL_TENSORCORE}[kernel]
    ws, need = _workspace(a.dims, dev, workspace)
    a.workspace, a.workspace_bytes = T.ptr(ws), need
    a.states_ready = 1 if (states_ready and ws is workspace) else 0
    a.grad_dtype = T.io_dtype(gdt)
    a.dv_st = T.st_bhlp(dv)
    if dz is not None:
        a.dz_st = T.st_bhlp(dz)
    C.check(C.lib().m3_siso_bwd(a, T.stream_handle(dev)))
    return RawGrads(dq=dq, dk=dk, dv=dv, dz=dz, ddt_raw=ddt, da_raw=da, dtrap_raw=dtr, dangles=dang,
                    ddt_bias=ddtb, dq_bias=dqb, dk_bias=dkb, dd_skip=ddsk, dseed_ssm=dss, dseed_k=dsk_,
                    dseed_v=dsv, dseed_phi=dsp)
