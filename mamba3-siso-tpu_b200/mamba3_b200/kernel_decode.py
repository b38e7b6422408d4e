"""Single-token decode through libm3siso.so (``mamba3_pallas/kernel_decode.py``).

The state is updated IN PLACE -- the counterpart of the reference donating its state
buffers (``kernel_decode.py:350-352``): the returned `SISOState` holds the same tensors
that were passed in (when they were already fp32 and contiguous), so callers thread it
through exactly as with the reference.
"""

from __future__ import annotations

import torch

from . import _capi as C
from . import _tensors as T
from .state import SISOState


def _prep_state(state: SISOState) -> SISOState:
    def f(t):
        return t if (t.dtype == torch.float32 and t.is_contiguous()) else t.float().contiguous()

    return SISOState(ssm=f(state.ssm), k=f(state.k), v=f(state.v), phi=f(state.phi))


def _launch(q, k, v, z, angles, q_bias, k_bias, d_skip, state, dtype_policy, raw, a_floor,
            adt=None, dt=None, lam=None, dt_raw=None, a_raw=None, trap_raw=None, dt_bias=None, y=None,
            q_norm_w=None, k_norm_w=None, norm_eps=1e-5):
    T.require_cuda(q, k, v)
    bsz, n = q.shape
    h, p = v.shape[1], v.shape[2]
    nr = angles.shape[-1]
    dt_io = v.dtype if v.dtype in (torch.bfloat16, torch.float32) else torch.float32
    q, k, v, z = (T.inner_contig(t, dt_io) for t in (q, k, v, z))
    if v.stride(1) != p or (z is not None and (z.stride(1) != p or z.stride(0) != v.stride(0))):
        v = v.contiguous()
        z = None if z is None else z.contiguous()
    if q.stride(0) != k.stride(0):
        q, k = q.contiguous(), k.contiguous()
    # bf16 scalar streams (the in_proj columns of a bf16 model) are read as they are
    scal = (dt_raw, a_raw, trap_raw, angles) if raw else (adt, dt, lam, angles)
    sbf = raw and all(t.dtype == torch.bfloat16 and t.stride(-1) == 1 for t in scal)
    if not sbf:
        angles = T.f32c(angles)
    st = _prep_state(state)
    if y is None:
        y = torch.empty(bsz, h, p, dtype=dt_io, device=q.device)
    a = C.M3DecodeArgs()
    a.batch, a.nheads, a.state_dim, a.headdim, a.n_angles = bsz, h, n, p, nr
    a.io_dtype = T.io_dtype(dt_io)
    a.policy = T.policy_code(dtype_policy)
    a.raw = 1 if raw else 0
    a.a_floor = a_floor
    a.q, a.k, a.qk_stride_b = T.ptr(q), T.ptr(k), q.stride(0)
    a.v, a.z, a.vz_stride_b = T.ptr(v), T.ptr(z), v.stride(0)
    keep = []
    a.scalar_dtype = C.M3_DTYPE_BF16 if sbf else C.M3_DTYPE_F32
    if q_norm_w is not None:
        qn, kn = T.f32dense(q_norm_w), T.f32dense(k_norm_w)
        keep += [qn, kn]
        a.q_norm_w, a.k_norm_w, a.norm_eps = T.ptr(qn), T.ptr(kn), norm_eps
    if raw:
        if not sbf:
            dt_raw, a_raw, trap_raw = (T.f32c(t) for t in (dt_raw, a_raw, trap_raw))
        if dt_raw.stride(0) != a_raw.stride(0) or dt_raw.stride(0) != trap_raw.stride(0):
            dt_raw, a_raw, trap_raw = dt_raw.contiguous(), a_raw.contiguous(), trap_raw.contiguous()
        dtb = T.f32dense(dt_bias)
        keep += [dt_raw, a_raw, trap_raw, dtb]
        a.dt_raw, a.a_raw, a.trap_raw, a.raw_stride_b = T.ptr(dt_raw), T.ptr(a_raw), T.ptr(trap_raw), dt_raw.stride(0)
        a.dt_bias = T.ptr(dtb)
    else:
        adt, dt, lam = (T.f32dense(t) for t in (adt, dt, lam))
        keep += [adt, dt, lam]
        a.adt, a.dt, a.lam = T.ptr(adt), T.ptr(dt), T.ptr(lam)
    a.angles, a.ang_stride_b = T.ptr(angles), angles.stride(0)
    qb, kb, dsk = T.f32dense(q_bias), T.f32dense(k_bias), T.f32dense(d_skip)
    a.q_bias, a.k_bias, a.d_skip = T.ptr(qb), T.ptr(kb), T.ptr(dsk)
    a.ssm, a.state_k, a.state_v, a.phi = T.ptr(st.ssm), T.ptr(st.k), T.ptr(st.v), T.ptr(st.phi)
    a.y = T.ptr(y)
    C.check(C.lib().m3_siso_decode(a, T.stream_handle(q.device)))
    return y, st


def siso_decode(q, k, v, adt, dt, lam, angles, q_bias, k_bias, state: SISOState, d_skip=None, z=None,
                dtype_policy: str = "bf16", interpret=False):
    """One decode step (``kernel_decode.py:252-360``).  ``angles`` are raw (pre-tanh).
    Returns ``(y, next_state)``; ``y`` is ``(B, H, P)``.  ``interpret`` (the reference's
    Pallas interpret mode) is accepted and has no effect."""
    return _launch(q, k, v, z, angles, q_bias, k_bias, d_skip, state, dtype_policy, False, 0.0,
                   adt=adt, dt=dt, lam=lam)


# The reference's head-folded grid (kernel_decode.py:363-464) is a VMEM-footprint choice;
# here one kernel serves both signatures.
siso_decode_folded = siso_decode


def siso_decode_raw(q, k, v, dt_raw, a_raw, trap_raw, angles, dt_bias, q_bias, k_bias, state: SISOState,
                    d_skip=None, z=None, a_floor: float = 1e-4, dtype_policy: str = "bf16", y=None,
                    q_norm_w=None, k_norm_w=None, norm_eps: float = 1e-5):
    """Decode step with ``lm_decode_step``'s length-1 preprocess fused
    (``model.py:274-277``): raw ``(B, H)`` dt/A/trap slices in (fp32, or bf16 in_proj
    columns as they are).  With ``q_norm_w`` / ``k_norm_w`` the q / k rows are the raw C / B
    columns and the layer's RMS norms (``layer.py:190-198``) run inside the kernel."""
    return _launch(q, k, v, z, angles, q_bias, k_bias, d_skip, state, dtype_policy, True, a_floor,
                   dt_raw=dt_raw, a_raw=a_raw, trap_raw=trap_raw, dt_bias=dt_bias, y=y,
                   q_norm_w=q_norm_w, k_norm_w=k_norm_w, norm_eps=norm_eps)


def decode_step(*args, folded: bool = True, **kw):
    """``kernel_decode.py:467-471``."""
    return siso_decode(*args, **kw)


def decode_loop(q, k, v, adt, dt, lam, angles, q_bias, k_bias, state: SISOState, d_skip=None, z=None,
                dtype_policy: str = "bf16", folded: bool = False, interpret=False):
    """``kernel_decode.py:536-573``: one step per token over ``(B, L, ...)`` inputs."""
    outs = []
    for t in range(q.shape[1]):
        y, state = siso_decode(q[:, t], k[:, t], v[:, :, t], adt[:, :, t], dt[:, :, t], lam[:, :, t],
                               angles[:, t], q_bias, k_bias, state, d_skip=d_skip,
                               z=None if z is None else z[:, :, t], dtype_policy=dtype_policy)
        outs.append(y)
    return torch.stack(outs, dim=2), state


def decode_scan(q, k, v, adt, dt, lam, angles, q_bias, k_bias, state: SISOState, d_skip=None, z=None,
                dtype_policy: str = "bf16", folded: bool = True, interpret=False):
    """``kernel_decode.py:474-533``: the device-only multi-step driver.  The steps are
    enqueued back to back with no host synchronisation between them; the result is the
    same as `decode_loop`."""
    return decode_loop(q, k, v, adt, dt, lam, angles, q_bias, k_bias, state, d_skip=d_skip, z=z,
                       dtype_policy=dtype_policy)
