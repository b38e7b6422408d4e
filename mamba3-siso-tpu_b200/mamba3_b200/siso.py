"""Differentiable boundary (``mamba3_pallas/siso.py``) as torch autograd Functions.

`siso` is the preprocessed-boundary core (``siso.py:39-151``: q, k, v, adt, gamma,
scale, phi, biases, D, z, seeds -> y and the final state).  `siso_segment` is the entry
point a layer calls (``siso.py:154-216``); unlike the reference it does not run the
preprocessing as separate ops: softplus / heavy-tail / sigmoid / the trapezoid shift and
the cumulative angles are fused into the forward and backward kernels (the raw
boundary of libm3siso.so).  The forward saves only its inputs; the backward kernel
recomputes the chunk states.
"""

from __future__ import annotations

from typing import NamedTuple, Optional

import torch

from . import kernel_bwd as KB
from . import kernel_fwd as KF
from .state import SISOState


class SISOOutput(NamedTuple):
    """``siso.py:27-36``."""

    y: torch.Tensor
    state: SISOState


def _need(x):
    return x is not None and x.requires_grad


class _SisoFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, adt, gamma, scale, phi, q_bias, k_bias, d_skip, z, seed_ssm, seed_kv, seed_coef,
                chunk, policy_name):
        n = q.shape[-1]
        sk = seed_kv[..., :n] if seed_kv is not None else None
        sv = seed_kv[..., n:] if seed_kv is not None else None
        y, fs, fk, fv = KF.siso_forward(q, k, v, adt, gamma, scale, phi, q_bias, k_bias, d_skip=d_skip, z=z,
                                        seed_ssm=seed_ssm, seed_k=sk, seed_v=sv, seed_coef=seed_coef,
                                        chunk=chunk, dtype_policy=policy_name)
        ctx.save_for_backward(q, k, v, adt, gamma, scale, phi, q_bias, k_bias, d_skip, z, seed_ssm, seed_kv, seed_coef)
        ctx.meta = (chunk, policy_name)
        return y, fs, fk, fv

    @staticmethod
    def backward(ctx, dy, dfs, dfk, dfv):
        q, k, v, adt, gamma, scale, phi, q_bias, k_bias, d_skip, z, seed_ssm, seed_kv, seed_coef = ctx.saved_tensors
        chunk, policy_name = ctx.meta
        n = q.shape[-1]
        sk = seed_kv[..., :n] if seed_kv is not None else None
        sv = seed_kv[..., n:] if seed_kv is not None else None
        if dy is None:
            dy = torch.zeros_like(v)
        g = KB.siso_backward(dy, q, k, v, adt, gamma, scale, phi, q_bias, k_bias, d_skip=d_skip, z=z,
                             seed_ssm=seed_ssm, seed_k=sk, seed_v=sv, seed_coef=seed_coef,
                             dfinal_ssm=dfs, dfinal_k=dfk, dfinal_v=dfv, chunk=chunk, dtype_policy=policy_name)
        dseed_kv = torch.cat([g.dseed_k, g.dseed_v], dim=-1) if seed_kv is not None else None

        def like(x, p):
            return None if (p is None or x is None) else x.to(p.dtype)

        return (like(g.dq, q), like(g.dk, k), like(g.dv, v), like(g.dadt, adt), like(g.dgamma, gamma),
                like(g.dscale, scale), like(g.dphi, phi), like(g.dq_bias, q_bias), like(g.dk_bias, k_bias),
                like(g.dd_skip, d_skip), like(g.dz, z), like(g.dseed_ssm, seed_ssm), like(dseed_kv, seed_kv),
                like(g.dseed_coef, seed_coef), None, None)


def siso(q, k, v, adt, gamma, scale, phi, q_bias, k_bias, d_skip, z, seed_ssm, seed_kv, seed_coef,
         chunk: int = 128, policy_name: str = "bf16"):
    """``siso.py:39-91``: returns ``(y, final_ssm, final_k, final_v)``."""
    return _SisoFn.apply(q, k, v, adt, gamma, scale, phi, q_bias, k_bias, d_skip, z, seed_ssm, seed_kv,
                         seed_coef, chunk, policy_name)


class _SegmentFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, z, dt_raw, a_raw, trap_raw, angles, dt_bias, q_bias, k_bias, d_skip,
                seed_ssm, seed_k, seed_v, seed_phi, a_floor, chunk, policy_name, y_blhp):
        y_out = None
        if y_blhp:  # write y straight into a (B, L, H, P) buffer, seen as (B, H, L, P)
            b_, l_, h_, p_ = v.shape[0], v.shape[2], v.shape[1], v.shape[3]
            y_out = torch.empty(b_, l_, h_, p_, dtype=v.dtype, device=v.device).permute(0, 2, 1, 3)
        # with gradients ahead, the backward's workspace is handed to the forward, which fills
        # in the chunk-start states when it runs on tensor cores (no recompute sweep later)
        ws = None
        if any(ctx.needs_input_grad):
            b_, l_, n_ = q.shape
            ws = torch.empty(KB.workspace_bytes(b_, l_, v.shape[1], n_, v.shape[3], angles.shape[-1], chunk),
                             dtype=torch.uint8, device=q.device)
        (y, fs, fk, fv, fphi), saved = KF.siso_forward_raw(
            q, k, v, dt_raw, a_raw, trap_raw, angles, dt_bias, q_bias, k_bias, d_skip=d_skip, z=z,
            seed_ssm=seed_ssm, seed_k=seed_k, seed_v=seed_v, seed_phi=seed_phi, a_floor=a_floor,
            chunk=chunk, dtype_policy=policy_name, y_out=y_out, bwd_states=ws, return_saved=True)
        ctx.save_for_backward(q, k, v, z, dt_raw, a_raw, trap_raw, angles, dt_bias, q_bias, k_bias, d_skip,
                              seed_ssm, seed_k, seed_v, seed_phi)
        ctx.meta = (a_floor, chunk, policy_name)
        ctx.ws, ctx.saved = ws, saved
        return y, fs, fk, fv, fphi

    @staticmethod
    def backward(ctx, dy, dfs, dfk, dfv, dfphi):
        (q, k, v, z, dt_raw, a_raw, trap_raw, angles, dt_bias, q_bias, k_bias, d_skip,
         seed_ssm, seed_k, seed_v, seed_phi) = ctx.saved_tensors
        a_floor, chunk, policy_name = ctx.meta
        if dy is None:
            dy = torch.zeros(v.shape, dtype=v.dtype, device=v.device)
        gdt = torch.bfloat16 if v.dtype == torch.bfloat16 else torch.float32

        def out_like(x):  # a gradient buffer with x's layout (e.g. a permuted in_proj slice)
            if x is None:
                return None
            b_, h_, l_, p_ = x.shape
            if x.stride(3) == 1 and x.stride(1) == p_ and x.stride(2) >= h_ * p_:
                return torch.empty(b_, l_, h_, p_, dtype=gdt, device=x.device).permute(0, 2, 1, 3)
            return None

        g = KB.siso_backward_raw(
            dy, q, k, v, dt_raw, a_raw, trap_raw, angles, dt_bias, q_bias, k_bias, d_skip=d_skip, z=z,
            seed_ssm=seed_ssm, seed_k=seed_k, seed_v=seed_v, seed_phi=seed_phi, dfinal_ssm=dfs,
            dfinal_k=dfk, dfinal_v=dfv, dfinal_phi=dfphi, a_floor=a_floor, chunk=chunk,
            dtype_policy=policy_name, workspace=ctx.ws, states_ready=ctx.saved,
            grad_dtype=gdt, dv_out=out_like(v), dz_out=out_like(z))
        ctx.ws = None

        def like(x, p):
            return None if (p is None or x is None) else x.to(p.dtype)

        return (like(g.dq, q), like(g.dk, k), like(g.dv, v), like(g.dz, z), like(g.ddt_raw, dt_raw),
                like(g.da_raw, a_raw), like(g.dtrap_raw, trap_raw), like(g.dangles, angles),
                like(g.ddt_bias, dt_bias), like(g.dq_bias, q_bias), like(g.dk_bias, k_bias),
                like(g.dd_skip, d_skip), like(g.dseed_ssm, seed_ssm), like(g.dseed_k, seed_k),
                like(g.dseed_v, seed_v), like(g.dseed_phi, seed_phi), None, None, None, None)


def siso_segment(q, k, v, dt_raw, a_raw, trap_raw, angles, dt_bias, q_bias, k_bias, d_skip=None, z=None,
                 state: Optional[SISOState] = None, a_floor: float = 1e-4, chunk: int = 128,
                 policy_name: str = "bf16", y_blhp: bool = False) -> SISOOutput:
    """``siso.py:154-216``: raw in_proj slices in, ``SISOOutput(y, SISOState)`` out.

    A carried ``state`` seeds the scan with ``dt_0 (1 - lam_0) v_prev k_prev^T`` and its
    ``phi`` continues the cumulative angles, computed from this segment's own inputs --
    the segmentation rule of ``siso.py:176-181``.  Differentiable in every tensor input,
    the carried state included.  ``y_blhp`` makes ``y`` a ``(B, H, L, P)`` view of a
    ``(B, L, H, P)`` buffer, which is what the layer's out_proj wants.
    """
    sp = sk = sv = sphi = None
    if state is not None:
        sp, sk, sv, sphi = state.ssm, state.k, state.v, state.phi
    y, fs, fk, fv, fphi = _SegmentFn.apply(q, k, v, z, dt_raw, a_raw, trap_raw, angles, dt_bias, q_bias, k_bias,
                                           d_skip, sp, sk, sv, sphi, a_floor, chunk, policy_name, y_blhp)
    return SISOOutput(y=y, state=SISOState(ssm=fs, k=fk, v=fv, phi=fphi))


def siso_segment_streamed(q, k, v, dt_raw, a_raw, trap_raw, angles, dt_bias, q_bias, k_bias, d_skip=None, z=None,
                          a_floor: float = 1e-4, chunk: int = 128, policy_name: str = "bf16",
                          segments: int = 8, y_out: Optional[torch.Tensor] = None) -> SISOOutput:
    """`siso_segment` over inputs that live in pinned host memory, with y written back to host.

    Layouts are the in_proj ones: q, k ``(B,L,N)``; v, z ``(B,L,H,P)``; raw dt / A / trap
    ``(B,L,H)``; angles ``(B,L,Nr)``; the per-head parameters are device tensors.  The
    sequence is cut into ``segments`` pieces along L (each a multiple of ``chunk``), scanned
    one after another with the state carried (the segmentation rule of ``siso.py:176-181``),
    while the next piece's inputs go host -> device and the previous piece's y goes device
    -> host on two side streams.  Returns ``SISOOutput(y_host (B,L,H,P), final state on the
    device)``; the caller's current stream is ordered after everything.  Forward only.
    """
    from . import _capi as C

    B, L = q.shape[0], q.shape[1]
    H, P = v.shape[2], v.shape[3]

    def rows_copy(dst, src, t0, n_tok, d_t0, stream):
        # tokens [t0, t0 + n_tok) of every batch row of src -> tokens [d_t0, ...) of dst, one
        # strided copy (both (B, L, ...) with contiguous rows)
        es = src.element_size()
        tok = src[0, 0].numel() * es
        if src.stride(1) * es != tok or dst.stride(1) * es != tok:
            raise ValueError("siso_segment_streamed: every batch row must be token-contiguous")
        C.check(C.lib().m3_copy2d_async(dst.data_ptr() + d_t0 * tok, dst.stride(0) * es, src.data_ptr() + t0 * tok,
                                        src.stride(0) * es, n_tok * tok, src.shape[0], stream.cuda_stream))

    seg = max(chunk, (L // max(segments, 1)) // chunk * chunk)
    while L % seg:
        seg -= chunk
    n_seg = L // seg
    cur = torch.cuda.current_stream()
    dev = q.device if q.is_cuda else dt_bias.device
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    s_in.wait_stream(cur)  # the device buffers below may reuse memory the current stream still reads
    names = ("q", "k", "v", "z", "dt_raw", "a_raw", "trap_raw", "angles")
    host = dict(q=q, k=k, v=v, z=z, dt_raw=dt_raw, a_raw=a_raw, trap_raw=trap_raw, angles=angles)
    dbuf = {n: torch.empty(t.shape, dtype=t.dtype, device=dev) for n, t in host.items() if t is not None}
    if y_out is None:
        y_out = torch.empty(B, L, H, P, dtype=v.dtype, pin_memory=True)
    state = None
    keep = []
    with torch.no_grad():
        for i in range(n_seg):
            sl = slice(i * seg, (i + 1) * seg)
            for n in names:
                if host[n] is not None:
                    rows_copy(dbuf[n], host[n], i * seg, seg, i * seg, s_in)
            ev_in = torch.cuda.Event()
            ev_in.record(s_in)
            cur.wait_event(ev_in)
            out = siso_segment(dbuf["q"][:, sl], dbuf["k"][:, sl], dbuf["v"][:, sl].permute(0, 2, 1, 3),
                               dbuf["dt_raw"][:, sl], dbuf["a_raw"][:, sl], dbuf["trap_raw"][:, sl],
                               dbuf["angles"][:, sl], dt_bias, q_bias, k_bias, d_skip,
                               None if z is None else dbuf["z"][:, sl].permute(0, 2, 1, 3), state=state,
                               a_floor=a_floor, chunk=chunk, policy_name=policy_name, y_blhp=True)
            state = out.state
            ybuf = out.y.permute(0, 2, 1, 3)  # (B, seg, H, P), contiguous
            ev_c = torch.cuda.Event()
            ev_c.record(cur)
            s_out.wait_event(ev_c)
            ybuf.record_stream(s_out)
            rows_copy(y_out, ybuf, 0, seg, i * seg, s_out)
            keep.append(ybuf)
    for t in dbuf.values():
        t.record_stream(s_in)
    cur.wait_stream(s_out)
    return SISOOutput(y=y_out, state=state)


@torch.no_grad()
def siso_segment_seq_parallel(q, k, v, dt_raw, a_raw, trap_raw, angles, dt_bias, q_bias, k_bias, d_skip=None,
                              z=None, state: Optional[SISOState] = None, a_floor: float = 1e-4, chunk: int = 128,
                              policy_name: str = "bf16", group=None, segment_fn=None) -> SISOOutput:
    """Sequence-parallel prefill: rank r of ``group`` holds the r-th contiguous L-slice of
    the same sequences (every other argument as for `siso_segment`; ``state`` is the
    carry entering rank 0's slice and is ignored on the other ranks).  Returns this
    rank's y and the exact carry at the end of its slice -- on the last rank, the state
    after the whole sequence.  Forward only.

    The chained-segment result (``siso.py:154-216`` applied slice after slice) is
    reached with two scans per rank and two all-gathers, no rank waiting on another's scan:

    1. The cumulative angle entering slice r is the carry's phi plus the earlier slices'
       sums of tanh(angle) pi dt (mod 2 pi), from an all-gather of each slice's sum.
    2. Scan 1 runs the slice from (ssm 0, k 0, v 0, phi_in) -- the states-only kernel where
       the shapes allow, as no y is needed: its final ssm S_r holds everything the slice
       itself adds, its final k and v are the true last-token ones.
    3. A carry enters a slice as the seeded state S_in + coef v_prev k_prev^T (coef =
       dt_1 (1 - lam_1) of the slice's first token, ``siso.py:207``), which the slice only
       decays, by e^{A} with A the slice's sum of adt.  So after an all-gather of
       (S_r, k_r, v_r, A_r, coef_r) every rank rebuilds
       S_end(j) = e^{A_j} (S_end(j-1) + coef_j v_{j-1} k_{j-1}^T) + S_j for the slices
       before it.
    4. Scan 2 runs the slice from the true carry (S_end(r-1), k_{r-1}, v_{r-1}, phi_in).

    ``segment_fn`` replaces `siso_segment` (same signature and result); tests use it to
    run the exchange logic on CPU ranks.
    """
    import torch.distributed as dist

    from .state import heavy_tail

    seg = segment_fn or siso_segment
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    b, h, p, n, nr = v.shape[0], v.shape[1], v.shape[-1], q.shape[-1], angles.shape[-1]
    dev, f32 = v.device, torch.float32
    if state is None:
        state = SISOState(ssm=torch.zeros(b, h, p, n, dtype=f32, device=dev),
                          k=torch.zeros(b, h, n, dtype=f32, device=dev),
                          v=torch.zeros(b, h, p, dtype=f32, device=dev),
                          phi=torch.zeros(b, h, nr, dtype=f32, device=dev))

    def gather(t):
        out = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(out, t.contiguous(), group=group)
        return out

    # per-slice scalars of the preprocessing (reference.py:160-199), float64 sums
    dt = torch.nn.functional.softplus(dt_raw.double() + dt_bias.double())             # (B, L, H)
    adt = torch.clamp(-heavy_tail(a_raw.double()), max=-a_floor) * dt
    lam = torch.sigmoid(trap_raw.double())
    inc = torch.einsum("blh,blr->bhr", dt, torch.tanh(angles.double())) * torch.pi  # angle increment
    a_all = adt.sum(1)                                                               # (B, H)
    coef = dt[:, 0] * (1.0 - lam[:, 0])
    # 1. entering angles
    incs = gather(inc)
    phi_in = gather(state.phi.double())[0].clone()  # rank 0's carry
    for j in range(rank):
        phi_in = phi_in + incs[j]
    phi_in = torch.remainder(phi_in, 2 * torch.pi).to(f32)
    if rank != 0:
        state = None  # only rank 0's carry is the caller's
    # 2. scan 1 from a zero carry at the true entering angle
    zero = SISOState(ssm=torch.zeros(b, h, p, n, dtype=f32, device=dev), k=torch.zeros(b, h, n, dtype=f32, device=dev),
                     v=torch.zeros(b, h, p, dtype=f32, device=dev), phi=phi_in)
    kw = dict(a_floor=a_floor, chunk=chunk, policy_name=policy_name)
    if segment_fn is None and KF.final_state_supported(q, v, angles, chunk, policy_name):
        # scan 1 needs no y: the states-only kernel
        _, fs, fk, fv, fphi = KF.siso_forward_raw(q, k, v, dt_raw, a_raw, trap_raw, angles, dt_bias, q_bias,
                                                  k_bias, d_skip=d_skip, z=z, seed_ssm=zero.ssm, seed_k=zero.k,
                                                  seed_v=zero.v, seed_phi=zero.phi, a_floor=a_floor, chunk=chunk,
                                                  dtype_policy=policy_name, states_only=True)
        f0 = SISOState(ssm=fs, k=fk, v=fv, phi=fphi)
    else:
        f0 = seg(q, k, v, dt_raw, a_raw, trap_raw, angles, dt_bias, q_bias, k_bias, d_skip, z, state=zero, **kw).state
    # 3. exchange and rebuild the carry entering this slice
    parts = gather(torch.cat([f0.ssm.reshape(b, h, -1).double(), f0.k.reshape(b, h, -1).double(),
                              f0.v.reshape(b, h, -1).double(), a_all[..., None], coef[..., None]], dim=-1))
    carry0 = gather(torch.cat([s.reshape(b, h, -1).double() for s in
                               (state if state is not None else zero)[:3]], dim=-1))[0]
    s_end = carry0[..., :p * n].reshape(b, h, p, n)
    k_end = carry0[..., p * n:p * n + n]
    v_end = carry0[..., p * n + n:p * n + n + p]
    for j in range(rank):
        pj = parts[j]
        s_j = pj[..., :p * n].reshape(b, h, p, n)
        k_j, v_j = pj[..., p * n:p * n + n], pj[..., p * n + n:p * n + n + p]
        aj, cj = pj[..., -2], pj[..., -1]
        s_end = torch.exp(aj)[..., None, None] * (s_end + cj[..., None, None] * v_end[..., :, None] * k_end[..., None, :])
        s_end = s_end + s_j
        k_end, v_end = k_j, v_j
    carry = SISOState(ssm=s_end.to(f32), k=k_end.to(f32), v=v_end.to(f32), phi=phi_in)
    # 4. scan 2 from the true carry
    return seg(q, k, v, dt_raw, a_raw, trap_raw, angles, dt_bias, q_bias, k_bias, d_skip, z, state=carry, **kw)
