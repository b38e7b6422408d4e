"""CPU oracle for the Mamba-3 SISO scan path -- TEST INFRASTRUCTURE ONLY.

This module is the parity checker. Only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline arm may import it; the product (the CUDA library and the
``mamba3_b200`` package) never does, and never falls back to it.

It restates, in plain torch on the CPU (float64 by default), the pure-JAX reference
``mamba3_pallas/reference.py`` of burak-colakkadioglu/mamba3-siso-tpu together with the
rotary / prefix-sum helpers of ``mamba3_pallas/layout.py``.  Every function cites the
reference lines it follows.  JAX is not installed on either machine, so the reference
module itself cannot run; the restatement is pinned instead against the reference's own
torch recurrence ``mamba3_pallas/torch_ref.py:64-138`` (``mamba3_siso_ref``), run in
this container by ``tests/golden/make_golden.py`` and committed as fixtures under
``tests/golden/``, and against the analytic rotation known-answer test of
``mamba3_pallas/tests.py:451-513``.

Layout conventions (the reference's): ``q``/``k`` are head-shared ``(B, L, N)`` in the
half-split ("permuted") rotary layout; ``v``/``z``/``y`` are ``(B, H, L, P)``; per-token
scalars are ``(B, H, L)``; cumulative angles are ``(B, H, L, Nr)``.

``policy="bf16"`` reproduces the points at which the reference *kernel* rounds matmul
operands to bfloat16 (``kernel_fwd.py:139-187``); everything else stays in the oracle's
dtype.  ``policy="f32"`` rounds nothing.
"""

from __future__ import annotations

import math
from typing import NamedTuple, Optional

import torch

TWO_PI = 2.0 * math.pi
LOG2_E = 1.4426950408889634


# --------------------------------------------------------------------------------------
# helpers from layout.py
# --------------------------------------------------------------------------------------


def deinterleave_perm(n: int) -> torch.Tensor:
    """``layout.py:299-321``: interleaved rotary pairs -> half-split layout.

    ``new[j] = old[2j]``, ``new[n/2 + j] = old[2j + 1]``.
    """
    if n % 2:
        raise ValueError(f"state dim must be even, got {n}")
    return torch.cat([torch.arange(0, n, 2), torch.arange(1, n, 2)])


def interleave_perm(n: int) -> torch.Tensor:
    """``layout.py:324-327``: inverse of `deinterleave_perm`."""
    return torch.argsort(deinterleave_perm(n))


def rope_cos_sin(phi: torch.Tensor, state_dim: int):
    """``layout.py:345-372``: full-width cos/sin; pairs past ``Nr`` pass through."""
    half = state_dim // 2
    nr = phi.shape[-1]
    if nr > half:
        raise ValueError(f"n_angles ({nr}) exceeds state_dim // 2 ({half})")
    if nr < half:
        pad = torch.zeros((*phi.shape[:-1], half - nr), dtype=phi.dtype)
        phi = torch.cat([phi, pad], dim=-1)
    full = torch.cat([phi, phi], dim=-1)
    return torch.cos(full), torch.sin(full)


def rope_apply(x, cos_full, sin_full):
    """``layout.py:375-398``: ``x * cos + rot_half(x) * sin``, ``rot_half = [-hi, lo]``."""
    half = x.shape[-1] // 2
    lo, hi = x[..., :half], x[..., half:]
    rot = torch.cat([-hi, lo], dim=-1)
    return x * cos_full + rot * sin_full


def rope_dphi(x_rot, dx_rot, n_angles: int):
    """``layout.py:414-428``: ``dphi_j = dhi_j * lo_j - dlo_j * hi_j`` for ``j < Nr``."""
    half = x_rot.shape[-1] // 2
    lo, hi = x_rot[..., :half], x_rot[..., half:]
    dlo, dhi = dx_rot[..., :half], dx_rot[..., half:]
    return (dhi * lo - dlo * hi)[..., :n_angles]


def num_chunks(seqlen: int, chunk: int) -> int:
    """``layout.py:500-506``."""
    if seqlen % chunk:
        raise ValueError(f"seqlen ({seqlen}) must be a multiple of chunk ({chunk})")
    return seqlen // chunk


def _bf16(x):
    return x.to(torch.bfloat16).to(x.dtype)


def _mm_round(policy: str):
    if policy == "bf16":
        return _bf16
    if policy == "f32":
        return lambda x: x
    raise ValueError(f"unknown policy {policy!r}")


# --------------------------------------------------------------------------------------
# state + preprocessing: reference.py:46-209
# --------------------------------------------------------------------------------------


class SISOState(NamedTuple):
    """``reference.py:46-63``: ssm (B,H,P,N), k (B,H,N) rotated-unscaled, v (B,H,P),
    phi (B,H,Nr)."""

    ssm: torch.Tensor
    k: torch.Tensor
    v: torch.Tensor
    phi: torch.Tensor


def zero_state(batch, nheads, headdim, state_dim, n_angles, dtype=torch.float64):
    """``reference.py:66-74``."""
    return SISOState(
        ssm=torch.zeros(batch, nheads, headdim, state_dim, dtype=dtype),
        k=torch.zeros(batch, nheads, state_dim, dtype=dtype),
        v=torch.zeros(batch, nheads, headdim, dtype=dtype),
        phi=torch.zeros(batch, nheads, n_angles, dtype=dtype),
    )


class Preprocessed(NamedTuple):
    """``reference.py:82-101``."""

    adt: torch.Tensor
    gamma: torch.Tensor
    scale: torch.Tensor
    phi: torch.Tensor
    lam: torch.Tensor
    dt: torch.Tensor


def heavy_tail(x):
    """``reference.py:202-209``: ``max(x,0) + 1/(1 - min(x,0))``."""
    return torch.clamp(x, min=0.0) + 1.0 / (1.0 - torch.clamp(x, max=0.0))


def trapezoid_coeffs(dt, lam):
    """``reference.py:104-131``: ``gamma = dt*lam``,
    ``scale_t = gamma_t + dt_{t+1} (1 - lam_{t+1})`` with a zero successor at the end."""
    gamma = dt * lam
    dt_next = torch.cat([dt[..., 1:], torch.zeros_like(dt[..., :1])], dim=-1)
    lam_next = torch.cat([lam[..., 1:], torch.zeros_like(lam[..., :1])], dim=-1)
    return gamma, gamma + dt_next * (1.0 - lam_next)


def cumulative_angles(angles, dt, phi_init=None):
    """``reference.py:134-157``: ``phi = (phi_init + cumsum(tanh(a) pi dt)) mod 2 pi``.

    ``angles`` is ``(B, H, L, Nr)`` raw, ``dt`` is ``(B, H, L)``.  The floor of the
    wrap has zero derivative, as in the reference.
    """
    theta = torch.tanh(angles) * math.pi * dt[..., None]
    phi = torch.cumsum(theta, dim=2)
    if phi_init is not None:
        phi = phi + phi_init[:, :, None, :]
    phi = phi - TWO_PI * torch.floor(phi.detach() / TWO_PI)
    return phi, phi[:, :, -1, :]


def preprocess(dt_raw, a_raw, trap_raw, angles, dt_bias, a_floor=1e-4, phi_init=None):
    """``reference.py:160-199``.  Raw ``(B, L, H)`` streams and head-shared
    ``(B, L, Nr)`` angles in; per-head ``(B, H, L)`` scalars and ``(B, H, L, Nr)`` phi out."""
    dt = torch.nn.functional.softplus(dt_raw + dt_bias).transpose(1, 2)
    a = -heavy_tail(a_raw).transpose(1, 2)
    a = torch.minimum(a, torch.full_like(a, -a_floor))
    lam = torch.sigmoid(trap_raw).transpose(1, 2)
    gamma, scale = trapezoid_coeffs(dt, lam)
    nheads = dt.shape[1]
    angles_h = angles[:, None, :, :].expand(angles.shape[0], nheads, *angles.shape[1:])
    phi, phi_final = cumulative_angles(angles_h, dt, phi_init)
    return Preprocessed(adt=a * dt, gamma=gamma, scale=scale, phi=phi, lam=lam, dt=dt), phi_final


# --------------------------------------------------------------------------------------
# recurrent ground truth: reference.py:217-287
# --------------------------------------------------------------------------------------


def siso_recurrent(q, k, v, adt, dt, lam, phi, q_bias, k_bias, d_skip=None, z=None, state=None):
    """Three-term trapezoidal scan, one token at a time (``reference.py:217-287``)."""
    batch, seqlen, n = q.shape
    nheads, p = v.shape[1], v.shape[3]
    if state is None:
        state = zero_state(batch, nheads, p, n, phi.shape[-1], q.dtype)
    ssm, k_prev, v_prev = state.ssm, state.k, state.v
    ys = []
    for t in range(seqlen):
        u = q[:, t][:, None, :] + q_bias[None]
        w = k[:, t][:, None, :] + k_bias[None]
        cos_f, sin_f = rope_cos_sin(phi[:, :, t, :], n)
        q_rot = rope_apply(u, cos_f, sin_f)
        k_rot = rope_apply(w, cos_f, sin_f)
        alpha = torch.exp(adt[:, :, t])
        beta = (1.0 - lam[:, :, t]) * dt[:, :, t] * alpha
        gamma = dt[:, :, t] * lam[:, :, t]
        v_t = v[:, :, t, :]
        ssm = (
            alpha[..., None, None] * ssm
            + beta[..., None, None] * (v_prev[..., :, None] * k_prev[..., None, :])
            + gamma[..., None, None] * (v_t[..., :, None] * k_rot[..., None, :])
        )
        y = torch.einsum("bhpn,bhn->bhp", ssm, q_rot)
        if d_skip is not None:
            y = y + d_skip[None, :, None] * v_t
        if z is not None:
            z_t = z[:, :, t, :]
            y = y * (z_t * torch.sigmoid(z_t))
        ys.append(y)
        k_prev, v_prev = k_rot, v_t
    y = torch.stack(ys, dim=2)
    return y, SISOState(ssm=ssm, k=k_prev, v=v_prev, phi=phi[:, :, -1, :])


# --------------------------------------------------------------------------------------
# chunked form (the gradient oracle): reference.py:295-434
# --------------------------------------------------------------------------------------


def siso_chunked(
    q, k, v, adt, gamma, scale, phi, q_bias, k_bias,
    d_skip=None, z=None, state=None, seed_dt=None, seed_lam=None,
    chunk=128, return_debug=False, policy="f32",
):
    """Chunked linear-attention form (``reference.py:295-434``).

    With ``policy="bf16"`` the matmul operands are rounded where the reference kernel
    rounds them (``kernel_fwd.py:139-187``): ``q~``, ``khat``, ``v``, the carried state
    at the readout, the masked score matrix, and the decayed ``v`` of the state update.
    The decay uses ``exp2`` of a ``log2 e`` prescaled prefix sum like the kernel
    (``kernel_fwd.py:116-120``); in float64 that is the same number as ``exp``.
    """
    rnd = _mm_round(policy)
    batch, seqlen, n = q.shape
    nheads, p = v.shape[1], v.shape[3]
    nc = num_chunks(seqlen, chunk)
    if state is None:
        s0 = torch.zeros(batch, nheads, p, n, dtype=q.dtype)
    else:
        if seed_dt is None or seed_lam is None:
            raise ValueError("seed_dt and seed_lam are required when passing a state")
        seed = (seed_dt * (1.0 - seed_lam))[..., None, None]
        s0 = state.ssm + seed * (state.v[..., :, None] * state.k[..., None, :])

    u = q[:, None, :, :] + q_bias[None, :, None, :]
    w = k[:, None, :, :] + k_bias[None, :, None, :]
    cos_f, sin_f = rope_cos_sin(phi, n)
    q_rot = rope_apply(u, cos_f, sin_f)
    k_rot = rope_apply(w, cos_f, sin_f)
    k_hat = k_rot * scale[..., None]
    qk_diag = (u * w).sum(-1) * gamma

    qm, km, vm = rnd(q_rot), rnd(k_hat), rnd(v)
    idx = torch.arange(chunk)
    strict = idx[:, None] > idx[None, :]
    ssm = s0
    outs, states = [], []
    for c in range(nc):
        sl = slice(c * chunk, (c + 1) * chunk)
        A = torch.cumsum(adt[:, :, sl] * LOG2_E, dim=-1)
        A_last = A[..., -1:]
        q_b, k_b, v_b = qm[:, :, sl], km[:, :, sl], vm[:, :, sl]
        out = torch.einsum("bhtn,bhpn->bhtp", q_b, rnd(ssm)) * torch.exp2(A)[..., None]
        s = torch.einsum("bhtn,bhsn->bhts", q_b, k_b)
        s = s * torch.exp2(torch.clamp(A[..., :, None] - A[..., None, :], max=0.0))
        s = torch.where(strict, s, torch.zeros_like(s))
        out = out + torch.einsum("bhts,bhsp->bhtp", rnd(s), v_b)
        coeff = qk_diag[:, :, sl]
        if d_skip is not None:
            coeff = coeff + d_skip[None, :, None]
        out = out + coeff[..., None] * v[:, :, sl]
        v_scaled = rnd(v[:, :, sl] * torch.exp2(A_last - A)[..., None])
        states.append(ssm)
        ssm = ssm * torch.exp2(A_last)[..., None] + torch.einsum("bhtp,bhtn->bhpn", v_scaled, k_b)
        outs.append(out)
    ybar = torch.cat(outs, dim=2)
    y = ybar * (z * torch.sigmoid(z)) if z is not None else ybar
    final = SISOState(ssm=ssm, k=k_rot[:, :, -1, :], v=v[:, :, -1, :], phi=phi[:, :, -1, :])
    if not return_debug:
        return y, final
    debug = {
        "ybar": ybar,
        "chunk_states": torch.stack(states, dim=2),
        "q_rot": q_rot,
        "k_rot": k_rot,
        "k_hat": k_hat,
        "qk_diag": qk_diag,
        "uw": (u * w).sum(-1),
        "seeded_state": s0,
    }
    return y, final, debug


# --------------------------------------------------------------------------------------
# decode reference: reference.py:442-490
# --------------------------------------------------------------------------------------


def siso_step(q, k, v, adt, dt, lam, angles, q_bias, k_bias, state, d_skip=None, z=None,
              policy="f32"):
    """One decode token, three-term form (``reference.py:442-490``).  ``policy="bf16"``
    rounds ``q~`` and the updated state at the readout (``kernel_decode.py:216-222``)."""
    rnd = _mm_round(policy)
    n = q.shape[-1]
    phi = state.phi + torch.tanh(angles)[:, None, :] * math.pi * dt[..., None]
    phi = phi - TWO_PI * torch.floor(phi.detach() / TWO_PI)
    u = q[:, None, :] + q_bias[None]
    w = k[:, None, :] + k_bias[None]
    cos_f, sin_f = rope_cos_sin(phi, n)
    q_rot = rope_apply(u, cos_f, sin_f)
    k_rot = rope_apply(w, cos_f, sin_f)
    alpha = torch.exp(adt)
    beta = alpha * dt * (1.0 - lam)
    gamma = dt * lam
    ssm = (
        alpha[..., None, None] * state.ssm
        + beta[..., None, None] * (state.v[..., :, None] * state.k[..., None, :])
        + gamma[..., None, None] * (v[..., :, None] * k_rot[..., None, :])
    )
    y = torch.einsum("bhpn,bhn->bhp", rnd(ssm), rnd(q_rot))
    if d_skip is not None:
        y = y + d_skip[None, :, None] * v
    if z is not None:
        y = y * (z * torch.sigmoid(z))
    return y, SISOState(ssm=ssm, k=k_rot, v=v, phi=phi)


# --------------------------------------------------------------------------------------
# segment wrapper: siso.py:154-216 (preprocess + seeded chunked scan)
# --------------------------------------------------------------------------------------


def siso_segment(q, k, v, dt_raw, a_raw, trap_raw, angles, dt_bias, q_bias, k_bias,
                 d_skip=None, z=None, state: Optional[SISOState] = None, a_floor=1e-4,
                 chunk=128, policy="f32"):
    """``siso.py:154-216``: this segment's own preprocessing, the ``seed_coef``
    ``dt_0 (1 - lam_0)`` seeding of a carried state, then the chunked scan.  Returns
    ``(y, SISOState)`` with ``phi`` taken from this segment's last position."""
    pre, _ = preprocess(dt_raw, a_raw, trap_raw, angles, dt_bias, a_floor=a_floor,
                        phi_init=None if state is None else state.phi)
    seed_dt = seed_lam = None
    if state is not None:
        seed_dt, seed_lam = pre.dt[:, :, 0], pre.lam[:, :, 0]
    y, fin = siso_chunked(q, k, v, pre.adt, pre.gamma, pre.scale, pre.phi, q_bias, k_bias,
                          d_skip, z, state=state, seed_dt=seed_dt, seed_lam=seed_lam,
                          chunk=chunk, policy=policy)
    return y, SISOState(ssm=fin.ssm, k=fin.k, v=fin.v, phi=pre.phi[:, :, -1, :])


# --------------------------------------------------------------------------------------
# layer: layer.py:163-262 (projections around the scan)
# --------------------------------------------------------------------------------------


def rms_norm(x, weight, eps):
    """``layer.py:190-198``: no mean subtraction, gain after scaling."""
    rstd = torch.rsqrt((x * x).mean(-1, keepdim=True) + eps)
    return x * rstd * weight


def split_in_proj(proj, d_inner, d_state, nheads, n_angles, headdim):
    """``layer.py:163-187``: ``[z, x, B, C, dd_dt, dd_A, trap, angles]``."""
    sizes = [d_inner, d_inner, d_state, d_state, nheads, nheads, nheads, n_angles]
    z, x, b, c, dt_raw, a_raw, trap_raw, angles = torch.split(proj, sizes, dim=-1)
    bsz, seqlen = proj.shape[:2]
    return (z.reshape(bsz, seqlen, nheads, headdim), x.reshape(bsz, seqlen, nheads, headdim),
            b, c, dt_raw, a_raw, trap_raw, angles)


def layer_forward(params: dict, u, *, d_state, headdim, nheads, n_angles, chunk,
                  a_floor=1e-4, norm_eps=1e-5, state=None, policy="f32"):
    """``layer.py:201-262``.  ``params`` holds ``in_proj (d_model, d_in_proj)``,
    ``out_proj (d_inner, d_model)``, ``dt_bias``, ``b_norm_weight``, ``c_norm_weight``,
    ``b_bias``, ``c_bias``, ``d_skip`` in the permuted layout."""
    d_inner = nheads * headdim
    proj = u @ params["in_proj"]
    z, x, b, c, dt_raw, a_raw, trap_raw, angles = split_in_proj(
        proj, d_inner, d_state, nheads, n_angles, headdim)
    b = rms_norm(b, params["b_norm_weight"], norm_eps)
    c = rms_norm(c, params["c_norm_weight"], norm_eps)
    y, st = siso_segment(c, b, x.transpose(1, 2), dt_raw, a_raw, trap_raw, angles,
                         params["dt_bias"], params["c_bias"], params["b_bias"],
                         params["d_skip"], z.transpose(1, 2), state=state, a_floor=a_floor,
                         chunk=chunk, policy=policy)
    bsz, seqlen = u.shape[:2]
    y = y.transpose(1, 2).reshape(bsz, seqlen, d_inner)
    return y @ params["out_proj"], st


# --------------------------------------------------------------------------------------
# sampling filter: train.py:454-500 (_pick_token, before the categorical draw)
# --------------------------------------------------------------------------------------


def nucleus_probs(logits, seen, temperature, top_p, rep_penalty):
    """``train.py:483-498``: the distribution ``_pick_token`` draws from, per row.

    Sign-aware repetition penalty on ``seen`` ids, division by the temperature, then the
    nucleus: sort descending -- ``argsort(lg)[::-1]``, so among equal values the higher
    index comes first -- and keep an entry iff the softmax mass strictly before it is
    < top_p.  Returns the softmax over the kept entries (zeros elsewhere), in the dtype of
    ``logits`` (float64 recommended).  ``logits`` ``(R, V)``, ``seen`` bool ``(R, V)``."""
    lg = torch.where(seen, torch.where(logits > 0, logits / rep_penalty, logits * rep_penalty), logits)
    lg = lg / temperature
    # stable ascending sort, then reversed: ties end up in descending index order
    order = torch.sort(lg, dim=-1, stable=True).indices.flip(-1)
    srt = torch.gather(lg, -1, order)
    probs = torch.softmax(srt, dim=-1)
    keep = (torch.cumsum(probs, dim=-1) - probs) < top_p
    masked = torch.where(keep, srt, torch.full_like(srt, -math.inf))
    out = torch.full_like(lg, -math.inf).scatter(-1, order, masked)
    return torch.softmax(out, dim=-1)
