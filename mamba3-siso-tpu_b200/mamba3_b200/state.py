"""Carried state and the per-token preprocessing, as device-side torch.

``SISOState`` / ``zero_state`` mirror ``mamba3_pallas/reference.py:46-74``.
``preprocess`` mirrors ``reference.py:104-209`` for callers that drive the
preprocessed-boundary kernels (`kernel_fwd.siso_forward`) themselves; the segment path
(`siso.siso_segment`, the layer and the model) never calls it -- there the same algebra
is fused into the CUDA kernels.
"""

from __future__ import annotations

import math
from typing import NamedTuple, Optional

import torch
import torch.nn.functional as F

TWO_PI = 2.0 * math.pi


class SISOState(NamedTuple):
    """ssm ``(B,H,P,N)`` f32; k ``(B,H,N)`` rotated-unscaled; v ``(B,H,P)``;
    phi ``(B,H,Nr)`` f32 (``reference.py:46-63``)."""

    ssm: torch.Tensor
    k: torch.Tensor
    v: torch.Tensor
    phi: torch.Tensor


def zero_state(batch, nheads, headdim, state_dim, n_angles, dtype=torch.float32, device="cuda") -> SISOState:
    """``reference.py:66-74``."""
    return SISOState(
        ssm=torch.zeros(batch, nheads, headdim, state_dim, dtype=torch.float32, device=device),
        k=torch.zeros(batch, nheads, state_dim, dtype=dtype, device=device),
        v=torch.zeros(batch, nheads, headdim, dtype=dtype, device=device),
        phi=torch.zeros(batch, nheads, n_angles, dtype=torch.float32, device=device),
    )


class Preprocessed(NamedTuple):
    adt: torch.Tensor
    gamma: torch.Tensor
    scale: torch.Tensor
    phi: torch.Tensor
    lam: torch.Tensor
    dt: torch.Tensor


def heavy_tail(x):
    """``reference.py:202-209``."""
    return torch.clamp(x, min=0.0) + 1.0 / (1.0 - torch.clamp(x, max=0.0))


def trapezoid_coeffs(dt, lam):
    """``reference.py:104-131``."""
    gamma = dt * lam
    dt_next = torch.cat([dt[..., 1:], torch.zeros_like(dt[..., :1])], dim=-1)
    lam_next = torch.cat([lam[..., 1:], torch.zeros_like(lam[..., :1])], dim=-1)
    return gamma, gamma + dt_next * (1.0 - lam_next)


def cumulative_angles(angles, dt, phi_init: Optional[torch.Tensor] = None):
    """``reference.py:134-157`` (angles ``(B,H,L,Nr)``, dt ``(B,H,L)``)."""
    theta = torch.tanh(angles.float()) * math.pi * dt[..., None]
    phi = torch.cumsum(theta.float(), dim=2)
    if phi_init is not None:
        phi = phi + phi_init[:, :, None, :].float()
    phi = phi - TWO_PI * torch.floor(phi.detach() / TWO_PI)
    return phi, phi[:, :, -1, :]


def preprocess(dt_raw, a_raw, trap_raw, angles, dt_bias, a_floor=1e-4, phi_init=None):
    """``reference.py:160-199``."""
    dt = F.softplus(dt_raw.float() + dt_bias.float()).transpose(1, 2)
    a = -heavy_tail(a_raw.float()).transpose(1, 2)
    a = torch.clamp(a, max=-a_floor)
    lam = torch.sigmoid(trap_raw.float()).transpose(1, 2)
    gamma, scale = trapezoid_coeffs(dt, lam)
    h = dt.shape[1]
    angles_h = angles[:, None].expand(angles.shape[0], h, *angles.shape[1:])
    phi, phi_final = cumulative_angles(angles_h, dt, phi_init)
    return Preprocessed(adt=a * dt, gamma=gamma, scale=scale, phi=phi, lam=lam, dt=dt), phi_final
