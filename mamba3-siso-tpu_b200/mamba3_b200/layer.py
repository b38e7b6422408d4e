"""The Mamba-3 SISO layer around the scan (``mamba3_pallas/layer.py``).

    in_proj -> [z, x, B, C, dd_dt, dd_A, trap, angles]
    B, C    -> RMSNorm
    scan    -> gated by silu(z)        (C is the query, B the key)
    out_proj

The projections are torch (cuBLAS) GEMMs; every slice of the fused projection reaches
the scan kernel as a strided view -- no transposes or copies of x, z or the scalar
streams -- and the kernel writes y straight into the (B, L, H, P) layout out_proj reads.
"""

from __future__ import annotations

import dataclasses
import itertools
import math
from typing import NamedTuple, Optional

import torch

from . import layout as L
from . import siso as SISO
from .state import SISOState


@dataclasses.dataclass(frozen=True)
class SISOConfig:
    """``layer.py:39-99``.  ``chunk`` must be a positive multiple of 64 here (the
    reference demands a multiple of 128, a TPU lane rule with no B200 counterpart)."""

    d_model: int
    d_state: int = 128
    headdim: int = 64
    expand: int = 2
    rope_fraction: float = 0.5
    chunk: int = 128
    a_floor: float = 1e-4
    norm_eps: float = 1e-5
    dt_min: float = 0.001
    dt_max: float = 0.1
    dt_init_floor: float = 1e-4
    policy_name: str = "bf16"

    @property
    def d_inner(self) -> int:
        return self.expand * self.d_model

    @property
    def nheads(self) -> int:
        if self.d_inner % self.headdim != 0:
            raise ValueError(f"d_inner {self.d_inner} not divisible by headdim {self.headdim}")
        return self.d_inner // self.headdim

    @property
    def n_angles(self) -> int:
        if self.rope_fraction not in (0.5, 1.0):
            raise ValueError(f"rope_fraction must be 0.5 or 1.0, got {self.rope_fraction}")
        width = int(self.d_state * self.rope_fraction)
        if width % 2:
            width -= 1
        n = width // 2
        if n <= 0:
            raise ValueError("rope_fraction too small: no rotary angles")
        return n

    @property
    def d_in_proj(self) -> int:
        return 2 * self.d_inner + 2 * self.d_state + 3 * self.nheads + self.n_angles

    def __post_init__(self):
        L.validate_chunk(self.chunk)
        L.policy(self.policy_name)
        _ = self.nheads, self.n_angles


class SISOParams(NamedTuple):
    """``layer.py:102-124``: in_proj ``(d_model, d_in_proj)``, out_proj
    ``(d_inner, d_model)``, dt_bias ``(H,)``, norm gains ``(N,)``, biases ``(H, N)``
    (permuted layout), d_skip ``(H,)``."""

    in_proj: torch.Tensor
    out_proj: torch.Tensor
    dt_bias: torch.Tensor
    b_norm_weight: torch.Tensor
    c_norm_weight: torch.Tensor
    b_bias: torch.Tensor
    c_bias: torch.Tensor
    d_skip: torch.Tensor


def _gen(key, device):
    if isinstance(key, torch.Generator):
        return key
    g = torch.Generator(device="cpu")
    g.manual_seed(int(key))
    return g


def init_params(cfg: SISOConfig, key=0, dtype=torch.float32, device="cuda") -> SISOParams:
    """``layer.py:127-160``: uniform ``+-1/sqrt(fan_in)`` projections, ``dt_bias`` the
    inverse softplus of a log-uniform ``[dt_min, dt_max]`` draw, norms / biases / D = 1.
    ``key`` is an int seed or a CPU ``torch.Generator`` (jax.random streams cannot be
    reproduced without JAX, so the values -- not the distributions -- differ)."""
    g = _gen(key, device)
    s_in = 1.0 / math.sqrt(cfg.d_model)
    s_out = 1.0 / math.sqrt(cfg.d_inner)
    u = torch.rand(cfg.nheads, generator=g, dtype=torch.float32)
    dt = torch.exp(u * (math.log(cfg.dt_max) - math.log(cfg.dt_min)) + math.log(cfg.dt_min))
    dt = torch.clamp(dt, min=cfg.dt_init_floor)
    dt_bias = dt + torch.log(-torch.expm1(-dt))
    in_proj = (torch.rand(cfg.d_model, cfg.d_in_proj, generator=g) * 2 - 1) * s_in
    out_proj = (torch.rand(cfg.d_inner, cfg.d_model, generator=g) * 2 - 1) * s_out
    to = dict(dtype=dtype, device=device)
    return SISOParams(
        in_proj=in_proj.to(**to), out_proj=out_proj.to(**to), dt_bias=dt_bias.to(**to),
        b_norm_weight=torch.ones(cfg.d_state, **to), c_norm_weight=torch.ones(cfg.d_state, **to),
        b_bias=torch.ones(cfg.nheads, cfg.d_state, **to), c_bias=torch.ones(cfg.nheads, cfg.d_state, **to),
        d_skip=torch.ones(cfg.nheads, **to))


def split_in_proj(proj: torch.Tensor, cfg: SISOConfig):
    """``layer.py:163-187``: ``(z, x, B, C, dt_raw, a_raw, trap_raw, angles)`` as views;
    z / x come back ``(B, L, H, P)``."""
    sizes = (cfg.d_inner, cfg.d_inner, cfg.d_state, cfg.d_state, cfg.nheads, cfg.nheads, cfg.nheads, cfg.n_angles)
    z, x, b, c, dt_raw, a_raw, trap_raw, angles = torch.split(proj, sizes, dim=-1)
    lead = proj.shape[:-1]
    return (z.unflatten(-1, (cfg.nheads, cfg.headdim)), x.unflatten(-1, (cfg.nheads, cfg.headdim)),
            b, c, dt_raw, a_raw, trap_raw, angles)


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """``layer.py:190-198``: f32 internally, gain after scaling, cast back.

    On CUDA rows it is one fused kernel (`m3_rms_norm`), with a fused backward
    (`m3_rms_norm_bwd`) when autograd needs one; other inputs take the torch ops below."""
    rs = _row_stride(x, weight)
    if rs is not None:
        if torch.is_grad_enabled() and (x.requires_grad or weight.requires_grad):
            if x.shape[-1] <= 2048:
                return _RMSNormFn.apply(x, weight, eps)
        else:
            return _rms_norm_fused(x, weight, eps, rs)[0]
    xf = x.float()
    rstd = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (xf * rstd * weight.float()).to(x.dtype)


def _row_stride(x, weight):
    """The row stride of x viewed as (rows, dim), or None if the fused kernels do not apply."""
    if not (x.is_cuda and weight.is_cuda) or x.dim() < 1 or x.stride(-1) != 1 or weight.dim() != 1:
        return None
    if x.dtype not in (torch.bfloat16, torch.float32) or weight.dtype not in (torch.bfloat16, torch.float32):
        return None
    if not weight.is_contiguous() or weight.shape[0] != x.shape[-1] or x.numel() == 0:
        return None
    if x.dim() == 1:
        return x.shape[-1]
    for d in range(x.dim() - 2):  # leading dims must collapse into one row index
        if x.stride(d) != x.shape[d + 1] * x.stride(d + 1):
            return None
    return x.stride(-2)


def _fused_norm_ok(x, weight) -> bool:
    return _row_stride(x, weight) is not None and not (torch.is_grad_enabled() and (x.requires_grad or
                                                                                   weight.requires_grad))


def _dtcode(t):
    from . import _capi as C

    return C.M3_DTYPE_BF16 if t.dtype == torch.bfloat16 else C.M3_DTYPE_F32


def _rms_norm_fused(x, weight, eps, rs, want_rstd=False):
    from . import _capi as C
    from . import _tensors as T

    dim = x.shape[-1]
    rows = x.numel() // dim
    y = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    rstd = torch.empty(rows, dtype=torch.float32, device=x.device) if want_rstd else None
    C.check(C.lib().m3_rms_norm(T.ptr(x), rs, T.ptr(weight), T.ptr(y), dim, rows, dim, float(eps), _dtcode(x),
                                _dtcode(weight), T.ptr(rstd), T.stream_handle(x.device)))
    return y, rstd


class _RMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, eps):
        y, rstd = _rms_norm_fused(x, weight, eps, _row_stride(x, weight), want_rstd=True)
        ctx.save_for_backward(x, weight, rstd)
        return y

    @staticmethod
    def backward(ctx, dy):
        from . import _capi as C
        from . import _tensors as T

        x, weight, rstd = ctx.saved_tensors
        dim = x.shape[-1]
        rows = x.numel() // dim
        dy = dy.contiguous()
        dx = torch.empty(x.shape, dtype=x.dtype, device=x.device)
        dw = torch.zeros(dim, dtype=torch.float32, device=x.device)
        C.check(C.lib().m3_rms_norm_bwd(T.ptr(x), _row_stride(x, weight), T.ptr(weight), T.ptr(rstd), T.ptr(dy), dim,
                                        T.ptr(dx), dim, T.ptr(dw), rows, dim, _dtcode(x), _dtcode(weight),
                                        T.stream_handle(x.device)))
        return dx, dw.to(weight.dtype), None


class _MixerFn(torch.autograd.Function):
    """The layer from the in_proj output to y (``layer.py:226-252``: split, B / C norms,
    the scan) as one autograd node, so that the backward writes every piece of the in_proj
    gradient straight into one buffer: dz / dx by the scan's backward through strided
    outputs, dB / dC by the norm backward's strided dx, the scalar columns by copies.  The
    forward also hands the scan's backward its workspace (the chunk-start states)."""

    @staticmethod
    def forward(ctx, proj, bnw, cnw, dt_bias, c_bias, b_bias, d_skip, s_ssm, s_k, s_v, s_phi, cfg):
        from . import kernel_bwd as KB
        from . import kernel_fwd as KF

        parts = _mixer_views(proj, cfg)
        z4, x4, b, c, raws = parts
        eps = cfg.norm_eps
        kn, rk = _rms_norm_fused(b, bnw, eps, _row_stride(b, bnw), want_rstd=True)
        qn, rq = _rms_norm_fused(c, cnw, eps, _row_stride(c, cnw), want_rstd=True)
        bsz, seqlen = proj.shape[0], proj.shape[1]
        h, p = cfg.nheads, cfg.headdim
        ws = torch.empty(KB.workspace_bytes(bsz, seqlen, h, cfg.d_state, p, cfg.n_angles, cfg.chunk),
                         dtype=torch.uint8, device=proj.device)
        y_out = torch.empty(bsz, seqlen, h, p, dtype=x4.dtype, device=proj.device).permute(0, 2, 1, 3)
        (y, fs, fk, fv, fphi), saved = KF.siso_forward_raw(
            qn, kn, x4, *raws, dt_bias, c_bias, b_bias, d_skip=d_skip, z=z4, seed_ssm=s_ssm, seed_k=s_k, seed_v=s_v,
            seed_phi=s_phi, a_floor=cfg.a_floor, chunk=cfg.chunk, dtype_policy=cfg.policy_name, y_out=y_out,
            bwd_states=ws, return_saved=True)
        ctx.save_for_backward(proj, bnw, cnw, dt_bias, c_bias, b_bias, d_skip, s_ssm, s_k, s_v, s_phi, qn, kn, rq, rk)
        ctx.cfg, ctx.ws, ctx.saved = cfg, ws, saved
        return y, fs, fk, fv, fphi

    @staticmethod
    def backward(ctx, dy, dfs, dfk, dfv, dfphi):
        from . import _capi as C
        from . import _tensors as T
        from . import kernel_bwd as KB

        (proj, bnw, cnw, dt_bias, c_bias, b_bias, d_skip, s_ssm, s_k, s_v, s_phi, qn, kn, rq, rk) = ctx.saved_tensors
        cfg = ctx.cfg
        z4, x4, b, c, raws = _mixer_views(proj, cfg)
        dproj = torch.empty(proj.shape, dtype=proj.dtype, device=proj.device)
        dz4, dx4, db, dc, draws = _mixer_views(dproj, cfg, convert_tail=False)
        if dy is None:
            dy = torch.zeros(x4.shape, dtype=x4.dtype, device=x4.device)
        g = KB.siso_backward_raw(
            dy, qn, kn, x4, *raws, dt_bias, c_bias, b_bias, d_skip=d_skip, z=z4, seed_ssm=s_ssm, seed_k=s_k,
            seed_v=s_v, seed_phi=s_phi, dfinal_ssm=dfs, dfinal_k=dfk, dfinal_v=dfv, dfinal_phi=dfphi,
            a_floor=cfg.a_floor, chunk=cfg.chunk, dtype_policy=cfg.policy_name, workspace=ctx.ws,
            states_ready=ctx.saved, grad_dtype=proj.dtype, dv_out=dx4, dz_out=dz4)
        ctx.ws = None
        dws = []
        for x, w, rstd, dn, dx in ((c, cnw, rq, g.dq, dc), (b, bnw, rk, g.dk, db)):
            dn = dn.to(proj.dtype).contiguous()  # the norm output's gradient in its own dtype
            dim = x.shape[-1]
            rows = x.numel() // dim
            dw = torch.zeros(dim, dtype=torch.float32, device=x.device)
            C.check(C.lib().m3_rms_norm_bwd(T.ptr(x), _row_stride(x, w), T.ptr(w), T.ptr(rstd), T.ptr(dn), dim,
                                            T.ptr(dx), _row_stride(dx, w), T.ptr(dw), rows, dim, _dtcode(x), _dtcode(w),
                                            T.stream_handle(x.device)))
            dws.append(dw.to(w.dtype))
        for dst, src in zip(draws, (g.ddt_raw, g.da_raw, g.dtrap_raw, g.dangles)):
            dst.copy_(src)

        def like(x, ref):
            return None if (ref is None or x is None) else x.to(ref.dtype)

        return (dproj, dws[1], dws[0], like(g.ddt_bias, dt_bias), like(g.dq_bias, c_bias), like(g.dk_bias, b_bias),
                like(g.dd_skip, d_skip), like(g.dseed_ssm, s_ssm), like(g.dseed_k, s_k), like(g.dseed_v, s_v),
                like(g.dseed_phi, s_phi), None)


def _mixer_views(proj, cfg, convert_tail=True):
    """z, x as (B, H, L, P) views, B, C, and the four scalar-column views of one in_proj output."""
    h, n = cfg.nheads, cfg.d_state
    z, x, b, c, tail = torch.split(proj, (cfg.d_inner, cfg.d_inner, n, n, 3 * h + cfg.n_angles), dim=-1)
    z4 = z.unflatten(-1, (h, cfg.headdim)).permute(0, 2, 1, 3)
    x4 = x.unflatten(-1, (h, cfg.headdim)).permute(0, 2, 1, 3)
    if convert_tail and tail.dtype != torch.float32:
        tail = tail.float()
    return z4, x4, b, c, (tail[..., :h], tail[..., h:2 * h], tail[..., 2 * h:3 * h], tail[..., 3 * h:])


def _mixer_fn_ok(proj, params, cfg) -> bool:
    if not (torch.is_grad_enabled() and proj.is_cuda and proj.dim() == 3 and proj.is_contiguous()):
        return False
    if proj.dtype not in (torch.bfloat16, torch.float32) or cfg.d_state > 2048:
        return False
    n, d = cfg.d_state, 2 * cfg.d_inner
    b = proj[..., d:d + n]
    return _row_stride(b, params.b_norm_weight) is not None and params.b_norm_weight.is_cuda


def mamba3_siso_layer(params: SISOParams, u: torch.Tensor, cfg: SISOConfig, state: Optional[SISOState] = None,
                      interpret=False, device_kind=None):
    """``layer.py:201-262``: ``u (B, L, d_model)`` -> ``(out (B, L, d_model), SISOState)``.
    ``interpret`` / ``device_kind`` (TPU options of the reference) have no effect."""
    bsz, seqlen, _ = u.shape
    proj = torch.matmul(u, params.in_proj.to(u.dtype))
    if _mixer_fn_ok(proj, params, cfg):  # training: one autograd node, one in_proj gradient buffer
        s = state
        y, fs, fk, fv, fphi = _MixerFn.apply(
            proj, params.b_norm_weight, params.c_norm_weight, params.dt_bias, params.c_bias, params.b_bias,
            params.d_skip, None if s is None else s.ssm, None if s is None else s.k, None if s is None else s.v,
            None if s is None else s.phi, cfg)
        y = y.permute(0, 2, 1, 3).reshape(bsz, seqlen, cfg.d_inner)
        return (torch.matmul(y.to(u.dtype), params.out_proj.to(u.dtype)),
                SISOState(ssm=fs, k=fk, v=fv, phi=fphi))
    # one split of proj (z, x, B, C, the scalar columns), so that autograd assembles the
    # in_proj gradient with one concatenation instead of zero-filled slices added together
    h, n = cfg.nheads, cfg.d_state
    z, x, b, c, tail = torch.split(proj, (cfg.d_inner, cfg.d_inner, n, n, 3 * h + cfg.n_angles), dim=-1)
    z, x = z.unflatten(-1, (h, cfg.headdim)), x.unflatten(-1, (h, cfg.headdim))
    if tail.dtype != torch.float32:
        tail = tail.float()
    dt_raw, a_raw, trap_raw, angles = tail[..., :h], tail[..., h:2 * h], tail[..., 2 * h:3 * h], tail[..., 3 * h:]
    b = rms_norm(b, params.b_norm_weight, cfg.norm_eps)
    c = rms_norm(c, params.c_norm_weight, cfg.norm_eps)
    out = SISO.siso_segment(
        q=c, k=b, v=x.permute(0, 2, 1, 3), dt_raw=dt_raw, a_raw=a_raw, trap_raw=trap_raw, angles=angles,
        dt_bias=params.dt_bias, q_bias=params.c_bias, k_bias=params.b_bias, d_skip=params.d_skip,
        z=z.permute(0, 2, 1, 3), state=state, a_floor=cfg.a_floor, chunk=cfg.chunk,
        policy_name=cfg.policy_name, y_blhp=True)
    y = out.y.permute(0, 2, 1, 3).reshape(bsz, seqlen, cfg.d_inner)
    return torch.matmul(y.to(u.dtype), params.out_proj.to(u.dtype)), out.state
