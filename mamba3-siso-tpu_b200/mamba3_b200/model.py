"""Stacked Mamba-3 SISO language model (``mamba3_pallas/model.py``).

Pre-norm residual blocks, optional gated MLP on its own residual, tied head.  Prefill
goes through `layer.mamba3_siso_layer` (chunked scan kernels); decode goes through the
in-place decode kernel with the length-1 preprocess fused (`lm_decode_step`).
"""

from __future__ import annotations

import dataclasses
import math
from typing import List, NamedTuple, Optional

import torch
import torch.nn.functional as F

from . import kernel_decode as KD
from . import layer as LY
from . import projection as PJ
from .state import SISOState, zero_state


@dataclasses.dataclass(frozen=True)
class LMConfig:
    """``model.py:39-92``."""

    vocab_size: int
    n_layers: int
    siso: LY.SISOConfig
    tie_head: bool = True
    d_intermediate: int = 0

    @property
    def d_model(self) -> int:
        return self.siso.d_model

    def param_count(self) -> int:
        c = self.siso
        per_layer = (c.d_model * c.d_in_proj + c.d_inner * c.d_model + c.nheads * 2 + c.d_state * 2
                     + c.nheads * c.d_state * 2 + c.d_model)
        if self.d_intermediate:
            per_layer += c.d_model * 2 * self.d_intermediate + self.d_intermediate * c.d_model + c.d_model
        head = 0 if self.tie_head else self.d_model * self.vocab_size
        return self.vocab_size * self.d_model + self.n_layers * per_layer + self.d_model + head


class MLPParams(NamedTuple):
    fc1: torch.Tensor   # (d_model, 2 * d_intermediate): value half first, gate half second
    fc2: torch.Tensor   # (d_intermediate, d_model)


class BlockParams(NamedTuple):
    norm_gain: torch.Tensor
    siso: LY.SISOParams
    mlp_norm_gain: Optional[torch.Tensor] = None
    mlp: Optional[MLPParams] = None


class LMParams(NamedTuple):
    embed: torch.Tensor
    blocks: List[BlockParams]
    final_norm: torch.Tensor
    head: Optional[torch.Tensor]


def gated_mlp(p: MLPParams, x: torch.Tensor) -> torch.Tensor:
    """``model.py:125-137``: ``fc2(value * silu(gate))``."""
    h = torch.matmul(x, p.fc1.to(x.dtype))
    value, gate = h.chunk(2, dim=-1)
    return torch.matmul(value * F.silu(gate), p.fc2.to(x.dtype))


def init_lm(cfg: LMConfig, key=0, dtype=torch.float32, device="cuda") -> LMParams:
    """``model.py:141-191``: N(0, 0.02) embedding, per-layer `init_params` with out_proj
    (and fc2) scaled by ``1/sqrt(2 n_layers)``."""
    g = key if isinstance(key, torch.Generator) else torch.Generator().manual_seed(int(key))
    to = dict(dtype=dtype, device=device)
    embed = (torch.randn(cfg.vocab_size, cfg.d_model, generator=g) * 0.02).to(**to)
    resid = 1.0 / math.sqrt(2.0 * cfg.n_layers)
    di = cfg.d_intermediate
    blocks = []
    for _ in range(cfg.n_layers):
        p = LY.init_params(cfg.siso, g, dtype=dtype, device=device)
        p = p._replace(out_proj=p.out_proj * resid)
        mlp = mlp_norm = None
        if di:
            fc1 = (torch.randn(cfg.d_model, 2 * di, generator=g) / math.sqrt(cfg.d_model)).to(**to)
            fc2 = (torch.randn(di, cfg.d_model, generator=g) / math.sqrt(di) * resid).to(**to)
            mlp = MLPParams(fc1=fc1, fc2=fc2)
            mlp_norm = torch.ones(cfg.d_model, **to)
        blocks.append(BlockParams(norm_gain=torch.ones(cfg.d_model, **to), siso=p, mlp_norm_gain=mlp_norm, mlp=mlp))
    head = None if cfg.tie_head else (torch.randn(cfg.d_model, cfg.vocab_size, generator=g) * 0.02).to(**to)
    return LMParams(embed=embed, blocks=blocks, final_norm=torch.ones(cfg.d_model, **to), head=head)


def lm_forward(params: LMParams, tokens: torch.Tensor, cfg: LMConfig, interpret=False, device_kind=None,
               states: Optional[List[SISOState]] = None, compute_dtype: Optional[torch.dtype] = None,
               return_hidden: bool = False, logits: str = "all"):
    """``model.py:194-232``: ``(B, L)`` tokens -> ``(B, L, vocab)`` logits (and the
    per-layer carry when ``states`` is given).  ``logits="last"`` computes the head for
    the final position only (``(B, vocab)``), ``"none"`` skips it (prefill for decode).
    ``interpret`` / ``device_kind`` keep the reference's argument order; no effect here."""
    x = params.embed[tokens]
    if compute_dtype is not None:
        x = x.to(compute_dtype)
    eps = cfg.siso.norm_eps
    new_states = []
    for i, b in enumerate(params.blocks):
        h = LY.rms_norm(x, b.norm_gain, eps)
        y, st = LY.mamba3_siso_layer(b.siso, h, cfg.siso, state=None if states is None else states[i])
        new_states.append(st)
        x = x + y
        if b.mlp is not None:
            x = x + gated_mlp(b.mlp, LY.rms_norm(x, b.mlp_norm_gain, eps))
    x = LY.rms_norm(x, params.final_norm, eps)
    if return_hidden:
        return x
    head = params.embed.t() if cfg.tie_head else params.head
    if logits == "none":
        out = None
    elif logits == "last":
        out = torch.matmul(x[:, -1], head.to(x.dtype))
    else:
        out = torch.matmul(x, head.to(x.dtype))
    return (out, new_states) if states is not None else out


def zero_states(cfg: LMConfig, batch: int, dtype=torch.float32, device="cuda") -> List[SISOState]:
    """``model.py:235-241``."""
    c = cfg.siso
    return [zero_state(batch, c.nheads, c.headdim, c.d_state, c.n_angles, dtype=torch.float32, device=device)
            for _ in range(cfg.n_layers)]


@torch.no_grad()
def lm_decode_step(params: LMParams, token: torch.Tensor, states: List[SISOState], cfg: LMConfig,
                   interpret=False, compute_dtype: Optional[torch.dtype] = None):
    """``model.py:244-296``: one token per sequence, ``(B,)`` -> ``(B, vocab)`` logits.
    The per-layer states are updated in place by the decode kernel."""
    c = cfg.siso
    x = params.embed[token]
    if compute_dtype is not None:
        x = x.to(compute_dtype)
    out_states = []
    small = PJ.eligible(x, params.blocks[0].siso.in_proj) if params.blocks else False
    for i, blk in enumerate(params.blocks):
        p = blk.siso
        if small:  # batch <= 8, bf16: W streamed by m3_gemv_bf16 with the norm folded in
            proj = PJ.small_proj(x, p.in_proj, norm_w=blk.norm_gain, eps=c.norm_eps)
        else:
            h = LY.rms_norm(x, blk.norm_gain, c.norm_eps)
            proj = torch.matmul(h, p.in_proj.to(h.dtype))
        z, xx, b, cc, _, _, _, _ = LY.split_in_proj(proj, c)
        s0 = 2 * c.d_inner + 2 * c.d_state  # dt / A / trap / angle columns, read in place
        hh = c.nheads
        dt_raw, a_raw, trap_raw = proj[:, s0:s0 + hh], proj[:, s0 + hh:s0 + 2 * hh], proj[:, s0 + 2 * hh:s0 + 3 * hh]
        angles = proj[:, s0 + 3 * hh:]
        # the B / C norms run inside the decode kernel
        y, st = KD.siso_decode_raw(cc, b, xx, dt_raw, a_raw, trap_raw, angles, p.dt_bias, p.c_bias, p.b_bias,
                                   states[i], d_skip=p.d_skip, z=z, a_floor=c.a_floor, dtype_policy=c.policy_name,
                                   q_norm_w=p.c_norm_weight, k_norm_w=p.b_norm_weight, norm_eps=c.norm_eps)
        out_states.append(st)
        # residual adds fused into the projections
        y2 = y.reshape(y.shape[0], c.d_inner).to(x.dtype)
        if small:
            x = PJ.small_proj(y2, p.out_proj, residual=x)
        else:
            x = torch.addmm(x, y2, p.out_proj.to(x.dtype))
        if blk.mlp is not None:
            if small:
                hm = PJ.small_proj(x, blk.mlp.fc1, norm_w=blk.mlp_norm_gain, eps=c.norm_eps)
                x = PJ.small_proj(hm, blk.mlp.fc2, silu_gate=True, residual=x)
            else:
                hm = torch.matmul(LY.rms_norm(x, blk.mlp_norm_gain, c.norm_eps), blk.mlp.fc1.to(x.dtype))
                x = torch.addmm(x, PJ.gated_act(hm), blk.mlp.fc2.to(x.dtype))
    x = LY.rms_norm(x, params.final_norm, c.norm_eps)
    head = params.embed.t() if cfg.tie_head else params.head
    return torch.matmul(x, head.to(x.dtype)), out_states


class DecodeGraph:
    """`lm_decode_step` captured once in a CUDA graph and replayed per token.

    The decode step is ~25 small launches per layer; replaying a graph removes the host
    launch cost between them.  The per-layer states are the graph's own buffers and are
    updated in place by every `step` (the capture leaves them as they were).
    """

    def __init__(self, params: LMParams, cfg: LMConfig, states: List[SISOState], batch: int,
                 compute_dtype: Optional[torch.dtype] = None):
        dev = params.embed.device
        self.states = states
        self.tok = torch.zeros(batch, dtype=torch.long, device=dev)
        snap = [[t.clone() for t in st] for st in states]
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(2):
                lm_decode_step(params, self.tok, states, cfg, compute_dtype=compute_dtype)
        torch.cuda.current_stream(dev).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.logits, _ = lm_decode_step(params, self.tok, states, cfg, compute_dtype=compute_dtype)
        for st, sn in zip(states, snap):
            for t, s0 in zip(st, sn):
                t.copy_(s0)

    def step(self, token: torch.Tensor) -> torch.Tensor:
        """One token for every sequence; returns the ``(B, vocab)`` logits buffer."""
        self.tok.copy_(token)
        self.graph.replay()
        return self.logits
