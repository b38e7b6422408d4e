"""Dtype policy, chunk rules and the rotary permutation.

Mirrors the host-side parts of ``mamba3_pallas/layout.py`` that callers use; the TPU
BlockSpec / VMEM / Mosaic-lowering machinery there has no counterpart on B200.
"""

from __future__ import annotations

import dataclasses
import functools

import torch

POLICIES = ("bf16", "f32")


@dataclasses.dataclass(frozen=True)
class DtypePolicy:
    """``layout.py:243-282``: the dtype of each role.  bf16 matmul operands with fp32
    accumulation (the production setting), or fp32 throughout (the parity setting).  On
    B200 an fp32 contraction is true fp32 (there is no silent truncation to undo), so
    ``highest`` only names the setting."""

    name: str = "bf16"
    matmul: torch.dtype = torch.bfloat16
    accum: torch.dtype = torch.float32
    state: torch.dtype = torch.float32
    saved_state: torch.dtype = torch.bfloat16

    @property
    def highest(self) -> bool:
        return self.matmul == torch.float32

    def __eq__(self, other):  # a policy also compares equal to its name
        if isinstance(other, str):
            return self.name == other
        return dataclasses.astuple(self) == dataclasses.astuple(other) if isinstance(other, DtypePolicy) else False

    def __hash__(self):
        return hash(self.name)

    def __str__(self):
        return self.name


#: Production setting: bf16 operands, fp32 accumulate.
BF16 = DtypePolicy()
#: Validation setting: everything fp32.
F32 = DtypePolicy(name="f32", matmul=torch.float32, saved_state=torch.float32)


def policy(name) -> DtypePolicy:
    """``layout.py:284-291``: a policy by name (``"bf16"`` / ``"bfloat16"`` / ``"default"``
    or ``"f32"`` / ``"fp32"`` / ``"float32"`` / ``"highest"``); a `DtypePolicy` passes through."""
    if isinstance(name, DtypePolicy):
        return name
    key = name.strip().lower()
    if key in ("bf16", "bfloat16", "default"):
        return BF16
    if key in ("f32", "fp32", "float32", "highest"):
        return F32
    raise ValueError(f"Unknown dtype policy {name!r}; want 'bf16' or 'f32'")


def validate_chunk(chunk: int) -> None:
    """Chunk must be a positive multiple of 64.

    The reference requires a multiple of 128 (``layout.py:225-235``) because Mosaic puts
    the chunk on the 128-wide lane axis.  These kernels have no such rule; 64 is the
    granularity of their internal tiling, and the recurrence is chunk-invariant.
    """
    if chunk <= 0 or chunk % 64 != 0:
        raise ValueError(f"chunk must be a positive multiple of 64, got {chunk}")


def num_chunks(seqlen: int, chunk: int) -> int:
    """``layout.py:500-506``."""
    if seqlen % chunk != 0:
        raise ValueError(
            f"seqlen ({seqlen}) must be a multiple of chunk ({chunk}); pad the sequence before calling.")
    return seqlen // chunk


@functools.lru_cache(maxsize=None)
def deinterleave_perm(n: int) -> torch.Tensor:
    """``layout.py:299-321``: ``new[j] = old[2j]``, ``new[n/2 + j] = old[2j + 1]``."""
    if n % 2 != 0:
        raise ValueError(f"state dim must be even for rotary pairing, got {n}")
    return torch.cat([torch.arange(0, n, 2), torch.arange(1, n, 2)])


@functools.lru_cache(maxsize=None)
def interleave_perm(n: int) -> torch.Tensor:
    """``layout.py:324-327``: inverse of `deinterleave_perm`."""
    return torch.argsort(deinterleave_perm(n))


def apply_perm(x: torch.Tensor, axis: int = -1) -> torch.Tensor:
    return torch.index_select(x, axis, deinterleave_perm(x.shape[axis]).to(x.device))


def unapply_perm(x: torch.Tensor, axis: int = -1) -> torch.Tensor:
    return torch.index_select(x, axis, interleave_perm(x.shape[axis]).to(x.device))


# --------------------------------------------------------------------------------------
# Rotation and in-chunk sums as torch (the kernels do these in registers)
# --------------------------------------------------------------------------------------


def rope_cos_sin(phi: torch.Tensor, state_dim: int):
    """``layout.py:345-372``: full-width ``(..., N)`` cos / sin for the half-split rotation
    from ``(..., n_angles)`` angles; pairs past ``n_angles`` get cos 1, sin 0."""
    half = state_dim // 2
    n_angles = phi.shape[-1]
    if n_angles > half:
        raise ValueError(f"n_angles ({n_angles}) exceeds state_dim // 2 ({half})")
    if n_angles < half:
        phi = torch.cat([phi, phi.new_zeros(*phi.shape[:-1], half - n_angles)], dim=-1)
    full = torch.cat([phi, phi], dim=-1)
    return torch.cos(full), torch.sin(full)


def rope_apply(x: torch.Tensor, cos_full: torch.Tensor, sin_full: torch.Tensor) -> torch.Tensor:
    """``layout.py:375-398``: ``x cos + rot_half(x) sin`` with ``rot_half = [-hi, lo]``."""
    half = x.shape[-1] // 2
    rot = torch.cat([-x[..., half:], x[..., :half]], dim=-1)
    return x * cos_full + rot * sin_full


def rope_dphi(x_rot: torch.Tensor, dx_rot: torch.Tensor, n_angles: int) -> torch.Tensor:
    """``layout.py:414-428``: angle gradient of a rotation from the rotated value and its
    cotangent, ``dhi * lo - dlo * hi`` over the first ``n_angles`` pairs."""
    half = x_rot.shape[-1] // 2
    lo, hi = x_rot[..., :half], x_rot[..., half:]
    return (dx_rot[..., half:] * lo - dx_rot[..., :half] * hi)[..., :n_angles]


def tril_ones(n: int, dtype: torch.dtype = torch.float32, device=None) -> torch.Tensor:
    """``layout.py:436-443``: ``(n, n)`` lower-triangular ones, diagonal included."""
    return torch.tril(torch.ones(n, n, dtype=dtype, device=device))


def prefix_sum(row: torch.Tensor, tril: torch.Tensor = None) -> torch.Tensor:
    """``layout.py:453-477``: inclusive prefix sum of a ``(1, n)`` row (or over the last
    axis of any tensor) in fp32; ``(n,)`` for a single row like the reference.  ``tril`` is
    accepted for signature compatibility (the kernels use warp scans)."""
    out = torch.cumsum(row.float(), dim=-1)
    return out[0] if row.dim() == 2 and row.shape[0] == 1 else out


def suffix_sum(row: torch.Tensor, tril: torch.Tensor = None) -> torch.Tensor:
    """``layout.py:480-497``: inclusive reverse prefix sum, ``out[t] = sum_{s >= t} row[s]``."""
    out = torch.flip(torch.cumsum(torch.flip(row.float(), dims=[-1]), dim=-1), dims=[-1])
    return out[0] if row.dim() == 2 and row.shape[0] == 1 else out
