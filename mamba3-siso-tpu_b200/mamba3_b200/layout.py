"""Dtype policy, chunk rules and the rotary permutation.

Mirrors the host-side parts of ``mamba3_pallas/layout.py`` that callers use; the TPU
BlockSpec / VMEM / Mosaic-lowering machinery there has no counterpart on B200.
"""

from __future__ import annotations

import functools

import torch

POLICIES = ("bf16", "f32")


def policy(name: str) -> str:
    """``layout.py:284-291``: normalise a policy name to ``"bf16"`` or ``"f32"``."""
    key = name.strip().lower()
    if key in ("bf16", "bfloat16", "default"):
        return "bf16"
    if key in ("f32", "fp32", "float32", "highest"):
        return "f32"
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
