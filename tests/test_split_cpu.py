"""Host-side rules of the forward's length split (`kernel_fwd._auto_split`,
`kernel_fwd._forward_raw_split`): the automatic segment count fills the SMs once, pays only
from 3 segments, divides the chunk count and stays within the carry kernel's 64 segments; an
explicit split that does not divide the chunks is refused before anything is launched."""

import pytest
import torch


def _shapes(b, h, l, n=128, p=64, nr=64):
    q = torch.zeros(b, l, n, dtype=torch.bfloat16)
    v = torch.zeros(b, h, l, p, dtype=torch.bfloat16)
    ang = torch.zeros(b, l, nr)
    return q, v, ang


@pytest.mark.parametrize("b,h,l,want", [
    (1, 32, 8192, 4),     # 32 sequences, 64 chunks: 4 segments -> 128 CTAs
    (2, 32, 8192, 1),     # 64 sequences: only 2 segments fit, which do not pay
    (8, 32, 8192, 1),     # 256 sequences already fill the GPU
    (1, 1, 2 ** 20, 64),  # one sequence of 8192 chunks: capped at the carry kernel's 64
    (1, 8, 1024, 1),      # 8 chunks: a segment needs at least 8
])
def test_auto_split_rule(b, h, l, want, monkeypatch):
    from mamba3_b200 import kernel_fwd as KF

    monkeypatch.setattr(KF, "_sm_count", lambda dev: 148)
    q, v, ang = _shapes(b, h, l)
    assert KF._auto_split(q, v, ang, 128, "bf16", "auto") == want


def test_auto_split_only_for_the_tensor_core_forward(monkeypatch):
    from mamba3_b200 import kernel_fwd as KF

    monkeypatch.setattr(KF, "_sm_count", lambda dev: 148)
    q, v, ang = _shapes(1, 32, 8192)
    assert KF._auto_split(q, v, ang, 128, "f32", "auto") == 1
    assert KF._auto_split(q, v, ang, 128, "bf16", "generic") == 1
    q2, v2, ang2 = _shapes(1, 32, 8192, n=64, p=64, nr=32)
    assert KF._auto_split(q2, v2, ang2, 128, "bf16", "auto") == 1


def test_explicit_split_must_divide_the_chunks():
    from mamba3_b200 import kernel_fwd as KF

    q, v, ang = _shapes(1, 4, 768)  # 6 chunks
    raw = torch.zeros(1, 768, 4)
    args = (q, q, v, raw, raw, raw, ang, torch.zeros(4), torch.zeros(4, 128), torch.zeros(4, 128))
    with pytest.raises(ValueError, match="equal segments"):
        KF.siso_forward_raw(*args, chunk=128, dtype_policy="bf16", lsplit=4)
