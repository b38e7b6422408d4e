"""Helpers for the GPU parity tests: move seeded oracle inputs to the device and run the
oracle (float64, CPU) on the same tensors."""

import torch

from oracle import siso_oracle as O
from tests.inputs import make_inputs

DEV = "cuda"


def dev(x, dtype=torch.float32):
    return None if x is None else x.to(device=DEV, dtype=dtype)


def cpu64(x):
    return None if x is None else x.detach().to("cpu", torch.float64)


def pre_inputs(b, h, l, n, p, nr, seed=0):
    x = make_inputs(b, h, l, state_dim=n, headdim=p, n_angles=nr, seed=seed)
    pre, _ = O.preprocess(x["dt_raw"], x["a_raw"], x["trap_raw"], x["angles"], x["dt_bias"])
    return x, pre


def rand_state(b, h, p, n, nr, seed=31):
    g = torch.Generator().manual_seed(seed)
    return O.SISOState(
        ssm=torch.randn(b, h, p, n, generator=g, dtype=torch.float64) * 0.5,
        k=torch.randn(b, h, n, generator=g, dtype=torch.float64),
        v=torch.randn(b, h, p, generator=g, dtype=torch.float64),
        phi=torch.rand(b, h, nr, generator=g, dtype=torch.float64) * 6.0,
    )
