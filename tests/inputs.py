"""Seeded kernel-boundary inputs with the reference test suite's distributions
(``mamba3_pallas/tests.py:179-212``), drawn with ``torch.Generator`` on the CPU.

``jax.random`` streams cannot be reproduced without JAX, so the values differ from the
reference's; both sides of every parity check are fed these same tensors.
"""

import math

import torch


def make_inputs(batch, nheads, seqlen, state_dim=128, headdim=64, n_angles=32, seed=0,
                dtype=torch.float64):
    g = torch.Generator().manual_seed(seed)

    def rn(*shape, scale=1.0):
        return torch.randn(*shape, generator=g, dtype=torch.float64) * scale

    def norm_rows(x):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6)

    b, h, l, n, p, nr = batch, nheads, seqlen, state_dim, headdim, n_angles
    q = norm_rows(rn(b, l, n))
    k = norm_rows(rn(b, l, n))
    v = rn(b, h, l, p)
    z = rn(b, h, l, p)
    dt = torch.exp(torch.rand(b, l, h, generator=g, dtype=torch.float64)
                   * (math.log(0.1) - math.log(0.001)) + math.log(0.001))
    x = {
        "q": q, "k": k, "v": v, "z": z,
        # inverse softplus of dt, so preprocess recovers dt exactly (dt_bias = 0)
        "dt_raw": torch.log(torch.expm1(dt)),
        "a_raw": rn(b, l, h),
        "trap_raw": rn(b, l, h),
        "angles": rn(b, l, nr, scale=0.5),
        "dt_bias": torch.zeros(h, dtype=torch.float64),
        "q_bias": rn(h, n, scale=0.1),
        "k_bias": rn(h, n, scale=0.1),
        "d_skip": rn(h),
        "dy": rn(b, h, l, p),
    }
    return {kk: vv.to(dtype) for kk, vv in x.items()}
