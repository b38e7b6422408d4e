"""Generate the golden fixtures that pin the oracle to the reference's own code.

Run in a container where the reference checkout is available::

    python tests/golden/make_golden.py /path/to/mamba3-siso-tpu

It imports ``mamba3_pallas/torch_ref.py`` (plain torch; the reference package's
``__init__`` needs JAX, so the file is loaded on its own) and runs

* ``mamba3_siso_ref`` (``torch_ref.py:64-138``) -- the reference's recurrent kernel-
  boundary reference, in the interleaved rotary layout, float64;
* ``Mamba3SISOTorch.forward`` (``torch_ref.py:141-237``) -- the reference's torch layer.

Inputs are written in the half-split ("permuted") layout the oracle and the CUDA
library use (``layout.py:299-321``); outputs that live on the state axis are permuted
the same way.  Nothing at test time reads the reference checkout: the fixtures are
committed as ``tests/golden/*.npz``.
"""

from __future__ import annotations

import importlib.util
import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _load_torch_ref(root: str):
    path = os.path.join(root, "mamba3_pallas", "torch_ref.py")
    spec = importlib.util.spec_from_file_location("ref_torch_ref", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _perm(n):
    return np.concatenate([np.arange(0, n, 2), np.arange(1, n, 2)])


def kernel_case(tr, name, b, h, l, n, p, nr, seed):
    g = torch.Generator().manual_seed(seed)
    f64 = torch.float64
    perm = torch.as_tensor(_perm(n))
    inv = torch.argsort(perm)

    def rn(*s, scale=1.0):
        return torch.randn(*s, generator=g, dtype=f64) * scale

    q = rn(b, l, n)
    q = q / q.pow(2).mean(-1, keepdim=True).sqrt()
    k = rn(b, l, n)
    k = k / k.pow(2).mean(-1, keepdim=True).sqrt()
    v = rn(b, h, l, p)
    z = rn(b, h, l, p)
    dt = torch.exp(torch.rand(b, h, l, generator=g, dtype=f64) * (math.log(0.1) - math.log(1e-3)) + math.log(1e-3))
    a = -(1.0 + torch.rand(h, generator=g, dtype=f64) * 3.0)
    adt = a[None, :, None] * dt
    trap = rn(b, h, l)
    angles = rn(b, l, nr, scale=0.5)
    q_bias = rn(h, n, scale=0.1)
    k_bias = rn(h, n, scale=0.1)
    d_skip = rn(h)

    # torch_ref wants per-head interleaved Q/K (B,L,H,N), V/Z (B,L,H,P), per-head raw angles.
    Q = q[..., inv][:, :, None, :].expand(b, l, h, n).contiguous()
    K = k[..., inv][:, :, None, :].expand(b, l, h, n).contiguous()
    V = v.permute(0, 2, 1, 3).contiguous()
    Z = z.permute(0, 2, 1, 3).contiguous()
    Ang = angles[:, :, None, :].expand(b, l, h, nr).contiguous()
    out, (ang_s, ssm_s, k_s, v_s) = tr.mamba3_siso_ref(
        Q, K, V, adt, dt, trap, q_bias[:, inv], k_bias[:, inv], Ang, D=d_skip, Z=Z)
    out_nz, _ = tr.mamba3_siso_ref(
        Q, K, V, adt, dt, trap, q_bias[:, inv], k_bias[:, inv], Ang)
    np.savez_compressed(
        os.path.join(HERE, f"{name}.npz"),
        q=q.numpy(), k=k.numpy(), v=v.numpy(), z=z.numpy(), adt=adt.numpy(), dt=dt.numpy(),
        trap=trap.numpy(), angles=angles.numpy(), q_bias=q_bias.numpy(), k_bias=k_bias.numpy(),
        d_skip=d_skip.numpy(),
        y=out.permute(0, 2, 1, 3).numpy(),
        y_nogate_noskip=out_nz.permute(0, 2, 1, 3).numpy(),
        ssm=ssm_s[..., perm].numpy(), k_final=k_s[..., perm].numpy(), v_final=v_s.numpy(),
        phi_final=ang_s.numpy(),
    )


def layer_case(tr, name, d_model, d_state, headdim, rope_fraction, b, l, seed):
    torch.manual_seed(seed)
    mod = tr.Mamba3SISOTorch(d_model=d_model, d_state=d_state, headdim=headdim,
                             rope_fraction=rope_fraction, dtype=torch.float64)
    mod = mod.double()
    with torch.no_grad():
        # non-trivial biases, gains and skip so their placement is pinned
        mod.B_bias.add_(0.1 * torch.randn_like(mod.B_bias))
        mod.C_bias.add_(0.1 * torch.randn_like(mod.C_bias))
        mod.B_norm_weight.add_(0.1 * torch.randn_like(mod.B_norm_weight))
        mod.C_norm_weight.add_(0.1 * torch.randn_like(mod.C_norm_weight))
        mod.D.add_(0.1 * torch.randn_like(mod.D))
    u = torch.randn(b, l, d_model, dtype=torch.float64) * 0.5
    y = mod(u)
    sd = {kk: vv.detach().numpy() for kk, vv in mod.state_dict().items()}
    np.savez_compressed(
        os.path.join(HERE, f"{name}.npz"), u=u.numpy(), y=y.numpy(),
        d_model=d_model, d_state=d_state, headdim=headdim, rope_fraction=rope_fraction,
        **{"sd__" + kk.replace(".", "__"): vv for kk, vv in sd.items()},
    )


def main(root):
    tr = _load_torch_ref(root)
    kernel_case(tr, "recurrent_n16_p16_nr4", b=2, h=3, l=128, n=16, p=16, nr=4, seed=0)
    kernel_case(tr, "recurrent_n32_p16_nr16", b=1, h=2, l=128, n=32, p=16, nr=16, seed=1)
    layer_case(tr, "layer_d32_n16_p16", d_model=32, d_state=16, headdim=16, rope_fraction=0.5,
               b=2, l=128, seed=2)
    print("wrote fixtures to", HERE)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_golden.py <reference checkout>")
    main(sys.argv[1])
