"""Backward kernel parity: every cotangent against float64 autograd through the oracle
(the reference's own gradient oracle is ``jax.grad`` of ``siso_chunked``,
``reference.py:313-316``; ``mamba3_pallas/tests.py:573-645``)."""

import pytest
import torch

from oracle import siso_oracle as O
from tests.gpu_common import DEV, cpu64, dev, pre_inputs, rand_state
from tests.metrics import rel_error

pytestmark = pytest.mark.gpu
F32_GRAD_TOL = 1e-5
BF16_GRAD_TOL = 2e-2


def _leaf(t):
    return t.clone().requires_grad_(True)


@pytest.mark.parametrize("shape", [(2, 3, 256, 128, 64, 32, 128), (2, 16, 128, 32, 32, 8, 64),
                                   (1, 2, 128, 16, 16, 4, 64)])
@pytest.mark.parametrize("seeded", [False, True])
def test_pre_boundary_grads_f32(shape, seeded):
    from mamba3_b200 import kernel_bwd as KB

    b, h, l, n, p, nr, chunk = shape
    x, pre = pre_inputs(b, h, l, n, p, nr, seed=21)
    g = torch.Generator().manual_seed(5)
    st = rand_state(b, h, p, n, nr) if seeded else None
    coef = torch.rand(b, h, generator=g, dtype=torch.float64) * 0.05 if seeded else None
    dfs = torch.randn(b, h, p, n, generator=g, dtype=torch.float64) * 0.1
    dfk = torch.randn(b, h, n, generator=g, dtype=torch.float64) * 0.1
    dfv = torch.randn(b, h, p, generator=g, dtype=torch.float64) * 0.1
    names = ["q", "k", "v", "adt", "gamma", "scale", "phi", "q_bias", "k_bias", "d_skip", "z"]
    vals = dict(q=x["q"], k=x["k"], v=x["v"], adt=pre.adt, gamma=pre.gamma, scale=pre.scale, phi=pre.phi,
                q_bias=x["q_bias"], k_bias=x["k_bias"], d_skip=x["d_skip"], z=x["z"])
    leaves = {k_: _leaf(v_) for k_, v_ in vals.items()}
    sl = None
    if seeded:
        sl = {k_: _leaf(v_) for k_, v_ in dict(ssm=st.ssm, k=st.k, v=st.v, coef=coef).items()}
        state = O.SISOState(sl["ssm"], sl["k"], sl["v"], st.phi)
        y, fin = O.siso_chunked(*(leaves[k_] for k_ in names), state=state, seed_dt=sl["coef"],
                                seed_lam=torch.zeros_like(coef), chunk=chunk)
    else:
        y, fin = O.siso_chunked(*(leaves[k_] for k_ in names), chunk=chunk)
    loss = (y * x["dy"]).sum() + (fin.ssm * dfs).sum() + (fin.k * dfk).sum() + (fin.v * dfv).sum()
    loss.backward()

    gk = KB.siso_backward(dev(x["dy"]), dev(x["q"]), dev(x["k"]), dev(x["v"]), dev(pre.adt), dev(pre.gamma),
                          dev(pre.scale), dev(pre.phi), dev(x["q_bias"]), dev(x["k_bias"]), d_skip=dev(x["d_skip"]),
                          z=dev(x["z"]), seed_ssm=dev(st.ssm) if seeded else None,
                          seed_k=dev(st.k) if seeded else None, seed_v=dev(st.v) if seeded else None,
                          seed_coef=dev(coef) if seeded else None, dfinal_ssm=dev(dfs), dfinal_k=dev(dfk),
                          dfinal_v=dev(dfv), chunk=chunk, dtype_policy="f32")
    pairs = dict(q=gk.dq, k=gk.dk, v=gk.dv, adt=gk.dadt, gamma=gk.dgamma, scale=gk.dscale, phi=gk.dphi,
                 q_bias=gk.dq_bias, k_bias=gk.dk_bias, d_skip=gk.dd_skip, z=gk.dz)
    errs = {k_: rel_error(pairs[k_], leaves[k_].grad) for k_ in names}
    if seeded:
        errs.update(seed_ssm=rel_error(gk.dseed_ssm, sl["ssm"].grad), seed_k=rel_error(gk.dseed_k, sl["k"].grad),
                    seed_v=rel_error(gk.dseed_v, sl["v"].grad), seed_coef=rel_error(gk.dseed_coef, sl["coef"].grad))
    bad = {k_: e for k_, e in errs.items() if not e < F32_GRAD_TOL}
    assert not bad, f"grad errors above {F32_GRAD_TOL}: {bad} (all: {errs})"


RAW_NAMES = ["q", "k", "v", "dt_raw", "a_raw", "trap_raw", "angles", "dt_bias", "q_bias", "k_bias", "d_skip", "z"]


def _raw_case(shape, seeded, seed=23):
    b, h, l, n, p, nr, chunk = shape
    x, _ = pre_inputs(b, h, l, n, p, nr, seed=seed)
    g = torch.Generator().manual_seed(seed + 1)
    x["dt_bias"] = torch.randn(h, generator=g, dtype=torch.float64) * 0.3
    st = rand_state(b, h, p, n, nr) if seeded else None
    dfs = torch.randn(b, h, p, n, generator=g, dtype=torch.float64) * 0.1
    dfk = torch.randn(b, h, n, generator=g, dtype=torch.float64) * 0.1
    dfv = torch.randn(b, h, p, generator=g, dtype=torch.float64) * 0.1
    dfp = torch.randn(b, h, nr, generator=g, dtype=torch.float64) * 0.1
    return x, st, (dfs, dfk, dfv, dfp)


def _raw_oracle_grads(x, st, cots, chunk, policy="f32", cast=None):
    cast = cast or (lambda t: t)
    leaves = {k_: _leaf(cast(x[k_]) if k_ in ("q", "k", "v", "z") else x[k_]) for k_ in RAW_NAMES}
    sl = None
    state = None
    if st is not None:
        sl = {k_: _leaf(getattr(st, k_)) for k_ in ("ssm", "k", "v", "phi")}
        state = O.SISOState(sl["ssm"], sl["k"], sl["v"], sl["phi"])
    y, fin = O.siso_segment(*(leaves[k_] for k_ in RAW_NAMES[:10]), leaves["d_skip"], leaves["z"], state=state,
                            chunk=chunk, policy=policy)
    dfs, dfk, dfv, dfp = cots
    loss = (y * x["dy"]).sum() + (fin.ssm * dfs).sum() + (fin.k * dfk).sum() + (fin.v * dfv).sum() + \
        (fin.phi * dfp).sum()
    loss.backward()
    return leaves, sl


def _raw_kernel_grads(x, st, cots, chunk, policy, dtype=torch.float32):
    from mamba3_b200 import kernel_bwd as KB

    dfs, dfk, dfv, dfp = cots
    io = lambda t: dev(t, dtype)
    return KB.siso_backward_raw(
        io(x["dy"]), io(x["q"]), io(x["k"]), io(x["v"]), dev(x["dt_raw"]), dev(x["a_raw"]), dev(x["trap_raw"]),
        dev(x["angles"]), dev(x["dt_bias"]), dev(x["q_bias"]), dev(x["k_bias"]), d_skip=dev(x["d_skip"]),
        z=io(x["z"]), seed_ssm=None if st is None else dev(st.ssm), seed_k=None if st is None else dev(st.k),
        seed_v=None if st is None else dev(st.v), seed_phi=None if st is None else dev(st.phi),
        dfinal_ssm=dev(dfs), dfinal_k=dev(dfk), dfinal_v=dev(dfv), dfinal_phi=dev(dfp), chunk=chunk,
        dtype_policy=policy)


def _raw_errors(gk, leaves, sl):
    pairs = dict(q=gk.dq, k=gk.dk, v=gk.dv, dt_raw=gk.ddt_raw, a_raw=gk.da_raw, trap_raw=gk.dtrap_raw,
                 angles=gk.dangles, dt_bias=gk.ddt_bias, q_bias=gk.dq_bias, k_bias=gk.dk_bias, d_skip=gk.dd_skip,
                 z=gk.dz)
    errs = {k_: rel_error(pairs[k_], leaves[k_].grad) for k_ in RAW_NAMES}
    if sl is not None:
        errs.update(seed_ssm=rel_error(gk.dseed_ssm, sl["ssm"].grad), seed_k=rel_error(gk.dseed_k, sl["k"].grad),
                    seed_v=rel_error(gk.dseed_v, sl["v"].grad), seed_phi=rel_error(gk.dseed_phi, sl["phi"].grad))
    return errs


@pytest.mark.parametrize("shape", [(2, 3, 256, 128, 64, 32, 128), (2, 16, 128, 32, 32, 8, 64)])
@pytest.mark.parametrize("seeded", [False, True])
def test_raw_boundary_grads_f32(shape, seeded):
    x, st, cots = _raw_case(shape, seeded)
    leaves, sl = _raw_oracle_grads(x, st, cots, shape[-1])
    gk = _raw_kernel_grads(x, st, cots, shape[-1], "f32")
    errs = _raw_errors(gk, leaves, sl)
    bad = {k_: e for k_, e in errs.items() if not e < F32_GRAD_TOL}
    assert not bad, f"grad errors above {F32_GRAD_TOL}: {bad} (all: {errs})"


def _normwise(a, b):
    a, b = a.detach().double().cpu(), b.detach().double().cpu()
    return float((a - b).norm() / b.norm())


def test_raw_boundary_grads_bf16():
    """bf16 I/O and bf16 matmul operands vs exact (float64) gradients of the SAME
    bf16-valued inputs, normwise.  An elementwise p95 bound of 2e-2 is not attainable for
    bf16 gradients by any implementation: exact arithmetic on bf16-quantised inputs alone
    moves them 2-5% (p95) from the fp32-input gradients, and the reference kernel's own
    bf16 operand rounding adds 2-7% more (measured with the oracle)."""
    shape = (2, 3, 256, 128, 64, 32, 128)
    x, st, cots = _raw_case(shape, True)
    r = lambda t: t.to(torch.bfloat16).double()
    xr = dict(x)
    xr["dy"] = r(x["dy"])
    leaves, sl = _raw_oracle_grads(xr, st, cots, shape[-1], policy="f32", cast=r)
    gk = _raw_kernel_grads(xr, st, cots, shape[-1], "bf16", dtype=torch.bfloat16)
    pairs = dict(q=gk.dq, k=gk.dk, v=gk.dv, dt_raw=gk.ddt_raw, a_raw=gk.da_raw, trap_raw=gk.dtrap_raw,
                 angles=gk.dangles, dt_bias=gk.ddt_bias, q_bias=gk.dq_bias, k_bias=gk.dk_bias, d_skip=gk.dd_skip,
                 z=gk.dz)
    errs = {k_: _normwise(pairs[k_], leaves[k_].grad) for k_ in RAW_NAMES}
    errs.update(seed_ssm=_normwise(gk.dseed_ssm, sl["ssm"].grad), seed_k=_normwise(gk.dseed_k, sl["k"].grad),
                seed_v=_normwise(gk.dseed_v, sl["v"].grad), seed_phi=_normwise(gk.dseed_phi, sl["phi"].grad))
    bad = {k_: e for k_, e in errs.items() if not e < BF16_GRAD_TOL}
    assert not bad, f"normwise grad errors above {BF16_GRAD_TOL}: {bad} (all: {errs})"
