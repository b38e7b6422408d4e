"""The tcgen05 tensor-core backward (raw boundary, bf16 I/O and operands, N=128, P=64)
against exact float64 gradients of the same bf16-valued inputs (normwise, as for the
generic kernel's bf16 test) and against the generic kernel."""

import pytest
import torch

from tests.test_bwd_gpu import BF16_GRAD_TOL, RAW_NAMES, _normwise, _raw_case, _raw_kernel_grads, _raw_oracle_grads

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _no_device_error():
    from mamba3_b200 import _capi as C

    C.lib().m3_device_error(1)
    yield
    assert C.lib().m3_device_error(1) == 0


def _kernel(x, st, cots, chunk, kernel):
    from mamba3_b200 import kernel_bwd as KB
    from tests.gpu_common import dev

    dfs, dfk, dfv, dfp = cots
    io = lambda t: dev(t, torch.bfloat16)
    return KB.siso_backward_raw(
        io(x["dy"]), io(x["q"]), io(x["k"]), io(x["v"]), dev(x["dt_raw"]), dev(x["a_raw"]), dev(x["trap_raw"]),
        dev(x["angles"]), dev(x["dt_bias"]), dev(x["q_bias"]), dev(x["k_bias"]), d_skip=dev(x["d_skip"]),
        z=io(x["z"]), seed_ssm=None if st is None else dev(st.ssm), seed_k=None if st is None else dev(st.k),
        seed_v=None if st is None else dev(st.v), seed_phi=None if st is None else dev(st.phi),
        dfinal_ssm=dev(dfs), dfinal_k=dev(dfk), dfinal_v=dev(dfv), dfinal_phi=dev(dfp), chunk=chunk,
        dtype_policy="bf16", kernel=kernel)


def _pairs(g):
    return dict(q=g.dq, k=g.dk, v=g.dv, dt_raw=g.ddt_raw, a_raw=g.da_raw, trap_raw=g.dtrap_raw, angles=g.dangles,
                dt_bias=g.ddt_bias, q_bias=g.dq_bias, k_bias=g.dk_bias, d_skip=g.dd_skip, z=g.dz)


@pytest.mark.parametrize("shape", [(2, 3, 256, 128, 64, 32, 128), (1, 2, 384, 128, 64, 64, 128)])
@pytest.mark.parametrize("seeded", [False, True])
def test_tc_backward_vs_exact_and_generic(shape, seeded):
    x, st, cots = _raw_case(shape, seeded)
    r = lambda t: t.to(torch.bfloat16).double()
    xr = dict(x)
    xr["dy"] = r(x["dy"])
    leaves, sl = _raw_oracle_grads(xr, st, cots, shape[-1], policy="f32", cast=r)
    g_tc = _kernel(xr, st, cots, shape[-1], "tensorcore")
    g_gen = _kernel(xr, st, cots, shape[-1], "generic")
    pt, pg = _pairs(g_tc), _pairs(g_gen)
    errs = {k: _normwise(pt[k], leaves[k].grad) for k in RAW_NAMES}
    vs_gen = {k: _normwise(pt[k], pg[k]) for k in RAW_NAMES}
    if seeded:
        errs.update(seed_ssm=_normwise(g_tc.dseed_ssm, sl["ssm"].grad), seed_k=_normwise(g_tc.dseed_k, sl["k"].grad),
                    seed_v=_normwise(g_tc.dseed_v, sl["v"].grad), seed_phi=_normwise(g_tc.dseed_phi, sl["phi"].grad))
    bad = {k: e for k, e in errs.items() if not e < BF16_GRAD_TOL}
    assert not bad, f"normwise errors vs exact above {BF16_GRAD_TOL}: {bad} (all {errs}; vs generic {vs_gen})"
    bad = {k: e for k, e in vs_gen.items() if not e < BF16_GRAD_TOL}
    assert not bad, f"normwise differences vs the generic kernel: {bad}"


def test_tc_backward_without_gate_or_skip():
    """No z (no gate, so no dz) and no D: the tensor-core backward against the generic one."""
    from mamba3_b200 import kernel_bwd as KB
    from tests.gpu_common import dev
    from tests.test_bwd_gpu import _normwise

    x, _, _ = _raw_case((1, 2, 256, 128, 64, 32, 128), False, seed=41)
    io = lambda t: dev(t, torch.bfloat16)
    args = (io(x["dy"]), io(x["q"]), io(x["k"]), io(x["v"]), dev(x["dt_raw"]), dev(x["a_raw"]), dev(x["trap_raw"]),
            dev(x["angles"]), dev(x["dt_bias"]), dev(x["q_bias"]), dev(x["k_bias"]))
    gt = KB.siso_backward_raw(*args, d_skip=None, z=None, chunk=128, dtype_policy="bf16", kernel="tensorcore")
    gg = KB.siso_backward_raw(*args, d_skip=None, z=None, chunk=128, dtype_policy="bf16", kernel="generic")
    assert gt.dz is None and gg.dz is None
    for name in ("dq", "dk", "dv", "ddt_raw", "da_raw", "dtrap_raw", "dangles", "dq_bias", "dk_bias", "ddt_bias"):
        e = _normwise(getattr(gt, name), getattr(gg, name))
        assert e < 2e-2, f"{name}: {e}"


@pytest.mark.parametrize("nr", [8])
def test_tc_forward_backward_few_rotary_pairs(nr):
    """n_angles = 8 (one rotary group; the other seven pass through): tensor-core forward and
    backward against the generic kernels.  (n_angles = 0 is refused at the boundary, as the
    reference's layer refuses a rotary fraction that leaves no angles.)"""
    from mamba3_b200 import kernel_bwd as KB
    from mamba3_b200 import kernel_fwd as KF
    from tests.gpu_common import dev
    from tests.metrics import rel_error
    from tests.test_bwd_gpu import _normwise

    x, _, _ = _raw_case((1, 2, 256, 128, 64, nr, 128), False, seed=43)
    io = lambda t: dev(t, torch.bfloat16)
    raw = (dev(x["dt_raw"]), dev(x["a_raw"]), dev(x["trap_raw"]), dev(x["angles"]), dev(x["dt_bias"]),
           dev(x["q_bias"]), dev(x["k_bias"]))
    yt = KF.siso_forward_raw(io(x["q"]), io(x["k"]), io(x["v"]), *raw, dev(x["d_skip"]), io(x["z"]), chunk=128,
                             dtype_policy="bf16", kernel="tensorcore")[0]
    yg = KF.siso_forward_raw(io(x["q"]), io(x["k"]), io(x["v"]), *raw, dev(x["d_skip"]), io(x["z"]), chunk=128,
                             dtype_policy="bf16", kernel="generic")[0]
    assert rel_error(yt, yg) < 2e-2
    args = (io(x["dy"]), io(x["q"]), io(x["k"]), io(x["v"]), *raw)
    gt = KB.siso_backward_raw(*args, d_skip=dev(x["d_skip"]), z=io(x["z"]), chunk=128, dtype_policy="bf16",
                              kernel="tensorcore")
    gg = KB.siso_backward_raw(*args, d_skip=dev(x["d_skip"]), z=io(x["z"]), chunk=128, dtype_policy="bf16",
                              kernel="generic")
    for name in ("dq", "dk", "dv", "dz", "ddt_raw", "da_raw", "dtrap_raw", "dq_bias", "dk_bias", "dangles"):
        e = _normwise(getattr(gt, name), getattr(gg, name))
        assert e < 2e-2, f"{name}: {e}"


@pytest.mark.parametrize("seeded", [False, True])
def test_tc_backward_preprocessed_boundary(seeded):
    """The reference kernel's own boundary (adt, gamma, scale, phi in; their gradients and
    dseed_coef out: ``kernel_bwd.py:534-669``) on the tensor-core backward, against exact
    float64 gradients of the bf16-valued inputs and against the generic kernel."""
    from mamba3_b200 import kernel_bwd as KB
    from oracle import siso_oracle as O
    from tests.gpu_common import dev, pre_inputs, rand_state
    from tests.test_bwd_gpu import _normwise

    b, h, l, n, p, nr, chunk = 2, 3, 256, 128, 64, 32, 128
    x, pre = pre_inputs(b, h, l, n, p, nr, seed=47)
    g = torch.Generator().manual_seed(9)
    st = rand_state(b, h, p, n, nr) if seeded else None
    coef = torch.rand(b, h, generator=g, dtype=torch.float64) * 0.05 if seeded else None
    dfs = torch.randn(b, h, p, n, generator=g, dtype=torch.float64) * 0.1
    dfk = torch.randn(b, h, n, generator=g, dtype=torch.float64) * 0.1
    dfv = torch.randn(b, h, p, generator=g, dtype=torch.float64) * 0.1
    r = lambda t: t.to(torch.bfloat16).double()
    names = ["q", "k", "v", "adt", "gamma", "scale", "phi", "q_bias", "k_bias", "d_skip", "z"]
    vals = dict(q=r(x["q"]), k=r(x["k"]), v=r(x["v"]), adt=pre.adt, gamma=pre.gamma, scale=pre.scale, phi=pre.phi,
                q_bias=x["q_bias"], k_bias=x["k_bias"], d_skip=x["d_skip"], z=r(x["z"]))
    dy = r(x["dy"])
    leaves = {k_: v_.clone().requires_grad_(True) for k_, v_ in vals.items()}
    if seeded:
        cl = coef.clone().requires_grad_(True)
        y, fin = O.siso_chunked(*(leaves[k_] for k_ in names), state=O.SISOState(st.ssm, st.k, st.v, st.phi),
                                seed_dt=cl, seed_lam=torch.zeros_like(coef), chunk=chunk)
    else:
        y, fin = O.siso_chunked(*(leaves[k_] for k_ in names), chunk=chunk)
    ((y * dy).sum() + (fin.ssm * dfs).sum() + (fin.k * dfk).sum() + (fin.v * dfv).sum()).backward()

    io = lambda t: dev(t, torch.bfloat16)

    def run(kernel):
        return KB.siso_backward(io(dy), io(vals["q"]), io(vals["k"]), io(vals["v"]), dev(pre.adt), dev(pre.gamma),
                                dev(pre.scale), dev(pre.phi), dev(x["q_bias"]), dev(x["k_bias"]),
                                d_skip=dev(x["d_skip"]), z=io(vals["z"]),
                                seed_ssm=dev(st.ssm) if seeded else None, seed_k=dev(st.k) if seeded else None,
                                seed_v=dev(st.v) if seeded else None, seed_coef=dev(coef) if seeded else None,
                                dfinal_ssm=dev(dfs), dfinal_k=dev(dfk), dfinal_v=dev(dfv), chunk=chunk,
                                dtype_policy="bf16", kernel=kernel)

    gt, gg = run("tensorcore"), run("generic")
    pick = lambda gk: dict(q=gk.dq, k=gk.dk, v=gk.dv, adt=gk.dadt, gamma=gk.dgamma, scale=gk.dscale, phi=gk.dphi,
                           q_bias=gk.dq_bias, k_bias=gk.dk_bias, d_skip=gk.dd_skip, z=gk.dz)
    pt, pg = pick(gt), pick(gg)
    errs = {k_: _normwise(pt[k_], leaves[k_].grad) for k_ in names}
    vs_gen = {k_: _normwise(pt[k_], pg[k_]) for k_ in names}
    if seeded:
        errs["seed_coef"] = _normwise(gt.dseed_coef, cl.grad)
        vs_gen["seed_coef"] = _normwise(gt.dseed_coef, gg.dseed_coef)
        vs_gen["seed_ssm"] = _normwise(gt.dseed_ssm, gg.dseed_ssm)
        vs_gen["seed_k"] = _normwise(gt.dseed_k, gg.dseed_k)
        vs_gen["seed_v"] = _normwise(gt.dseed_v, gg.dseed_v)
    bad = {k_: e for k_, e in errs.items() if not e < BF16_GRAD_TOL}
    assert not bad, f"normwise errors vs exact above {BF16_GRAD_TOL}: {bad} (all {errs}; vs generic {vs_gen})"
    bad = {k_: e for k_, e in vs_gen.items() if not e < BF16_GRAD_TOL}
    assert not bad, f"normwise differences vs the generic kernel: {bad}"


def test_forward_saved_states_equal_the_recompute_sweep():
    """The tensor-core forward given the backward's workspace writes the chunk-start states
    the backward's sweep would recompute: gradients with the sweep skipped match those with
    it; and autograd through `siso_segment` (which uses this) agrees."""
    from mamba3_b200 import kernel_bwd as KB
    from mamba3_b200 import kernel_fwd as KF
    from mamba3_b200 import siso as SISO
    from mamba3_b200.state import SISOState
    from tests.gpu_common import dev

    x, st, _ = _raw_case((2, 3, 384, 128, 64, 32, 128), True, seed=45)
    io = lambda t: dev(t, torch.bfloat16)
    q, k, v, z, dy = io(x["q"]), io(x["k"]), io(x["v"]), io(x["z"]), io(x["dy"])
    raw = (dev(x["dt_raw"]), dev(x["a_raw"]), dev(x["trap_raw"]), dev(x["angles"]), dev(x["dt_bias"]),
           dev(x["q_bias"]), dev(x["k_bias"]))
    seeds = dict(seed_ssm=dev(st.ssm), seed_k=dev(st.k), seed_v=dev(st.v), seed_phi=dev(st.phi))
    ws = torch.zeros(KB.workspace_bytes(2, 384, 3, 128, 64, 32, 128), dtype=torch.uint8, device="cuda")
    _, saved = KF.siso_forward_raw(q, k, v, *raw, d_skip=dev(x["d_skip"]), z=z, **seeds, chunk=128,
                                   dtype_policy="bf16", bwd_states=ws, return_saved=True)
    assert saved
    common = dict(d_skip=dev(x["d_skip"]), z=z, **seeds, chunk=128, dtype_policy="bf16", kernel="tensorcore")
    g1 = KB.siso_backward_raw(dy, q, k, v, *raw, workspace=ws, states_ready=True, **common)
    g2 = KB.siso_backward_raw(dy, q, k, v, *raw, **common)
    for name in ("dq", "dk", "dv", "dz", "ddt_raw", "da_raw", "dtrap_raw", "dangles", "dseed_ssm", "dseed_phi"):
        a, b = getattr(g1, name).double(), getattr(g2, name).double()
        # the saving forward (warp-specialised kernel) and the states-only sweep round a few
        # bf16 state elements differently; the gradients agree far inside the bf16 bound
        assert float((a - b).norm() / b.norm()) < 1e-2, name
    leaves = [t.clone().requires_grad_(True) for t in (q, k, v)]
    out = SISO.siso_segment(*leaves, *raw, d_skip=dev(x["d_skip"]), z=z, state=SISOState(**{
        "ssm": seeds["seed_ssm"], "k": seeds["seed_k"], "v": seeds["seed_v"], "phi": seeds["seed_phi"]}),
        chunk=128, policy_name="bf16")
    out.y.backward(dy)
    for leaf, ref in zip(leaves, (g2.dq, g2.dk, g2.dv)):
        a, b = leaf.grad.double(), ref.double()
        assert float((a - b).norm() / b.norm()) < 1e-2


@pytest.mark.parametrize("kernel", ["tensorcore", "generic"])
def test_bf16_gradient_outputs(kernel):
    """grad_dtype=bf16: dv / dz written as bf16 equal the fp32 outputs rounded to bf16."""
    from mamba3_b200 import kernel_bwd as KB
    from tests.gpu_common import dev

    x, _, _ = _raw_case((1, 2, 256, 128, 64, 32, 128), False, seed=53)
    io = lambda t: dev(t, torch.bfloat16)
    args = (io(x["dy"]), io(x["q"]), io(x["k"]), io(x["v"]), dev(x["dt_raw"]), dev(x["a_raw"]), dev(x["trap_raw"]),
            dev(x["angles"]), dev(x["dt_bias"]), dev(x["q_bias"]), dev(x["k_bias"]))
    kw = dict(d_skip=dev(x["d_skip"]), z=io(x["z"]), chunk=128, dtype_policy="bf16", kernel=kernel)
    g32 = KB.siso_backward_raw(*args, **kw)
    g16 = KB.siso_backward_raw(*args, **kw, grad_dtype=torch.bfloat16)
    assert g16.dv.dtype == torch.bfloat16 and g16.dz.dtype == torch.bfloat16
    for a, b in ((g16.dv, g32.dv), (g16.dz, g32.dz)):
        # the same fp32 values rounded once (red.add order aside, dv / dz involve no atomics)
        assert (a.float() - b.to(torch.bfloat16).float()).abs().max() <= 1e-2 * b.abs().max()


@pytest.mark.parametrize("kernel", ["tensorcore", "generic"])
def test_strided_gradient_outputs(kernel):
    """dv / dz written through (B, L, H, P) buffers seen as (B, H, L, P) (the layout of the
    layer's in_proj slices) equal the dense outputs."""
    from mamba3_b200 import kernel_bwd as KB
    from tests.gpu_common import dev

    x, _, _ = _raw_case((2, 3, 256, 128, 64, 32, 128), False, seed=57)
    io = lambda t: dev(t, torch.bfloat16)
    args = (io(x["dy"]), io(x["q"]), io(x["k"]), io(x["v"]), dev(x["dt_raw"]), dev(x["a_raw"]), dev(x["trap_raw"]),
            dev(x["angles"]), dev(x["dt_bias"]), dev(x["q_bias"]), dev(x["k_bias"]))
    kw = dict(d_skip=dev(x["d_skip"]), z=io(x["z"]), chunk=128, dtype_policy="bf16", kernel=kernel,
              grad_dtype=torch.bfloat16)
    dense = KB.siso_backward_raw(*args, **kw)
    bufv = torch.full((2, 256, 3, 64), float("nan"), dtype=torch.bfloat16, device="cuda")
    bufz = torch.full_like(bufv, float("nan"))
    strided = KB.siso_backward_raw(*args, **kw, dv_out=bufv.permute(0, 2, 1, 3), dz_out=bufz.permute(0, 2, 1, 3))
    assert not torch.isnan(bufv).any() and not torch.isnan(bufz).any()
    # dv / dz involve no atomics: the same values whatever the layout
    assert torch.equal(strided.dv, dense.dv) and torch.equal(strided.dz, dense.dz)
