"""The oracle itself: pinned to the reference's own torch code (golden fixtures made by
``tests/golden/make_golden.py``) and to the reference test suite's self-consistency
stages (``mamba3_pallas/tests.py``: refs 405-443, rotation 451-513, segments 653-726,
decode chain 827-875).  CPU only."""

import math
import os

import numpy as np
import pytest
import torch

from oracle import siso_oracle as O
from tests.inputs import make_inputs
from tests.metrics import max_rel, rel_error

GOLD = os.path.join(os.path.dirname(__file__), "golden")
F64 = torch.float64


def _load(name):
    d = np.load(os.path.join(GOLD, name + ".npz"))
    return {k: torch.from_numpy(d[k]) for k in d.files}


@pytest.mark.parametrize("case", ["recurrent_n16_p16_nr4", "recurrent_n32_p16_nr16"])
def test_oracle_matches_reference_torch_recurrence(case):
    g = _load(case)
    lam = torch.sigmoid(g["trap"])
    b, h, l = g["dt"].shape
    nr = g["angles"].shape[-1]
    ang_h = g["angles"][:, None].expand(b, h, l, nr)
    phi, _ = O.cumulative_angles(ang_h, g["dt"])
    args = (g["q"], g["k"], g["v"], g["adt"], g["dt"], lam, phi, g["q_bias"], g["k_bias"])
    y, st = O.siso_recurrent(*args, g["d_skip"], g["z"])
    assert max_rel(y, g["y"]) < 1e-10
    assert max_rel(st.ssm, g["ssm"]) < 1e-10
    assert max_rel(st.k, g["k_final"]) < 1e-10
    assert max_rel(st.v, g["v_final"]) < 1e-12
    assert rel_error(st.phi, g["phi_final"], angle=True) < 1e-10
    y0, _ = O.siso_recurrent(*args)
    assert max_rel(y0, g["y_nogate_noskip"]) < 1e-10
    gamma, scale = O.trapezoid_coeffs(g["dt"], lam)
    for chunk in (8, 16, 32):
        yc, stc = O.siso_chunked(g["q"], g["k"], g["v"], g["adt"], gamma, scale, phi,
                                 g["q_bias"], g["k_bias"], g["d_skip"], g["z"], chunk=chunk)
        assert max_rel(yc, g["y"]) < 1e-9
        assert max_rel(stc.ssm, g["ssm"]) < 1e-9


def test_oracle_layer_matches_reference_torch_layer():
    g = _load("layer_d32_n16_p16")
    d_model, n, p = int(g["d_model"]), int(g["d_state"]), int(g["headdim"])
    sd = {k[4:].replace("__", "."): v for k, v in g.items() if k.startswith("sd__")}
    perm = O.deinterleave_perm(n)
    nheads = 2 * d_model // p
    nr = int(n * float(g["rope_fraction"])) // 2
    d_inner = nheads * p
    in_proj = sd["in_proj.weight"].T.clone()
    for start in (2 * d_inner, 2 * d_inner + n):
        in_proj[:, start:start + n] = in_proj[:, start:start + n][:, perm]
    params = {
        "in_proj": in_proj, "out_proj": sd["out_proj.weight"].T.clone(),
        "dt_bias": sd["dt_bias"], "b_norm_weight": sd["B_norm_weight"][perm],
        "c_norm_weight": sd["C_norm_weight"][perm], "b_bias": sd["B_bias"][:, 0][:, perm],
        "c_bias": sd["C_bias"][:, 0][:, perm], "d_skip": sd["D"],
    }
    y, _ = O.layer_forward(params, g["u"], d_state=n, headdim=p, nheads=nheads,
                           n_angles=nr, chunk=16)
    # torch_ref casts dd_A and the angles to float32 (torch_ref.py:216, 228), so the
    # float64 fixture carries float32 rounding there.
    assert max_rel(y, g["y"]) < 1e-6


def test_perm_roundtrip():
    for n in (16, 32, 128):
        x = torch.randn(3, n, dtype=F64)
        assert torch.equal(x[..., O.deinterleave_perm(n)][..., O.interleave_perm(n)], x)


@pytest.mark.parametrize("dtype,tol", [(torch.float64, 1e-10), (torch.float32, 1e-5)])
def test_refs_recurrent_vs_chunked(dtype, tol):
    x = make_inputs(2, 3, 256, seed=0, dtype=dtype)
    pre, _ = O.preprocess(x["dt_raw"], x["a_raw"], x["trap_raw"], x["angles"], x["dt_bias"])
    y_rec, st_rec = O.siso_recurrent(x["q"], x["k"], x["v"], pre.adt, pre.dt, pre.lam, pre.phi,
                                     x["q_bias"], x["k_bias"], x["d_skip"], x["z"])
    y_chk, st_chk = O.siso_chunked(x["q"], x["k"], x["v"], pre.adt, pre.gamma, pre.scale,
                                   pre.phi, x["q_bias"], x["k_bias"], x["d_skip"], x["z"],
                                   chunk=128)
    assert rel_error(y_chk, y_rec) < tol
    assert rel_error(st_chk.ssm, st_rec.ssm) < tol
    assert rel_error(st_chk.k, st_rec.k) < tol
    assert max_rel(st_chk.v, st_rec.v) < 1e-6


def _rotation_case(chunk=128):
    """Inputs of the analytic parity task (``tests.py:451-513``)."""
    batch, nheads, seqlen, n, p, nr = 2, 1, 2 * chunk, 128, 64, 32
    g = torch.Generator().manual_seed(0)
    bits = (torch.rand(batch, seqlen, generator=g) < 0.5).to(F64)
    bits[:, 0] = 0.0
    parity = torch.cumsum(bits, 1) % 2
    atanh_one = math.atanh(1 - 1e-6)
    angles = torch.where(bits[:, :, None] > 0.5, atanh_one, 0.0) * torch.ones(1, 1, nr, dtype=F64)
    dt = torch.ones(batch, nheads, seqlen, dtype=F64)
    lam = torch.ones(batch, nheads, seqlen, dtype=F64)
    adt = torch.full((batch, nheads, seqlen), -1e-6, dtype=F64)
    e0 = torch.zeros(n, dtype=F64)
    e0[0] = 1.0
    q = e0.expand(batch, seqlen, n).clone()
    k = torch.zeros(batch, seqlen, n, dtype=F64)
    k[:, 0] = e0
    v = torch.ones(batch, nheads, seqlen, p, dtype=F64)
    want = torch.where(parity[:, None, :, None] > 0.5, -1.0, 1.0).to(F64)
    return dict(q=q, k=k, v=v, adt=adt, dt=dt, lam=lam, angles=angles, want=want,
                qb=torch.zeros(nheads, n, dtype=F64), kb=torch.zeros(nheads, n, dtype=F64))


def test_rotation_parity_kat():
    c = _rotation_case()
    gamma, scale = O.trapezoid_coeffs(c["dt"], c["lam"])
    phi, _ = O.cumulative_angles(c["angles"][:, None], c["dt"])
    y_rec, _ = O.siso_recurrent(c["q"], c["k"], c["v"], c["adt"], c["dt"], c["lam"], phi,
                                c["qb"], c["kb"])
    y_chk, _ = O.siso_chunked(c["q"], c["k"], c["v"], c["adt"], gamma, scale, phi,
                              c["qb"], c["kb"], chunk=128)
    for y in (y_rec, y_chk):
        assert float((torch.sign(y) == torch.sign(c["want"])).to(F64).mean()) == 1.0
        assert float((y - c["want"]).abs().max()) <= 1e-3


def test_segments_equal_one_call():
    x = make_inputs(2, 3, 256, seed=0)
    half = 128

    def run(sl, state=None):
        return O.siso_segment(x["q"][:, sl], x["k"][:, sl], x["v"][:, :, sl], x["dt_raw"][:, sl],
                              x["a_raw"][:, sl], x["trap_raw"][:, sl], x["angles"][:, sl],
                              x["dt_bias"], x["q_bias"], x["k_bias"], x["d_skip"],
                              x["z"][:, :, sl], state=state, chunk=128)

    y_full, st_full = run(slice(None))
    y1, s1 = run(slice(0, half))
    y2, s2 = run(slice(half, 256), state=s1)
    assert rel_error(torch.cat([y1, y2], 2), y_full) < 1e-10
    assert rel_error(s2.ssm, st_full.ssm) < 1e-10
    assert rel_error(s2.k, st_full.k) < 1e-10
    assert rel_error(s2.phi, st_full.phi, angle=True) < 1e-10


def test_decode_chain_equals_prefill():
    x = make_inputs(1, 2, 64, seed=11)
    pre, _ = O.preprocess(x["dt_raw"], x["a_raw"], x["trap_raw"], x["angles"], x["dt_bias"])
    st = O.zero_state(1, 2, 64, 128, 32)
    ys = []
    for t in range(64):
        y, st = O.siso_step(x["q"][:, t], x["k"][:, t], x["v"][:, :, t], pre.adt[:, :, t],
                            pre.dt[:, :, t], pre.lam[:, :, t], x["angles"][:, t],
                            x["q_bias"], x["k_bias"], st, x["d_skip"], x["z"][:, :, t])
        ys.append(y)
    y_pre, fin = O.siso_chunked(x["q"], x["k"], x["v"], pre.adt, pre.gamma, pre.scale, pre.phi,
                                x["q_bias"], x["k_bias"], x["d_skip"], x["z"], chunk=32)
    assert rel_error(torch.stack(ys, 2), y_pre) < 1e-10
    assert rel_error(st.ssm, fin.ssm) < 1e-10
    assert rel_error(st.k, fin.k) < 1e-10


def test_chunked_gradients_vs_finite_differences():
    x = make_inputs(1, 1, 32, state_dim=16, headdim=8, n_angles=4, seed=3)
    keys = ["q", "v", "dt_raw", "angles", "trap_raw", "a_raw"]

    def f(*args):
        d = dict(x)
        d.update(zip(keys, args))
        y, st = O.siso_segment(d["q"], d["k"], d["v"], d["dt_raw"], d["a_raw"], d["trap_raw"],
                               d["angles"], d["dt_bias"], d["q_bias"], d["k_bias"],
                               d["d_skip"], d["z"], chunk=8)
        return (y * d["dy"]).sum() + st.ssm.pow(2).sum()

    inputs = tuple(x[k].clone().requires_grad_(True) for k in keys)
    assert torch.autograd.gradcheck(f, inputs, eps=1e-6, atol=1e-6, rtol=1e-5)


def test_layout_helpers_match_oracle():
    """The torch rope / prefix-sum helpers of `mamba3_b200.layout` (``layout.py:345-497``)
    against the oracle's rotation and plain sums; the policy object (``layout.py:243-291``)."""
    from mamba3_b200 import layout as LA

    g = torch.Generator().manual_seed(3)
    n, nr = 32, 10
    phi = torch.rand(2, 5, nr, generator=g, dtype=F64) * 6
    x = torch.randn(2, 5, n, generator=g, dtype=F64)
    cos_f, sin_f = LA.rope_cos_sin(phi, n)
    ocos, osin = O.rope_cos_sin(phi, n)
    assert torch.allclose(cos_f, ocos) and torch.allclose(sin_f, osin)
    xr = LA.rope_apply(x, cos_f, sin_f)
    assert torch.allclose(xr, O.rope_apply(x, ocos, osin))
    # dphi: derivative of <dx, R(phi) x> in phi, against a finite difference
    dx = torch.randn(2, 5, n, generator=g, dtype=F64)
    dphi = LA.rope_dphi(xr, dx, nr)
    eps = 1e-6
    for j in (0, 3, nr - 1):
        pp = phi.clone()
        pp[..., j] += eps
        c2, s2 = LA.rope_cos_sin(pp, n)
        fd = ((LA.rope_apply(x, c2, s2) - xr) * dx).sum(-1) / eps
        assert torch.allclose(dphi[..., j], fd, atol=1e-4)
    row = torch.randn(1, 16, generator=g, dtype=F64)
    tril = LA.tril_ones(16)
    assert torch.allclose(LA.prefix_sum(row, tril).double(), (row @ tril.double().T)[0], atol=1e-5)
    assert torch.allclose(LA.suffix_sum(row, tril).double(), (row @ tril.double())[0], atol=1e-5)
    assert LA.policy("default") is LA.BF16 and LA.policy("highest").highest and LA.policy(LA.F32) is LA.F32
    assert LA.policy("bf16") == "bf16" and LA.BF16.saved_state == torch.bfloat16
    with pytest.raises(ValueError):
        LA.policy("fp8")
