"""Forward kernel parity against the oracle (``mamba3_pallas/tests.py`` stages forward
521-565, rotation 451-513, segments 653-726), through the C ABI."""

import math
import os

import numpy as np
import pytest
import torch

from oracle import siso_oracle as O
from tests.gpu_common import DEV, cpu64, dev, pre_inputs, rand_state
from tests.metrics import max_rel, rel_error

pytestmark = pytest.mark.gpu

F32_TOL = 1e-5     # fp32 policy vs the float64 oracle (BASELINE north-star tolerance)
BF16_TOL = 2e-2    # bf16 policy vs the bf16-rounding oracle
BF16_EXACT_TOL = 5e-2  # bf16 policy vs exact float64 (mamba3_pallas/tests.py:534)


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")


SHAPES = [  # (B, H, L, N, P, Nr, chunk)
    (2, 3, 256, 128, 64, 32, 128),
    (2, 16, 128, 32, 32, 8, 64),
    (1, 2, 192, 64, 64, 32, 64),
    (2, 2, 128, 16, 16, 4, 64),
    (1, 3, 128, 32, 16, 16, 128),
]


@pytest.mark.parametrize("shape", SHAPES)
def test_forward_f32_matches_oracle(shape):
    from mamba3_b200 import kernel_fwd as KF

    b, h, l, n, p, nr, chunk = shape
    x, pre = pre_inputs(b, h, l, n, p, nr, seed=0)
    y_ref, st_ref, dbg = O.siso_chunked(x["q"], x["k"], x["v"], pre.adt, pre.gamma, pre.scale, pre.phi,
                                        x["q_bias"], x["k_bias"], x["d_skip"], x["z"], chunk=chunk,
                                        return_debug=True)
    y, fs, fk, fv, res = KF.siso_forward(
        dev(x["q"]), dev(x["k"]), dev(x["v"]), dev(pre.adt), dev(pre.gamma), dev(pre.scale), dev(pre.phi),
        dev(x["q_bias"]), dev(x["k_bias"]), dev(x["d_skip"]), dev(x["z"]), chunk=chunk, dtype_policy="f32",
        save_residuals=True)
    assert rel_error(y, y_ref) < F32_TOL
    assert rel_error(fs, st_ref.ssm) < F32_TOL
    assert rel_error(fk, st_ref.k) < F32_TOL
    assert max_rel(fv, st_ref.v) < 1e-7
    assert rel_error(res.ybar, dbg["ybar"]) < F32_TOL
    assert rel_error(res.chunk_states, dbg["chunk_states"]) < F32_TOL


def test_forward_bf16_policy():
    from mamba3_b200 import kernel_fwd as KF

    b, h, l, n, p, nr, chunk = 2, 3, 256, 128, 64, 32, 128
    x, pre = pre_inputs(b, h, l, n, p, nr, seed=0)
    bf = {k_: x[k_].to(torch.bfloat16).double() for k_ in ("q", "k", "v", "z")}
    y_rnd, st_rnd, dbg = O.siso_chunked(bf["q"], bf["k"], bf["v"], pre.adt, pre.gamma, pre.scale, pre.phi,
                                        x["q_bias"], x["k_bias"], x["d_skip"], bf["z"], chunk=chunk,
                                        policy="bf16", return_debug=True)
    y_ex, st_ex = O.siso_chunked(x["q"], x["k"], x["v"], pre.adt, pre.gamma, pre.scale, pre.phi,
                                 x["q_bias"], x["k_bias"], x["d_skip"], x["z"], chunk=chunk)
    b16 = torch.bfloat16
    y, fs, fk, fv, res = KF.siso_forward(
        dev(x["q"], b16), dev(x["k"], b16), dev(x["v"], b16), dev(pre.adt), dev(pre.gamma), dev(pre.scale),
        dev(pre.phi), dev(x["q_bias"]), dev(x["k_bias"]), dev(x["d_skip"]), dev(x["z"], b16), chunk=chunk,
        dtype_policy="bf16", save_residuals=True)
    assert y.dtype == torch.bfloat16 and res.chunk_states.dtype == torch.bfloat16
    assert rel_error(y, y_rnd) < BF16_TOL
    assert rel_error(fs, st_rnd.ssm) < BF16_TOL
    assert rel_error(fk, st_rnd.k) < BF16_TOL
    assert rel_error(res.ybar, dbg["ybar"]) < BF16_TOL
    assert rel_error(y, y_ex) < BF16_EXACT_TOL
    assert rel_error(fs, st_ex.ssm) < BF16_EXACT_TOL


def test_forward_no_gate_no_skip():
    from mamba3_b200 import kernel_fwd as KF

    b, h, l, n, p, nr, chunk = 2, 3, 256, 128, 64, 32, 128
    x, pre = pre_inputs(b, h, l, n, p, nr, seed=5)
    y_ref, _ = O.siso_chunked(x["q"], x["k"], x["v"], pre.adt, pre.gamma, pre.scale, pre.phi,
                              x["q_bias"], x["k_bias"], None, None, chunk=chunk)
    y, *_ = KF.siso_forward(dev(x["q"]), dev(x["k"]), dev(x["v"]), dev(pre.adt), dev(pre.gamma), dev(pre.scale),
                            dev(pre.phi), dev(x["q_bias"]), dev(x["k_bias"]), None, None, chunk=chunk,
                            dtype_policy="f32")
    assert rel_error(y, y_ref) < F32_TOL


def test_forward_seeded_state():
    from mamba3_b200 import kernel_fwd as KF

    b, h, l, n, p, nr, chunk = 2, 3, 128, 128, 64, 32, 64
    x, pre = pre_inputs(b, h, l, n, p, nr, seed=7)
    st = rand_state(b, h, p, n, nr)
    sdt, slam = pre.dt[:, :, 0], pre.lam[:, :, 0]
    y_ref, fin = O.siso_chunked(x["q"], x["k"], x["v"], pre.adt, pre.gamma, pre.scale, pre.phi, x["q_bias"],
                                x["k_bias"], x["d_skip"], x["z"], state=st, seed_dt=sdt, seed_lam=slam, chunk=chunk)
    y, fs, fk, fv = KF.siso_forward(
        dev(x["q"]), dev(x["k"]), dev(x["v"]), dev(pre.adt), dev(pre.gamma), dev(pre.scale), dev(pre.phi),
        dev(x["q_bias"]), dev(x["k_bias"]), dev(x["d_skip"]), dev(x["z"]), seed_ssm=dev(st.ssm), seed_k=dev(st.k),
        seed_v=dev(st.v), seed_coef=dev(sdt * (1 - slam)), chunk=chunk, dtype_policy="f32")
    assert rel_error(y, y_ref) < F32_TOL
    assert rel_error(fs, fin.ssm) < F32_TOL


@pytest.mark.parametrize("with_state", [False, True])
@pytest.mark.parametrize("shape", [(2, 3, 256, 128, 64, 32, 128), (2, 16, 128, 32, 32, 8, 64)])
def test_raw_boundary_segment_matches_oracle(shape, with_state):
    """Fused preprocess (softplus / heavy tail / sigmoid / trapezoid shift / cumulative
    angles) + scan vs the oracle's preprocess + chunked scan (siso.py:154-216)."""
    from mamba3_b200 import kernel_fwd as KF

    b, h, l, n, p, nr, chunk = shape
    x, _ = pre_inputs(b, h, l, n, p, nr, seed=3)
    x["dt_bias"] = torch.randn(h, dtype=torch.float64, generator=torch.Generator().manual_seed(9)) * 0.3
    st = rand_state(b, h, p, n, nr) if with_state else None
    y_ref, fin = O.siso_segment(x["q"], x["k"], x["v"], x["dt_raw"], x["a_raw"], x["trap_raw"], x["angles"],
                                x["dt_bias"], x["q_bias"], x["k_bias"], x["d_skip"], x["z"], state=st, chunk=chunk)
    y, fs, fk, fv, fphi = KF.siso_forward_raw(
        dev(x["q"]), dev(x["k"]), dev(x["v"]), dev(x["dt_raw"]), dev(x["a_raw"]), dev(x["trap_raw"]),
        dev(x["angles"]), dev(x["dt_bias"]), dev(x["q_bias"]), dev(x["k_bias"]), dev(x["d_skip"]), dev(x["z"]),
        seed_ssm=None if st is None else dev(st.ssm), seed_k=None if st is None else dev(st.k),
        seed_v=None if st is None else dev(st.v), seed_phi=None if st is None else dev(st.phi),
        chunk=chunk, dtype_policy="f32")
    assert rel_error(y, y_ref) < F32_TOL
    assert rel_error(fs, fin.ssm) < F32_TOL
    assert rel_error(fk, fin.k) < F32_TOL
    assert max_rel(fv, fin.v) < 1e-7
    assert rel_error(fphi, fin.phi, angle=True) < 1e-5


def test_rotation_parity_kat_on_kernel():
    """tests.py:451-513: sign accuracy exactly 1, |y - (-1)^parity| <= 1e-3."""
    from mamba3_b200 import kernel_fwd as KF
    from tests.test_oracle import _rotation_case

    c = _rotation_case(chunk=128)
    gamma, scale = O.trapezoid_coeffs(c["dt"], c["lam"])
    phi, _ = O.cumulative_angles(c["angles"][:, None], c["dt"])
    y, *_ = KF.siso_forward(dev(c["q"]), dev(c["k"]), dev(c["v"]), dev(c["adt"]), dev(gamma), dev(scale), dev(phi),
                            dev(c["qb"]), dev(c["kb"]), None, None, chunk=128, dtype_policy="f32")
    want = c["want"].to(DEV).float()
    assert float((torch.sign(y) == torch.sign(want)).float().mean()) == 1.0
    assert float((y - want).abs().max()) <= 1e-3


def test_golden_fixtures_through_kernel():
    """The reference's own torch recurrence (torch_ref.mamba3_siso_ref) as fixtures."""
    from mamba3_b200 import kernel_fwd as KF

    gold = os.path.join(os.path.dirname(__file__), "golden")
    for name in ("recurrent_n16_p16_nr4", "recurrent_n32_p16_nr16"):
        g = {k_: torch.from_numpy(v_) for k_, v_ in np.load(os.path.join(gold, name + ".npz")).items()}
        lam = torch.sigmoid(g["trap"])
        b, h, l = g["dt"].shape
        phi, _ = O.cumulative_angles(g["angles"][:, None].expand(b, h, l, g["angles"].shape[-1]), g["dt"])
        gamma, scale = O.trapezoid_coeffs(g["dt"], lam)
        y, fs, fk, fv = KF.siso_forward(dev(g["q"]), dev(g["k"]), dev(g["v"]), dev(g["adt"]), dev(gamma),
                                        dev(scale), dev(phi), dev(g["q_bias"]), dev(g["k_bias"]), dev(g["d_skip"]),
                                        dev(g["z"]), chunk=64, dtype_policy="f32")
        assert rel_error(y, g["y"]) < F32_TOL
        assert rel_error(fs, g["ssm"]) < F32_TOL
        assert rel_error(fk, g["k_final"]) < F32_TOL


def test_unsupported_shape_raises():
    from mamba3_b200 import kernel_fwd as KF
    from mamba3_b200._capi import M3Error

    b, h, l, n, p, nr = 1, 1, 64, 16, 8, 4
    x, pre = pre_inputs(b, h, l, n, p, nr)
    with pytest.raises(M3Error):
        KF.siso_forward(dev(x["q"]), dev(x["k"]), dev(x["v"]), dev(pre.adt), dev(pre.gamma), dev(pre.scale),
                        dev(pre.phi), dev(x["q_bias"]), dev(x["k_bias"]), chunk=64, dtype_policy="f32")
    with pytest.raises(ValueError):
        KF.siso_forward(dev(x["q"]), dev(x["k"]), dev(x["v"]), dev(pre.adt), dev(pre.gamma), dev(pre.scale),
                        dev(pre.phi), dev(x["q_bias"]), dev(x["k_bias"]), chunk=96, dtype_policy="f32")
