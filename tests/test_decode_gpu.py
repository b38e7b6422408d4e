"""Decode kernel parity (``mamba3_pallas/tests.py:734-877``): one step vs the step
oracle from zero and seeded states, the raw (fused preprocess) step, a chain vs the
chunked prefill, and the prefill -> decode handoff."""

import pytest
import torch

from oracle import siso_oracle as O
from tests.gpu_common import DEV, dev, pre_inputs, rand_state
from tests.metrics import rel_error

pytestmark = pytest.mark.gpu
F32_TOL = 1e-5


def _st_dev(st):
    from mamba3_b200.state import SISOState

    return SISOState(*(dev(t).contiguous() for t in st))


@pytest.mark.parametrize("shape", [(2, 3, 128, 64, 32), (3, 16, 32, 32, 8), (2, 2, 16, 16, 4), (1, 2, 64, 64, 32)])
@pytest.mark.parametrize("seeded", [False, True])
def test_one_step_matches_step_oracle(shape, seeded):
    from mamba3_b200 import kernel_decode as KD

    b, h, n, p, nr = shape
    x, pre = pre_inputs(b, h, 64, n, p, nr, seed=11)
    st = rand_state(b, h, p, n, nr) if seeded else O.zero_state(b, h, p, n, nr)
    args = (x["q"][:, 0], x["k"][:, 0], x["v"][:, :, 0], pre.adt[:, :, 0], pre.dt[:, :, 0], pre.lam[:, :, 0],
            x["angles"][:, 0], x["q_bias"], x["k_bias"])
    y_ref, s_ref = O.siso_step(*args, st, x["d_skip"], x["z"][:, :, 0])
    sd = _st_dev(st)
    y, s = KD.siso_decode(*(dev(a) for a in args), sd, d_skip=dev(x["d_skip"]), z=dev(x["z"][:, :, 0]),
                          dtype_policy="f32")
    assert s.ssm.data_ptr() == sd.ssm.data_ptr()  # updated in place, like the reference's donation
    assert rel_error(y, y_ref) < F32_TOL
    assert rel_error(s.ssm, s_ref.ssm) < F32_TOL
    assert rel_error(s.k, s_ref.k) < F32_TOL
    assert rel_error(s.v, s_ref.v) < 1e-7
    assert rel_error(s.phi, s_ref.phi, angle=True) < 1e-5


def test_raw_step_fuses_preprocess():
    from mamba3_b200 import kernel_decode as KD

    b, h, n, p, nr = 4, 8, 128, 64, 32
    x, pre = pre_inputs(b, h, 64, n, p, nr, seed=12)
    x["dt_bias"] = torch.randn(h, dtype=torch.float64) * 0.2
    pre, _ = O.preprocess(x["dt_raw"], x["a_raw"], x["trap_raw"], x["angles"], x["dt_bias"])
    st = rand_state(b, h, p, n, nr)
    y_ref, s_ref = O.siso_step(x["q"][:, 0], x["k"][:, 0], x["v"][:, :, 0], pre.adt[:, :, 0], pre.dt[:, :, 0],
                               pre.lam[:, :, 0], x["angles"][:, 0], x["q_bias"], x["k_bias"], st, x["d_skip"],
                               x["z"][:, :, 0])
    y, s = KD.siso_decode_raw(dev(x["q"][:, 0]), dev(x["k"][:, 0]), dev(x["v"][:, :, 0]), dev(x["dt_raw"][:, 0]),
                              dev(x["a_raw"][:, 0]), dev(x["trap_raw"][:, 0]), dev(x["angles"][:, 0]),
                              dev(x["dt_bias"]), dev(x["q_bias"]), dev(x["k_bias"]), _st_dev(st),
                              d_skip=dev(x["d_skip"]), z=dev(x["z"][:, :, 0]), dtype_policy="f32")
    assert rel_error(y, y_ref) < F32_TOL
    assert rel_error(s.ssm, s_ref.ssm) < F32_TOL


def test_bf16_step():
    from mamba3_b200 import kernel_decode as KD

    b, h, n, p, nr = 4, 8, 128, 64, 32
    x, pre = pre_inputs(b, h, 64, n, p, nr, seed=13)
    st = rand_state(b, h, p, n, nr)
    r = lambda t: t.to(torch.bfloat16).double()
    y_ref, s_ref = O.siso_step(r(x["q"][:, 0]), r(x["k"][:, 0]), r(x["v"][:, :, 0]), pre.adt[:, :, 0],
                               pre.dt[:, :, 0], pre.lam[:, :, 0], x["angles"][:, 0], x["q_bias"], x["k_bias"], st,
                               x["d_skip"], r(x["z"][:, :, 0]), policy="bf16")
    b16 = torch.bfloat16
    y, s = KD.siso_decode(dev(x["q"][:, 0], b16), dev(x["k"][:, 0], b16), dev(x["v"][:, :, 0], b16),
                          dev(pre.adt[:, :, 0]), dev(pre.dt[:, :, 0]), dev(pre.lam[:, :, 0]), dev(x["angles"][:, 0]),
                          dev(x["q_bias"]), dev(x["k_bias"]), _st_dev(st), d_skip=dev(x["d_skip"]),
                          z=dev(x["z"][:, :, 0], b16), dtype_policy="bf16")
    assert y.dtype == torch.bfloat16
    assert rel_error(y, y_ref) < 2e-2
    assert rel_error(s.ssm, s_ref.ssm) < 1e-5


def test_chain_equals_prefill_and_handoff():
    from mamba3_b200 import kernel_decode as KD
    from mamba3_b200 import kernel_fwd as KF
    from mamba3_b200.state import zero_state

    b, h, l, n, p, nr = 1, 2, 256, 128, 64, 32
    x, pre = pre_inputs(b, h, l, n, p, nr, seed=11)
    d = {k_: dev(v_) for k_, v_ in x.items()}
    dp = {k_: dev(getattr(pre, k_)) for k_ in ("adt", "dt", "lam", "gamma", "scale", "phi")}
    y_dec, s_dec = KD.decode_loop(d["q"], d["k"], d["v"], dp["adt"], dp["dt"], dp["lam"], d["angles"], d["q_bias"],
                                  d["k_bias"], zero_state(b, h, p, n, nr, device=DEV), d["d_skip"], d["z"],
                                  dtype_policy="f32")
    y_pre, fs, fk, fv = KF.siso_forward(d["q"], d["k"], d["v"], dp["adt"], dp["gamma"], dp["scale"], dp["phi"],
                                        d["q_bias"], d["k_bias"], d["d_skip"], d["z"], chunk=128, dtype_policy="f32")
    assert rel_error(y_dec, y_pre) < 2e-5
    assert rel_error(s_dec.ssm, fs) < 2e-5
    assert rel_error(s_dec.k, fk) < 2e-5
    # prefill half, decode the rest (tests.py:846-875)
    half = l // 2
    import mamba3_b200.siso as S

    o1 = S.siso_segment(d["q"][:, :half], d["k"][:, :half], d["v"][:, :, :half], d["dt_raw"][:, :half],
                        d["a_raw"][:, :half], d["trap_raw"][:, :half], d["angles"][:, :half], d["dt_bias"],
                        d["q_bias"], d["k_bias"], d["d_skip"], d["z"][:, :, :half], chunk=128, policy_name="f32")
    st = o1.state
    ys = []
    for t in range(half, l):
        y, st = KD.siso_decode_raw(d["q"][:, t], d["k"][:, t], d["v"][:, :, t], d["dt_raw"][:, t], d["a_raw"][:, t],
                                   d["trap_raw"][:, t], d["angles"][:, t], d["dt_bias"], d["q_bias"], d["k_bias"],
                                   st, d_skip=d["d_skip"], z=d["z"][:, :, t], dtype_policy="f32")
        ys.append(y)
    y_all = torch.cat([o1.y, torch.stack(ys, 2)], dim=2)
    assert rel_error(y_all, y_pre) < 2e-5


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("shape", [(4, 8, 128, 64, 32), (3, 4, 32, 32, 8)])
def test_fused_norms_and_inproj_columns(dtype, shape):
    """The decode step as `model.lm_decode_step` drives it: raw C / B columns normalised in
    the kernel and the dt / A / trap / angle columns of one in_proj row read in place
    (bf16 in a bf16 model), against the layer's own RMS norm + fp32 columns."""
    from mamba3_b200 import kernel_decode as KD
    from mamba3_b200 import layer as LY
    from mamba3_b200.state import SISOState

    b, h, n, p, nr = shape
    g = torch.Generator(device="cuda").manual_seed(3)
    r = lambda *s: torch.randn(*s, device="cuda", generator=g)
    width = 2 * h * p + 2 * n + 3 * h + nr
    proj = (r(b, width) * 0.7).to(dtype)
    s0 = 2 * h * p + 2 * n
    z, xx = proj[:, :h * p].view(b, h, p), proj[:, h * p:2 * h * p].view(b, h, p)
    kb, qc = proj[:, 2 * h * p:2 * h * p + n], proj[:, 2 * h * p + n:s0]
    cols = [proj[:, s0:s0 + h], proj[:, s0 + h:s0 + 2 * h], proj[:, s0 + 2 * h:s0 + 3 * h], proj[:, s0 + 3 * h:]]
    wq, wk = 1 + 0.1 * r(n), 1 + 0.1 * r(n)
    dtb, qb, kbias, dsk = 0.3 * r(h), 0.1 * r(h, n), 0.1 * r(h, n), r(h)

    def state():
        gs = torch.Generator(device="cuda").manual_seed(4)
        rs = lambda *s: torch.randn(*s, device="cuda", generator=gs)
        return SISOState(ssm=rs(b, h, p, n) * 0.3, k=rs(b, h, n), v=rs(b, h, p), phi=rs(b, h, nr).abs())

    s1, s2 = state(), state()
    y1, _ = KD.siso_decode_raw(qc, kb, xx, *cols, dtb, qb, kbias, s1, d_skip=dsk, z=z, q_norm_w=wq, k_norm_w=wk,
                               norm_eps=1e-5, dtype_policy="f32" if dtype == torch.float32 else "bf16")
    qn, kn = LY.rms_norm(qc, wq, 1e-5), LY.rms_norm(kb, wk, 1e-5)
    y2, _ = KD.siso_decode_raw(qn, kn, xx, *(c.float() for c in cols), dtb, qb, kbias, s2, d_skip=dsk, z=z,
                               dtype_policy="f32" if dtype == torch.float32 else "bf16")
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    assert rel_error(y1, y2) < tol
    for name, a, c in zip(("ssm", "k", "v", "phi"), s1, s2):
        assert rel_error(a, c) < tol, name
