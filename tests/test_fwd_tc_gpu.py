"""The tcgen05 tensor-core forward (bf16 I/O, bf16 operands, N=128, P=64, chunk % 128 == 0)
against the oracle with the reference kernel's bf16 rounding points (kernel_fwd.py:139-187)
and against the generic kernel, on both boundaries."""

import pytest
import torch

from oracle import siso_oracle as O
from tests.gpu_common import dev, pre_inputs, rand_state
from tests.metrics import max_rel, rel_error

pytestmark = pytest.mark.gpu
TOL = 2e-2
B16 = torch.bfloat16


def _r(t):
    return t.to(B16).double()


@pytest.fixture(autouse=True)
def _no_device_error():
    from mamba3_b200 import _capi as C

    C.lib().m3_device_error(1)
    yield
    assert C.lib().m3_device_error(1) == 0


@pytest.mark.parametrize("shape", [(2, 3, 256, 128, 64, 32, 128), (1, 3, 512, 128, 64, 64, 256),
                                   (3, 1, 128, 128, 64, 16, 128)])
@pytest.mark.parametrize("seeded", [False, True])
def test_tc_raw_boundary(shape, seeded):
    from mamba3_b200 import kernel_fwd as KF

    b, h, l, n, p, nr, chunk = shape
    x, _ = pre_inputs(b, h, l, n, p, nr, seed=4)
    x["dt_bias"] = torch.randn(h, dtype=torch.float64, generator=torch.Generator().manual_seed(8)) * 0.3
    st = rand_state(b, h, p, n, nr) if seeded else None
    y_ref, fin = O.siso_segment(_r(x["q"]), _r(x["k"]), _r(x["v"]), x["dt_raw"], x["a_raw"], x["trap_raw"],
                                x["angles"], x["dt_bias"], x["q_bias"], x["k_bias"], x["d_skip"], _r(x["z"]),
                                state=st, chunk=chunk, policy="bf16")
    args = (dev(x["q"], B16), dev(x["k"], B16), dev(x["v"], B16), dev(x["dt_raw"]), dev(x["a_raw"]),
            dev(x["trap_raw"]), dev(x["angles"]), dev(x["dt_bias"]), dev(x["q_bias"]), dev(x["k_bias"]),
            dev(x["d_skip"]), dev(x["z"], B16))
    kw = dict(seed_ssm=None if st is None else dev(st.ssm), seed_k=None if st is None else dev(st.k),
              seed_v=None if st is None else dev(st.v), seed_phi=None if st is None else dev(st.phi), chunk=chunk,
              dtype_policy="bf16")
    y, fs, fk, fv, fphi = KF.siso_forward_raw(*args, kernel="tensorcore", **kw)
    assert rel_error(y, y_ref) < TOL
    assert rel_error(fs, fin.ssm) < TOL
    assert rel_error(fk, fin.k) < 1e-5
    assert max_rel(fv, _r(fin.v)) < 1e-6
    assert rel_error(fphi, fin.phi, angle=True) < 1e-5
    yg, fsg, *_ = KF.siso_forward_raw(*args, kernel="generic", **kw)
    assert rel_error(y, yg) < TOL
    assert rel_error(fs, fsg) < TOL


def test_tc_raw_boundary_strong_decay():
    """Large dt in the first half of the sequence: there the decay over a 32-token block
    exceeds 2^64, so the mask takes its direct exp2(min(A_i - A_j, 0)) form; the second half
    takes the factored form.  Both against the oracle."""
    from mamba3_b200 import kernel_fwd as KF

    b, h, l, n, p, nr, chunk = 2, 2, 512, 128, 64, 32, 128
    x, _ = pre_inputs(b, h, l, n, p, nr, seed=11)
    x["dt_raw"][:, : l // 2] += 3.0
    x["dt_bias"] = torch.zeros(h, dtype=torch.float64)
    y_ref, fin = O.siso_segment(_r(x["q"]), _r(x["k"]), _r(x["v"]), x["dt_raw"], x["a_raw"], x["trap_raw"],
                                x["angles"], x["dt_bias"], x["q_bias"], x["k_bias"], x["d_skip"], _r(x["z"]),
                                chunk=chunk, policy="bf16")
    args = (dev(x["q"], B16), dev(x["k"], B16), dev(x["v"], B16), dev(x["dt_raw"]), dev(x["a_raw"]),
            dev(x["trap_raw"]), dev(x["angles"]), dev(x["dt_bias"]), dev(x["q_bias"]), dev(x["k_bias"]),
            dev(x["d_skip"]), dev(x["z"], B16))
    y, fs, *_ = KF.siso_forward_raw(*args, kernel="tensorcore", chunk=chunk, dtype_policy="bf16")
    assert torch.isfinite(y.float()).all()
    assert rel_error(y, y_ref) < TOL
    assert rel_error(fs, fin.ssm) < TOL


@pytest.mark.parametrize("gate_skip", [True, False])
def test_tc_preprocessed_boundary_with_residuals(gate_skip):
    from mamba3_b200 import kernel_fwd as KF

    b, h, l, n, p, nr, chunk = 2, 3, 384, 128, 64, 32, 128
    x, pre = pre_inputs(b, h, l, n, p, nr, seed=6)
    dsk = x["d_skip"] if gate_skip else None
    z = x["z"] if gate_skip else None
    y_ref, st_ref, dbg = O.siso_chunked(_r(x["q"]), _r(x["k"]), _r(x["v"]), pre.adt, pre.gamma, pre.scale, pre.phi,
                                        x["q_bias"], x["k_bias"], dsk, None if z is None else _r(z), chunk=chunk,
                                        policy="bf16", return_debug=True)
    y, fs, fk, fv, res = KF.siso_forward(dev(x["q"], B16), dev(x["k"], B16), dev(x["v"], B16), dev(pre.adt),
                                         dev(pre.gamma), dev(pre.scale), dev(pre.phi), dev(x["q_bias"]),
                                         dev(x["k_bias"]), dev(dsk), dev(z, B16) if z is not None else None,
                                         chunk=chunk, dtype_policy="bf16", save_residuals=True, kernel="tensorcore")
    assert rel_error(y, y_ref) < TOL
    assert rel_error(fs, st_ref.ssm) < TOL
    assert rel_error(res.ybar, dbg["ybar"]) < TOL
    assert rel_error(res.chunk_states, dbg["chunk_states"]) < TOL


def test_tc_strided_views_like_the_layer():
    """v / z as permuted views of a (B, L, H, P) buffer, y written into one."""
    from mamba3_b200 import kernel_fwd as KF

    b, h, l, n, p, nr = 2, 4, 256, 128, 64, 32
    x, _ = pre_inputs(b, h, l, n, p, nr, seed=2)
    vb = dev(x["v"], B16).permute(0, 2, 1, 3).contiguous()   # (B, L, H, P)
    zb = dev(x["z"], B16).permute(0, 2, 1, 3).contiguous()
    yb = torch.empty_like(vb)
    common = (dev(x["q"], B16), dev(x["k"], B16))
    rest = (dev(x["dt_raw"]), dev(x["a_raw"]), dev(x["trap_raw"]), dev(x["angles"]), dev(x["dt_bias"]),
            dev(x["q_bias"]), dev(x["k_bias"]), dev(x["d_skip"]))
    KF.siso_forward_raw(*common, vb.permute(0, 2, 1, 3), *rest, z=zb.permute(0, 2, 1, 3), chunk=128,
                        dtype_policy="bf16", y_out=yb.permute(0, 2, 1, 3), kernel="tensorcore")
    y2, *_ = KF.siso_forward_raw(*common, dev(x["v"], B16), *rest, z=dev(x["z"], B16), chunk=128,
                                 dtype_policy="bf16", kernel="tensorcore")
    assert torch.equal(yb.permute(0, 2, 1, 3), y2)


def test_tc_rejects_ineligible_shapes():
    from mamba3_b200 import kernel_fwd as KF
    from mamba3_b200._capi import M3Error

    x, pre = pre_inputs(1, 2, 128, 64, 64, 16)
    with pytest.raises(M3Error):
        KF.siso_forward(dev(x["q"], B16), dev(x["k"], B16), dev(x["v"], B16), dev(pre.adt), dev(pre.gamma),
                        dev(pre.scale), dev(pre.phi), dev(x["q_bias"]), dev(x["k_bias"]), chunk=128,
                        dtype_policy="bf16", kernel="tensorcore")


def test_states_only_forward_matches_full_forward():
    """y == NULL runs the states-only kernel: the final state equals the full forward's."""
    from mamba3_b200 import kernel_fwd as KF
    from tests.gpu_common import dev
    from tests.test_bwd_gpu import _raw_case

    x, st, _ = _raw_case((2, 3, 256, 128, 64, 32, 128), True, seed=51)
    io = lambda t: dev(t, torch.bfloat16)
    args = (io(x["q"]), io(x["k"]), io(x["v"]), dev(x["dt_raw"]), dev(x["a_raw"]), dev(x["trap_raw"]),
            dev(x["angles"]), dev(x["dt_bias"]), dev(x["q_bias"]), dev(x["k_bias"]))
    kw = dict(d_skip=dev(x["d_skip"]), z=io(x["z"]), seed_ssm=dev(st.ssm), seed_k=dev(st.k), seed_v=dev(st.v),
              seed_phi=dev(st.phi), chunk=128, dtype_policy="bf16")
    assert KF.final_state_supported(args[0], args[2], args[6], 128)
    full = KF.siso_forward_raw(*args, **kw)
    only = KF.siso_forward_raw(*args, **kw, states_only=True)
    assert only[0] is None
    # the two instantiations round a few bf16 operands differently (measured: 1e-4 relative
    # on the state at most), well inside the bf16-policy tolerance
    for name, a, b in zip(("ssm", "k", "v", "phi"), only[1:], full[1:]):
        assert rel_error(a, b) < 1e-3 and float((a - b).abs().max()) < 1e-3, (name, float((a - b).abs().max()))
