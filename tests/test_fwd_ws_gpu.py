"""The warp-specialised TMA-fed tensor-core forward (raw boundary) against the float64
oracle with the reference kernel's bf16 rounding points (kernel_fwd.py:139-187), and
against the two-sequence tensor-core kernel it replaces: several sequences per CTA,
ungated and skip-free variants, seeds, few rotary pairs, the layer's strided views, the
saved backward states, and the forward without its rotary-rate workspace."""

import ctypes

import pytest
import torch

from oracle import siso_oracle as O
from tests.gpu_common import dev, pre_inputs, rand_state
from tests.metrics import max_rel, rel_error

pytestmark = pytest.mark.gpu
TOL = 2e-2
B16 = torch.bfloat16


@pytest.fixture(autouse=True)
def _no_device_error():
    from mamba3_b200 import _capi as C

    C.lib().m3_device_error(1)
    yield
    assert C.lib().m3_device_error(1) == 0


def _r(t):
    return t.to(B16).double()


def _case(b, h, l, nr, seed, seeded=False, gate=True, skip=True):
    x, _ = pre_inputs(b, h, l, 128, 64, nr, seed=seed)
    x["dt_bias"] = torch.randn(h, dtype=torch.float64, generator=torch.Generator().manual_seed(seed + 1)) * 0.3
    st = rand_state(b, h, 64, 128, nr) if seeded else None
    if not gate:
        x["z"] = None
    if not skip:
        x["d_skip"] = None
    return x, st


def _run(x, st, kernel, **kw):
    from mamba3_b200 import kernel_fwd as KF

    args = (dev(x["q"], B16), dev(x["k"], B16), dev(x["v"], B16), dev(x["dt_raw"]), dev(x["a_raw"]),
            dev(x["trap_raw"]), dev(x["angles"]), dev(x["dt_bias"]), dev(x["q_bias"]), dev(x["k_bias"]))
    seeds = {} if st is None else dict(seed_ssm=dev(st.ssm), seed_k=dev(st.k), seed_v=dev(st.v),
                                       seed_phi=dev(st.phi))
    return KF.siso_forward_raw(*args, d_skip=dev(x["d_skip"]), z=None if x["z"] is None else dev(x["z"], B16),
                               chunk=128, dtype_policy="bf16", kernel=kernel, **seeds, **kw)


def _oracle(x, st):
    return O.siso_segment(_r(x["q"]), _r(x["k"]), _r(x["v"]), x["dt_raw"], x["a_raw"], x["trap_raw"], x["angles"],
                          x["dt_bias"], x["q_bias"], x["k_bias"], x["d_skip"],
                          None if x["z"] is None else _r(x["z"]), state=st, chunk=128, policy="bf16")


@pytest.mark.parametrize("shape", [(2, 3, 256, 32), (1, 2, 512, 64), (3, 1, 128, 16), (2, 2, 384, 8)])
@pytest.mark.parametrize("seeded", [False, True])
def test_ws_forward_vs_oracle(shape, seeded):
    b, h, l, nr = shape
    x, st = _case(b, h, l, nr, seed=3 + l + nr, seeded=seeded)
    y_ref, fin = _oracle(x, st)
    y, fs, fk, fv, fphi = _run(x, st, "tensorcore")
    assert rel_error(y, y_ref) < TOL
    assert rel_error(fs, fin.ssm) < TOL
    assert rel_error(fk, fin.k) < 1e-5
    assert max_rel(fv, _r(fin.v)) < 1e-6
    assert rel_error(fphi, fin.phi, angle=True) < 1e-5
    y1, fs1, *_ = _run(x, st, "tensorcore_v1")
    assert rel_error(y, y1) < TOL
    assert rel_error(fs, fs1) < TOL


@pytest.mark.parametrize("gate,skip", [(False, True), (True, False), (False, False)])
def test_ws_forward_without_gate_or_skip(gate, skip):
    x, st = _case(2, 2, 256, 32, seed=17, gate=gate, skip=skip)
    y_ref, fin = _oracle(x, st)
    y, fs, *_ = _run(x, st, "tensorcore")
    assert rel_error(y, y_ref) < TOL
    assert rel_error(fs, fin.ssm) < TOL


def test_ws_forward_many_sequences_per_cta():
    """B·H = 320 > 148 SMs: most CTAs walk two or three sequences back to back, so the
    pipeline's barrier phases, TMEM buffers and carries cross sequence boundaries."""
    x, st = _case(10, 32, 256, 64, seed=29, seeded=True)
    y_ref, fin = _oracle(x, st)
    y, fs, fk, fv, fphi = _run(x, st, "tensorcore")
    assert rel_error(y, y_ref) < TOL
    assert rel_error(fs, fin.ssm) < TOL
    assert rel_error(fk, fin.k) < 1e-5
    assert rel_error(fphi, fin.phi, angle=True) < 1e-5
    # every sequence's output is there (a skipped one would hide inside a percentile)
    per_seq = (y.double().cpu() - y_ref).abs().amax((2, 3)) / y_ref.abs().amax((2, 3))
    assert float(per_seq.max()) < 0.1


def test_ws_forward_without_rotary_rate_workspace():
    """The same forward when the caller passes no workspace: tanh of the angles in-kernel."""
    from mamba3_b200 import _capi as C
    from mamba3_b200 import _tensors as T

    x, st = _case(2, 3, 256, 32, seed=41, seeded=True)
    y_ws, fs_ws, *_ = _run(x, st, "tensorcore")
    # direct C-ABI call with fwd_workspace = NULL
    b, h, l, n, p, nr = 2, 3, 256, 128, 64, 32
    io = lambda t: dev(t, B16).contiguous()
    q, k, v, z = io(x["q"]), io(x["k"]), io(x["v"]), io(x["z"])
    f = lambda t: dev(t).contiguous()
    raw = [f(x[n_]) for n_ in ("dt_raw", "a_raw", "trap_raw", "angles", "dt_bias", "q_bias", "k_bias", "d_skip")]
    seeds = [f(t) for t in (st.ssm, st.k, st.v, st.phi)]
    y = torch.empty(b, h, l, p, dtype=B16, device="cuda")
    fs = torch.empty(b, h, p, n, device="cuda")
    fk, fv, fphi = torch.empty(b, h, n, device="cuda"), torch.empty(b, h, p, device="cuda"), torch.empty(b, h, nr,
                                                                                                         device="cuda")
    a = C.M3FwdArgs()
    a.dims = C.M3Dims(b, l, h, n, p, nr, 128)
    a.io_dtype, a.policy, a.raw, a.a_floor = C.M3_DTYPE_BF16, C.M3_POLICY_BF16, 1, 1e-4
    a.q, a.k, a.v, a.z = q.data_ptr(), k.data_ptr(), v.data_ptr(), z.data_ptr()
    a.dt_raw, a.a_raw, a.trap_raw, a.angles, a.dt_bias, a.q_bias, a.k_bias, a.d_skip = (t.data_ptr() for t in raw)
    a.seed_ssm, a.seed_k, a.seed_v, a.seed_phi = (t.data_ptr() for t in seeds)
    a.y, a.final_ssm, a.final_k, a.final_v, a.final_phi = (t.data_ptr() for t in (y, fs, fk, fv, fphi))
    a.kernel = C.M3_KERNEL_TENSORCORE
    assert C.lib().m3_siso_fwd(ctypes.byref(a), T.stream_handle(y.device)) == C.M3_OK, C.lib().m3_last_error()
    torch.cuda.synchronize()
    assert rel_error(y, y_ws) < 1e-3
    assert rel_error(fs, fs_ws) < 1e-4


def test_ws_forward_layer_views_and_saved_states():
    """v / z / y as (B, L, H, P) buffers seen as (B, H, L, P) (the layer's in_proj slices),
    and the backward's chunk-start states saved by this forward: a backward that uses them
    matches one that recomputes them."""
    from mamba3_b200 import kernel_bwd as KB
    from mamba3_b200 import kernel_fwd as KF

    b, h, l, nr = 2, 4, 256, 32
    x, st = _case(b, h, l, nr, seed=53, seeded=True)
    vb = dev(x["v"], B16).permute(0, 2, 1, 3).contiguous()
    zb = dev(x["z"], B16).permute(0, 2, 1, 3).contiguous()
    yb = torch.empty_like(vb)
    raw = (dev(x["dt_raw"]), dev(x["a_raw"]), dev(x["trap_raw"]), dev(x["angles"]), dev(x["dt_bias"]),
           dev(x["q_bias"]), dev(x["k_bias"]))
    seeds = dict(seed_ssm=dev(st.ssm), seed_k=dev(st.k), seed_v=dev(st.v), seed_phi=dev(st.phi))
    ws = torch.zeros(KB.workspace_bytes(b, l, h, 128, 64, nr, 128), dtype=torch.uint8, device="cuda")
    q, k = dev(x["q"], B16), dev(x["k"], B16)
    _, saved = KF.siso_forward_raw(q, k, vb.permute(0, 2, 1, 3), *raw, d_skip=dev(x["d_skip"]),
                                   z=zb.permute(0, 2, 1, 3), chunk=128, dtype_policy="bf16", kernel="tensorcore",
                                   y_out=yb.permute(0, 2, 1, 3), bwd_states=ws, return_saved=True, **seeds)
    assert saved
    y_ref, _ = _oracle(x, st)
    assert rel_error(yb.permute(0, 2, 1, 3), y_ref) < TOL
    dy = dev(x["dy"], B16)
    common = dict(d_skip=dev(x["d_skip"]), z=dev(x["z"], B16), chunk=128, dtype_policy="bf16", kernel="tensorcore",
                  **seeds)
    v = dev(x["v"], B16)
    g_saved = KB.siso_backward_raw(dy, q, k, v, *raw, workspace=ws, states_ready=True, **common)
    g_sweep = KB.siso_backward_raw(dy, q, k, v, *raw, **common)
    for name in ("dq", "dk", "dv", "dz", "ddt_raw", "da_raw", "dtrap_raw", "dangles", "dseed_ssm", "dseed_phi"):
        a_, b_ = getattr(g_saved, name).double(), getattr(g_sweep, name).double()
        e = float((a_ - b_).norm() / b_.norm())
        assert e < 1e-2, (name, e)
