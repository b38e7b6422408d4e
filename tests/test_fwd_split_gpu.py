"""The forward with every sequence cut into segments scanned side by side
(`kernel_fwd._forward_raw_split`: per-tile angle and decay sums, a states-only pass, the
carries rebuilt serially over the segments, then the full forward of all segments), against the unsplit forward and the
float64 oracle -- with and without a carried state, and the automatic choice of the
segment count for a batch of few (b, h) sequences."""

import pytest
import torch

from oracle import siso_oracle as O
from tests.gpu_common import dev, rand_state
from tests.metrics import rel_error
from tests.test_baseline_shapes_gpu import RAW, _dev_args, cfg1_inputs

pytestmark = pytest.mark.gpu
B16 = torch.bfloat16
TOL = 2e-2


@pytest.fixture(autouse=True)
def _no_device_error():
    from mamba3_b200 import _capi as C

    C.lib().m3_device_error(1)
    yield
    assert C.lib().m3_device_error(1) == 0


@pytest.mark.parametrize("seeded", [False, True])
@pytest.mark.parametrize("b,h,l,segments", [(1, 8, 4096, 2), (1, 8, 4096, 4), (2, 3, 2048, 4)])
def test_split_forward_matches_unsplit_and_oracle(seeded, b, h, l, segments):
    from mamba3_b200 import kernel_fwd as KF

    x = cfg1_inputs(b, h, l, seed=300 + segments + int(seeded))
    st = rand_state(b, h, 64, 128, 64) if seeded else None
    seeds = {} if st is None else dict(seed_ssm=dev(st.ssm), seed_k=dev(st.k), seed_v=dev(st.v),
                                       seed_phi=dev(st.phi))
    kw = dict(d_skip=dev(x["d_skip"]), z=dev(x["z"], B16), chunk=128, dtype_policy="bf16", kernel="tensorcore",
              **seeds)
    y1, s1, k1, v1, p1 = KF.siso_forward_raw(*_dev_args(x), lsplit=1, **kw)
    ys, ss, ks, vs, ps = KF.siso_forward_raw(*_dev_args(x), lsplit=segments, **kw)
    y_ref, fin = O.siso_segment(*(x[k_] for k_ in RAW), x["d_skip"], x["z"], state=st, chunk=128, policy="bf16")
    assert rel_error(ys, y1) < TOL and rel_error(ys, y_ref) < TOL
    assert rel_error(ss, s1) < TOL and rel_error(ss, fin.ssm) < TOL
    assert rel_error(ks, fin.k) < 1e-4
    assert torch.equal(vs, v1)
    assert rel_error(ps, fin.phi, angle=True) < 1e-4
    # every segment's output is there
    per = (ys.double().cpu() - y_ref).abs().amax(-1) / y_ref.abs().amax()
    assert float(per.max()) < 0.1


def test_auto_split_fills_the_gpu():
    from mamba3_b200 import kernel_fwd as KF

    b, h, l = 1, 32, 8192
    x = cfg1_inputs(b, h, l, seed=17)
    q = dev(x["q"], B16)
    v = dev(x["v"], B16)
    g = KF._auto_split(q, v, dev(x["angles"]), 128, "bf16", "auto")
    nsm = torch.cuda.get_device_properties(0).multi_processor_count
    assert g > 1 and b * h * g <= nsm
    y, fs, *_ = KF.siso_forward_raw(*_dev_args(x), d_skip=dev(x["d_skip"]), z=dev(x["z"], B16), chunk=128,
                                    dtype_policy="bf16")
    y_ref, fin = O.siso_segment(*(x[k_] for k_ in RAW), x["d_skip"], x["z"], chunk=128, policy="bf16")
    assert rel_error(y, y_ref) < TOL
    assert rel_error(fs, fin.ssm) < TOL


@pytest.mark.parametrize("seeded", [False, True])
@pytest.mark.parametrize("b,h,l", [(2, 32, 4096), (1, 8, 2048)])
def test_two_segment_chain_matches_unsplit_and_oracle(seeded, b, h, l):
    """`kernel_fwd._forward_raw_chain2` (segment 0's full pass on a side stream beside its
    states-only pass, then segment 1 from that carry): the automatic path when B * H fills
    at most half the SMs."""
    from mamba3_b200 import kernel_fwd as KF

    x = cfg1_inputs(b, h, l, seed=400 + b + int(seeded))
    st = rand_state(b, h, 64, 128, 64) if seeded else None
    seeds = {} if st is None else dict(seed_ssm=dev(st.ssm), seed_k=dev(st.k), seed_v=dev(st.v),
                                       seed_phi=dev(st.phi))
    kw = dict(d_skip=dev(x["d_skip"]), z=dev(x["z"], B16), chunk=128, dtype_policy="bf16", kernel="tensorcore",
              **seeds)
    args = _dev_args(x)
    assert KF._chain_fits(args[0], args[2], args[6], 128, "bf16", "tensorcore")
    y1, s1, k1, v1, p1 = KF.siso_forward_raw(*args, lsplit=1, **kw)
    yc, sc, kc, vc, pc = KF._forward_raw_chain2(*args, kw["d_skip"], kw["z"], *(seeds.get(n) for n in (
        "seed_ssm", "seed_k", "seed_v", "seed_phi")), 1e-4, 128, "bf16", None, "tensorcore")
    ya, *_ = KF.siso_forward_raw(*args, **kw)  # the automatic choice takes the same path
    torch.cuda.synchronize()
    assert torch.equal(ya, yc)
    y_ref, fin = O.siso_segment(*(x[k_] for k_ in RAW), x["d_skip"], x["z"], state=st, chunk=128, policy="bf16")
    assert rel_error(yc, y1) < TOL and rel_error(yc, y_ref) < TOL
    assert rel_error(sc, s1) < TOL and rel_error(sc, fin.ssm) < TOL
    assert rel_error(kc, fin.k) < 1e-4
    assert torch.equal(vc, v1)
    assert rel_error(pc, fin.phi, angle=True) < 1e-4
    per = (yc.double().cpu() - y_ref).abs().amax(-1) / y_ref.abs().amax()
    assert float(per.max()) < 0.1
