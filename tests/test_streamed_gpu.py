"""`siso_segment_streamed` (pinned host inputs, segments along L, host y) against
`siso_segment` on device tensors: the same scan, cut where the reference's segmentation
rule allows (siso.py:176-181)."""

import pytest
import torch

from tests.gpu_common import dev, pre_inputs
from tests.metrics import rel_error

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shape,dtype,policy,tol", [((2, 3, 512, 128, 64, 32, 128), torch.bfloat16, "bf16", 2e-2),
                                                   ((2, 3, 256, 32, 16, 8, 64), torch.float32, "fp32", 1e-5)])
def test_streamed_matches_device_segment(shape, dtype, policy, tol):
    from mamba3_b200 import siso as S

    b, h, l, n, p, nr, chunk = shape
    x, _ = pre_inputs(b, h, l, n, p, nr, seed=21)
    hq, hk = x["q"].to(dtype).pin_memory(), x["k"].to(dtype).pin_memory()
    hv = x["v"].permute(0, 2, 1, 3).contiguous().to(dtype).pin_memory()  # (B, L, H, P)
    hz = x["z"].permute(0, 2, 1, 3).contiguous().to(dtype).pin_memory()
    raw = {k_: x[k_].float().pin_memory() for k_ in ("dt_raw", "a_raw", "trap_raw", "angles")}
    par = [dev(x[k_]) for k_ in ("dt_bias", "q_bias", "k_bias", "d_skip")]
    out = S.siso_segment_streamed(hq, hk, hv, raw["dt_raw"], raw["a_raw"], raw["trap_raw"], raw["angles"], *par,
                                  hz, chunk=chunk, policy_name=policy, segments=4)
    torch.cuda.synchronize()
    ref = S.siso_segment(hq.cuda(), hk.cuda(), hv.cuda().permute(0, 2, 1, 3), raw["dt_raw"].cuda(),
                         raw["a_raw"].cuda(), raw["trap_raw"].cuda(), raw["angles"].cuda(), *par,
                         hz.cuda().permute(0, 2, 1, 3), chunk=chunk, policy_name=policy)
    assert out.y.device.type == "cpu" and out.y.is_pinned()
    assert rel_error(out.y.permute(0, 2, 1, 3), ref.y.cpu()) < tol
    assert rel_error(out.state.ssm, ref.state.ssm) < tol
    assert rel_error(out.state.phi, ref.state.phi, angle=True) < 1e-5
