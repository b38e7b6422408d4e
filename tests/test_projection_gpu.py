"""Small-batch decode projections (`projection.small_proj`, ``m3_gemv_bf16``) against the
torch ops they replace in ``model.py:244-296`` (rms_norm -> matmul, addmm, the gated MLP),
and `lm_decode_step` at batch <= 8 against its cuBLAS path."""

import pytest
import torch


pytestmark = pytest.mark.gpu


def _normwise(a, b):
    a, b = a.double(), b.double()
    return float((a - b).norm() / b.norm())


@pytest.mark.parametrize("m", [1, 3, 8])
@pytest.mark.parametrize("k,n", [(2048, 8672), (4096, 2048), (512, 1064)])
def test_modes_match_torch(m, k, n):
    from mamba3_b200 import layer as LY
    from mamba3_b200 import projection as PJ

    g = torch.Generator(device="cuda").manual_seed(m * 7 + k)
    r = lambda *s: torch.randn(*s, device="cuda", generator=g)
    w = (r(k, n) / k ** 0.5).bfloat16()
    x = r(m, k).bfloat16()
    nw = 1 + 0.1 * r(k)
    res = r(m, n).bfloat16()
    xx = r(m, 2 * k).bfloat16()
    cases = {
        "plain": (PJ.small_proj(x, w), torch.matmul(x, w)),
        "norm": (PJ.small_proj(x, w, norm_w=nw, eps=1e-5), torch.matmul(LY.rms_norm(x, nw, 1e-5), w)),
        "residual": (PJ.small_proj(x, w, residual=res), torch.addmm(res, x, w)),
        "silu_gate": (PJ.small_proj(xx, w, silu_gate=True, residual=res),
                      torch.addmm(res, xx[:, :k] * torch.nn.functional.silu(xx[:, k:]), w)),
    }
    for name, (got, want) in cases.items():
        assert got.shape == want.shape and got.dtype == torch.bfloat16
        assert _normwise(got, want) < 1e-2, name  # bf16 output rounding, different summation order
    again = PJ.small_proj(xx, w, silu_gate=True, residual=res)
    assert torch.equal(again, cases["silu_gate"][0]), "not deterministic"


@pytest.mark.parametrize("batch", [1])
def test_decode_step_small_batch_path(batch, monkeypatch):
    from mamba3_b200 import layer as LY
    from mamba3_b200 import model as M
    from mamba3_b200 import projection as PJ

    scfg = LY.SISOConfig(d_model=256, d_state=128, headdim=64, chunk=128, policy_name="bf16")
    cfg = M.LMConfig(vocab_size=512, n_layers=3, siso=scfg, d_intermediate=384)
    params = M.init_lm(cfg, key=1, dtype=torch.bfloat16)
    toks = torch.randint(0, 512, (batch, 6), device="cuda", generator=torch.Generator(device="cuda").manual_seed(1))
    st_a, st_b = M.zero_states(cfg, batch), M.zero_states(cfg, batch)
    for t in range(6):
        la, st_a = M.lm_decode_step(params, toks[:, t], st_a, cfg)
        with monkeypatch.context() as mp:
            mp.setattr(PJ, "eligible", lambda *a: False)
            lb, st_b = M.lm_decode_step(params, toks[:, t], st_b, cfg)
        assert _normwise(la.float(), lb.float()) < 2e-2, t
    for a, b in zip(st_a, st_b):  # bf16 rounding differences carried through 6 steps
        assert _normwise(a.ssm, b.ssm) < 2e-2


@pytest.mark.parametrize("rows,k", [(256, 4096), (3, 1064)])
def test_gated_activation_matches_torch(rows, k):
    """`projection.gated_act` (``m3_gated_act_bf16``) equals value * silu(gate) in torch bf16."""
    from mamba3_b200 import projection as PJ

    h = torch.randn(rows, 2 * k, device="cuda", generator=torch.Generator(device="cuda").manual_seed(k)).bfloat16()
    got = PJ.gated_act(h)
    value, gate = h.chunk(2, dim=-1)
    want = value * torch.nn.functional.silu(gate)
    assert got.shape == want.shape and got.dtype == torch.bfloat16
    assert (got.float() - want.float()).abs().max() <= 1e-2 * want.float().abs().max()
