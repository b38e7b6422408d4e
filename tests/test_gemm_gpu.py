"""The skinny tcgen05 GEMM of the decode step's projections (``m3_gemm_bf16``) against a
plain PyTorch fp32 product of the same bf16 operands, rounded once to bf16 -- the matmul /
addmm calls of ``model.lm_decode_step`` it replaces (``model.py:244-296``): the configs[3]
projection shapes at B = 256 (in_proj with its N tail, out_proj and fc2 with the residual
and their K split over 4-CTA clusters, fc1), ragged row counts, the residual added in
place, a strided weight view, the tied head's K-major ``embed.t()``; and bit-equal repeats."""

import pytest
import torch

from tests.metrics import rel_error

pytestmark = pytest.mark.gpu
B16 = torch.bfloat16


@pytest.fixture(autouse=True)
def _no_device_error():
    from mamba3_b200 import _capi as C

    C.lib().m3_device_error(1)
    yield
    assert C.lib().m3_device_error(1) == 0


def _ref(x, w, residual=None):
    r = x.float() @ w.float()
    if residual is not None:
        r = r + residual.float()
    return r


def _check(out, ref):
    # one bf16 rounding of an fp32 sum whose order differs from torch's: within 2 bf16 ulps
    err = (out.float() - ref).abs()
    bound = ref.abs() * 2.0 ** -7 + 1e-3 * ref.abs().max()
    assert bool((err <= bound).all()), float((err - bound).max())
    assert rel_error(out, ref) < 5e-3


def _rand(*shape, scale=1.0, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(B16).cuda()


@pytest.mark.parametrize("m,k,n,res", [
    (256, 2048, 8672, False),   # in_proj: 68 column tiles, the last one 96 wide
    (256, 4096, 2048, True),    # out_proj + residual: 16 tiles x 4-CTA K split
    (256, 2048, 8192, False),   # fc1
    (100, 4096, 2048, True),    # ragged rows (one 128-row half only)
    (129, 512, 136, False),     # just over one half; an 8-column tail tile
    (1, 1024, 64, True),        # one row, a column tile of 64
    (32, 2048, 8672, False),    # decode batch 32 per GPU
    (30, 4096, 2048, True),     # rows not a multiple of 8
    (64, 2048, 8192, False),
    (120, 4096, 2048, True),
])
def test_gemm_matches_fp32_product(m, k, n, res):
    from mamba3_b200 import projection as PJ

    x = _rand(m, k, scale=0.5, seed=m + k)
    w = _rand(k, n, scale=k ** -0.5, seed=n)
    r = _rand(m, n, seed=7) if res else None
    assert PJ.gemm_eligible(x, w)
    out = PJ.gemm(x, w, residual=r)
    torch.cuda.synchronize()
    _check(out, _ref(x, w, r))
    again = PJ.gemm(x, w, residual=r)
    torch.cuda.synchronize()
    assert torch.equal(out, again)  # the K split is summed in a fixed order


@pytest.mark.parametrize("ksplit", [1, 2, 4])
def test_gemm_explicit_k_split(ksplit):
    from mamba3_b200 import projection as PJ

    m, k, n = 200, 1024, 512
    x = _rand(m, k, scale=0.5, seed=21)
    w = _rand(k, n, scale=k ** -0.5, seed=22)
    r = _rand(m, n, seed=23)
    _check(PJ.gemm(x, w, residual=r, ksplit=ksplit), _ref(x, w, r))


def test_gemm_residual_in_place_and_strided_views():
    """out_proj's ``x = x + y @ W`` written over x; x and w as column slices of wider buffers."""
    from mamba3_b200 import projection as PJ

    m, k, n = 256, 4096, 2048
    xbuf = _rand(m, k + 64, scale=0.5, seed=1)
    x = xbuf[:, 64:]
    wbuf = _rand(k, n + 128, scale=k ** -0.5, seed=2)
    w = wbuf[:, :n]
    res = _rand(m, n, seed=3)
    want = _ref(x, w, res)
    PJ.gemm(x, w, residual=res, out=res)
    torch.cuda.synchronize()
    _check(res, want)


def test_gemm_k_major_weights_tied_head():
    """The tied head ``x @ embed.t()`` with embed (V, d) row-major: w is K-major."""
    from mamba3_b200 import projection as PJ

    m, d, v = 256, 2048, 4096
    x = _rand(m, d, scale=0.5, seed=11)
    embed = _rand(v, d, scale=d ** -0.5, seed=12)
    w = embed.t()
    assert PJ.gemm_eligible(x, w, w_kmajor=True)
    out = PJ.gemm(x, w, w_kmajor=True)
    torch.cuda.synchronize()
    _check(out, _ref(x, w))


def test_gemm_rejects_unsupported_shapes():
    from mamba3_b200 import _capi as C

    a = C.M3GemmArgs()
    a.m, a.n, a.k = 300, 128, 64
    a.a = a.w = a.out = 256
    assert C.lib().m3_gemm_bf16(a, None) == C.M3_ERR_SHAPE
    a.m, a.k = 16, 100
    assert C.lib().m3_gemm_bf16(a, None) == C.M3_ERR_UNSUPPORTED
