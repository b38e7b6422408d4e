"""Token sampling (``train.py:454-500`` `_pick_token`, window bookkeeping
``train.py:548-579``): the oracle's filter against hand-worked cases, the CUDA sampler's
filtered distribution against the oracle, its draws against that distribution, and the
device-side window / stop / history state against a host replay of the reference loop."""

import math

import pytest
import torch

from oracle import siso_oracle as O

F64 = torch.float64


def test_oracle_nucleus_known_answers():
    # probabilities 4/9, 2/9, 2/9, 1/9; descending order with ties by higher index: 0, 2, 1, 3
    lg = torch.log(torch.tensor([[4.0, 2.0, 2.0, 1.0]], dtype=F64))
    no = torch.zeros_like(lg, dtype=torch.bool)
    p = O.nucleus_probs(lg, no, 1.0, 0.7, 1.0)  # mass before: 0, 4/9, 6/9, 8/9
    assert torch.allclose(p, torch.tensor([[0.5, 0.25, 0.25, 0.0]], dtype=F64))
    p = O.nucleus_probs(lg, no, 1.0, 0.5, 1.0)  # the tie at 2/9 splits: index 2 stays, 1 goes
    assert torch.allclose(p, torch.tensor([[4 / 6, 0.0, 2 / 6, 0.0]], dtype=F64))
    p = O.nucleus_probs(lg, no, 1.0, 0.01, 1.0)  # the top-1 is always kept
    assert torch.allclose(p, torch.tensor([[1.0, 0.0, 0.0, 0.0]], dtype=F64))
    # sign-aware penalty: a positive logit is divided, a negative one multiplied
    lg = torch.tensor([[2.0, -1.0, 0.5]], dtype=F64)
    seen = torch.tensor([[True, True, False]])
    p = O.nucleus_probs(lg, seen, 2.0, 1.5, 2.0)
    want = torch.softmax(torch.tensor([[1.0, -2.0, 0.5]], dtype=F64) / 2.0, -1)
    assert torch.allclose(p, want)


def _seen_mask(r, v, frac, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.rand(r, v, generator=g) < frac


@pytest.mark.gpu
@pytest.mark.parametrize("vocab", [256, 50_000, 128_256])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("top_p", [0.0, 0.5, 0.95, 1.0])
def test_filtered_distribution_matches_oracle(vocab, dtype, top_p):
    from mamba3_b200.sampling import TokenSampler

    rows = 3
    g = torch.Generator().manual_seed(vocab)
    logits = (torch.randn(rows, vocab, generator=g) * 3.0).to(dtype)  # bf16: many exact ties
    seen = _seen_mask(rows, vocab, 0.01, 5)
    smp = TokenSampler(rows, vocab, "cuda", temperature=0.9, top_p=top_p, rep_penalty=1.15)
    smp.seen.copy_(seen.to(torch.int32))
    got = smp.filtered_probs(logits.cuda()).double().cpu()
    # the oracle sees the same fp32 values the kernel computes with
    lf = logits.float()
    lf = torch.where(seen, torch.where(lf > 0, lf / 1.15, lf * 1.15), lf) / 0.9
    ref = O.nucleus_probs(lf.double(), torch.zeros_like(seen), 1.0, top_p, 1.0)
    if top_p == 0.0:  # no mass before the top-1 is < 0: the kernel keeps the top-1 alone
        ref = O.nucleus_probs(lf.double(), torch.zeros_like(seen), 1.0, 1e-12, 1.0)
    # the kernel's fixed-point mass (2^-32 of the top entry) drops entries below ~1e-10,
    # which a float32 cumsum drops as well; nothing larger may differ
    mism = (got > 0) != (ref > 0)
    assert not mism.any() or max(float(got[mism].max()), float(ref[mism].max())) < 1e-9, "kept sets differ"
    assert torch.allclose(got, ref, rtol=2e-5, atol=1e-9)


@pytest.mark.gpu
def test_large_vocabulary_uses_the_workspace():
    """Above 184,320 entries a row's eighth no longer fits in shared memory and the kernel
    keeps its (key, mass) pairs in the workspace instead."""
    test_filtered_distribution_matches_oracle(200_003, torch.float32, 0.9)


@pytest.mark.gpu
def test_draws_follow_the_distribution():
    from mamba3_b200.sampling import TokenSampler

    rows, vocab, draws = 4096, 12, 16
    g = torch.Generator().manual_seed(1)
    logits = torch.randn(1, vocab, generator=g).expand(rows, vocab).contiguous().cuda()
    smp = TokenSampler(rows, vocab, "cuda", seed=123, temperature=1.0, top_p=0.9, rep_penalty=1.0,
                       history_cap=draws)
    p = smp.filtered_probs(logits)[0].double().cpu()
    for _ in range(draws):  # every draw: a new counter value, the same logits (no penalty)
        smp.pick(logits)
    h = smp.history.cpu().reshape(-1)
    counts = torch.bincount(h, minlength=vocab).double()
    n = counts.sum()
    assert torch.all(counts[p == 0] == 0)
    exp = p * n
    chi2 = float((((counts - exp) ** 2) / exp.clamp_min(1e-12))[p > 0].sum())
    dof = int((p > 0).sum()) - 1
    assert chi2 < dof + 6 * math.sqrt(2 * dof), (chi2, dof)


@pytest.mark.gpu
def test_window_stop_and_history_follow_the_reference_loop():
    from mamba3_b200.sampling import TokenSampler

    vocab, window, steps = 40, 5, 60
    prompt = [3, 7, 7, 11, 2, 9, 9]
    g = torch.Generator().manual_seed(2)
    logit_seq = torch.randn(steps, 1, vocab, generator=g).cuda()
    smp = TokenSampler(1, vocab, "cuda", seed=9, temperature=0.8, top_p=0.95, rep_penalty=1.3, rep_window=window,
                       stop_ids=[vocab - 1], history_cap=steps)
    smp.reset([prompt])
    # host replay of train.py:548-579 from the drawn ids
    seen = [False] * vocab
    win = prompt[-window:]
    for t in win:
        seen[t] = True
    for i in range(steps):
        smp.pick(logit_seq[i])
        torch.cuda.synchronize()
        if int(smp.done[0]):
            break
        nxt = int(smp.token[0])
        win.append(nxt)
        if len(win) > window:
            dropped = win.pop(0)
            if dropped not in win:
                seen[dropped] = False
        seen[nxt] = True
        assert [c > 0 for c in smp.seen[0].tolist()] == seen, f"step {i}"
    n = int(smp.counter[0])
    assert smp.history[0, :n].tolist()[-1] == int(smp.token[0])
    # a row whose only finite logit is the stop id stops at once and then stays put
    smp2 = TokenSampler(1, vocab, "cuda", stop_ids=[5], history_cap=4)
    smp2.reset([[1]])
    lg = torch.full((1, vocab), -math.inf, device="cuda")
    lg[0, 5] = 0.0
    smp2.pick(lg)
    smp2.pick(torch.zeros(1, vocab, device="cuda"))
    assert int(smp2.done[0]) == 1 and int(smp2.counter[0]) == 1 and smp2.history[0, 0].item() == 5


@pytest.mark.gpu
def test_generate_graph_loop_equals_eager_loop():
    from mamba3_b200 import train as TR
    from tests.test_model_gpu import _small_lm

    cfg, params = _small_lm()
    prompt = list(range(70))
    seen = []
    a = TR.generate(params, cfg, 11, prompt, n_tokens=40, device_loop=True, sync_every=7, on_token=seen.append)
    b = TR.generate(params, cfg, 11, prompt, n_tokens=40, device_loop=False)
    assert a == b and len(a) == 110 and seen == a[70:]
    stop = a[75]  # the 6th generated id: generation ends there, stop id included
    c = TR.generate(params, cfg, 11, prompt, n_tokens=40, stop_ids=[stop], sync_every=4)
    first = a[70:].index(stop)
    assert c == a[:70 + first + 1]
