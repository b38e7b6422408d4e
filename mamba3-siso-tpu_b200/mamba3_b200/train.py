"""Training step and generation (``mamba3_pallas/train.py:382-624``).

`make_step` is one AdamW step of the LM; with an initialised ``torch.distributed``
process group it is data parallel: each rank runs its batch shard and the gradients are
averaged with NCCL all-reduces issued bucket by bucket as the backward produces them
(the counterpart of ``jax.lax.pmean`` inside ``shard_map``, ``train.py:427-451``).
`generate` is chunked prefill through the scan kernels, then one decode-kernel step per
token with the sampling filters applied on the device.
"""

from __future__ import annotations

from typing import Callable, Iterable, List, Optional

import numpy as np
import torch
import torch.nn.functional as F

from . import _capi as C
from . import _tensors as T
from . import model as M
from .sampling import TokenSampler


def param_list(params: M.LMParams) -> List[torch.Tensor]:
    """Flat list of the parameter tensors of an `LMParams` tree."""
    out = [params.embed]
    for b in params.blocks:
        out.append(b.norm_gain)
        out.extend(list(b.siso))
        if b.mlp is not None:
            out.extend([b.mlp_norm_gain, b.mlp.fc1, b.mlp.fc2])
    out.append(params.final_norm)
    if params.head is not None:
        out.append(params.head)
    return out


class GradBucketer:
    """All-reduce gradients in buckets as soon as every tensor of a bucket has its grad,
    so communication overlaps the rest of the backward.  Gradients are averaged over the
    process group."""

    def __init__(self, params: List[torch.Tensor], bucket_bytes: int = 16 << 20, group=None):
        import torch.distributed as dist

        self.dist, self.group = dist, group
        self.world = dist.get_world_size(group)
        self.params = [p for p in params if p.requires_grad]
        # reverse order: the last layers' grads arrive first
        self.buckets: List[List[torch.Tensor]] = []
        cur, size = [], 0
        for p in reversed(self.params):
            cur.append(p)
            size += p.numel() * p.element_size()
            if size >= bucket_bytes:
                self.buckets.append(cur)
                cur, size = [], 0
        if cur:
            self.buckets.append(cur)
        self.owner = {id(p): i for i, bk in enumerate(self.buckets) for p in bk}
        self.pending = [len(bk) for bk in self.buckets]
        self.works = []
        self.flats = [None] * len(self.buckets)
        self.hooks = [p.register_post_accumulate_grad_hook(self._hook) for p in self.params]

    def _hook(self, p):
        i = self.owner[id(p)]
        self.pending[i] -= 1
        if self.pending[i] == 0:
            flat = torch.cat([q.grad.reshape(-1) for q in self.buckets[i]])
            flat.div_(self.world)
            self.flats[i] = flat
            self.works.append((i, self.dist.all_reduce(flat, group=self.group, async_op=True)))

    def finish(self):
        for i, w in self.works:
            w.wait()
            off = 0
            for q in self.buckets[i]:
                n = q.numel()
                q.grad.copy_(self.flats[i][off:off + n].view_as(q.grad))
                off += n
        self.works.clear()
        self.pending = [len(bk) for bk in self.buckets]
        self.flats = [None] * len(self.buckets)


def make_step(cfg: M.LMConfig, params: M.LMParams, lr: float = 1e-3, betas=(0.9, 0.95), eps: float = 1e-8,
              weight_decay: float = 0.0, clip: Optional[float] = 1.0, compute_dtype=torch.bfloat16,
              distributed: Optional[bool] = None):
    """Build ``step(xs, ys) -> loss`` for fp32 master ``params`` (trained in place).

    Forward and backward run in ``compute_dtype`` (bf16: the scan kernels take bf16
    operands with fp32 state); the optimizer is torch's fused AdamW on the fp32 masters,
    after a global-norm clip like ``optax.clip_by_global_norm`` (``train.py:799-805``).
    """
    import torch.distributed as dist

    plist = param_list(params)
    for p in plist:
        p.requires_grad_(True)
    if distributed is None:
        distributed = dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1
    bucketer = GradBucketer(plist) if distributed else None
    opt = torch.optim.AdamW(plist, lr=lr, betas=betas, eps=eps, weight_decay=weight_decay,
                            fused=plist[0].is_cuda)

    def step(xs: torch.Tensor, ys: torch.Tensor) -> torch.Tensor:
        opt.zero_grad(set_to_none=False)
        logits = M.lm_forward(params, xs, cfg, compute_dtype=compute_dtype)
        loss = F.cross_entropy(logits.float().reshape(-1, logits.shape[-1]), ys.reshape(-1))
        loss.backward()
        if bucketer is not None:
            bucketer.finish()
            loss = loss.detach().clone()
            dist.all_reduce(loss)
            loss /= dist.get_world_size()
        if clip is not None:
            torch.nn.utils.clip_grad_norm_(plist, clip, foreach=True)
        opt.step()
        return loss.detach()

    step.optimizer = opt
    step.params = plist
    return step


def _seed_from(key, device) -> int:
    """A 64-bit sampler seed from an int or a torch.Generator (one draw from it)."""
    if isinstance(key, torch.Generator):
        return int(torch.randint(0, 2**62, (1,), generator=key, device=key.device))
    return int(key)


def _pick_token(logits: torch.Tensor, seen: torch.Tensor, gen, temperature: float, top_p: float,
                rep_penalty: float, vocab: int) -> torch.Tensor:
    """``train.py:454-500``: repetition penalty on ``seen`` (bool ``(vocab,)``), temperature,
    nucleus filter, one categorical draw -- the ``m3_sample_tokens`` kernel, one row."""
    smp = TokenSampler(1, vocab, logits.device, seed=_seed_from(gen, logits.device), temperature=temperature,
                       top_p=top_p, rep_penalty=rep_penalty)
    smp.seen.copy_(seen.reshape(1, -1)[:, :vocab].to(torch.int32))
    a, keep = smp._args(logits.reshape(1, -1), update=False)
    C.check(C.lib().m3_sample_tokens(a, T.stream_handle(logits.device)))
    del keep
    return smp.token[0].clone()


class _GenerateGraph:
    """One decode step fed by the sampler's token buffer, then the sampler writing the next
    token into that buffer, captured once as a CUDA graph: each replay generates a token
    with no host involvement.  The warm-up runs leave the per-layer states as they were."""

    def __init__(self, params, cfg, states, smp: TokenSampler, compute_dtype):
        dev = params.embed.device
        snap = [[t.clone() for t in st] for st in states]
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(2):
                M.lm_decode_step(params, smp.token, states, cfg, compute_dtype=compute_dtype)
        torch.cuda.current_stream(dev).wait_stream(side)
        for st, sn in zip(states, snap):
            for t, s0 in zip(st, sn):
                t.copy_(s0)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            logits, _ = M.lm_decode_step(params, smp.token, states, cfg, compute_dtype=compute_dtype)
            smp.pick(logits)

    def replay(self):
        self.graph.replay()


@torch.no_grad()
def generate(params: M.LMParams, cfg: M.LMConfig, key, prompt_ids, n_tokens: int = 192, temperature: float = 0.9,
             top_p: float = 0.95, rep_penalty: float = 1.15, rep_window: int = 64,
             stop_ids: Optional[Iterable[int]] = None, on_token: Optional[Callable[[int], None]] = None,
             compute_dtype=None, device_loop: bool = True, sync_every: int = 32, interpret=False) -> List[int]:
    """``train.py:503-582``: prefill the prompt in whole chunks, feed the remainder token
    by token through `model.lm_decode_step`, then sample ``n_tokens`` (fewer if a stop id
    is drawn; it is included, as in the reference).

    Sampling, the repetition window and the stop test run on the device
    (`sampling.TokenSampler`).  With ``device_loop`` the decode step and the sampler are
    one CUDA graph replayed per token, and the host looks at the device only every
    ``sync_every`` tokens (stop test, ``on_token`` delivery); otherwise the same kernels
    are launched eagerly per token.  ``key`` (int or torch.Generator) seeds the draw; the
    random stream differs from JAX's, so ids match the reference in distribution only."""
    ids = [int(t) for t in np.asarray(prompt_ids).reshape(-1)]
    if not ids:
        raise ValueError("prompt_ids is empty; at least one token is needed")
    dev = params.embed.device
    chunk = cfg.siso.chunk
    states = M.zero_states(cfg, 1, device=dev)
    n_whole = (len(ids) - 1) // chunk * chunk
    last = None
    if n_whole:
        logits, states = M.lm_forward(params, torch.tensor([ids[:n_whole]], device=dev), cfg, states=states,
                                      compute_dtype=compute_dtype, logits="last")
        last = logits
    for t in ids[n_whole:]:
        last, states = M.lm_decode_step(params, torch.tensor([t], device=dev), states, cfg,
                                        compute_dtype=compute_dtype)
    if n_tokens <= 0:
        return ids
    smp = TokenSampler(1, cfg.vocab_size, dev, seed=_seed_from(key, dev), temperature=temperature, top_p=top_p,
                       rep_penalty=rep_penalty, rep_window=rep_window, stop_ids=stop_ids, history_cap=n_tokens)
    smp.reset([ids])
    smp.pick(last.reshape(1, -1))
    step = None
    if device_loop and n_tokens > 1:
        step = _GenerateGraph(params, cfg, states, smp, compute_dtype).replay
    elif n_tokens > 1:
        def step():
            lg, _ = M.lm_decode_step(params, smp.token, states, cfg, compute_dtype=compute_dtype)
            smp.pick(lg)
    produced, delivered = 1, 0
    while True:
        n_drawn, done = (int(v) for v in torch.stack([smp.counter[0], smp.done[0].long()]).tolist())
        if on_token is not None and n_drawn > delivered:
            for t in smp.history[0, delivered:n_drawn].tolist():
                on_token(int(t))
            delivered = n_drawn
        if done or produced >= n_tokens:
            break
        for _ in range(min(max(1, sync_every), n_tokens - produced)):
            step()
            produced += 1
    return ids + smp.history[0, :n_drawn].tolist()


def sample(params: M.LMParams, cfg: M.LMConfig, key, prompt: bytes = b"the ", n_tokens: int = 192,
           **kw) -> bytes:
    """``train.py:585-624``: byte-level wrapper over `generate`."""
    ids = generate(params, cfg, key, list(prompt), n_tokens=n_tokens, **kw)
    return bytes(i % 256 for i in ids)
