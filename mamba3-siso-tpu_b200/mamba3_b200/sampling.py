"""Token sampling on the device (``train.py:454-500`` `_pick_token` and the window
bookkeeping of ``train.py:559-579``) through ``m3_sample_tokens``.

`TokenSampler` owns the per-row device state -- the window ring and its occurrence
counts (an id is "seen" while its count is > 0, which is the reference's bool mask with
its "dropped and not still in the window" rule), a draw counter that keys the random
stream, a done flag per row for stop ids, and optionally a history buffer -- so that one
sampling call needs no host round trip and can sit inside a replayed CUDA graph.
"""

from __future__ import annotations

from typing import Iterable, Optional, Sequence

import torch

from . import _capi as C
from . import _tensors as T


class TokenSampler:
    """Sampler state for ``batch`` rows over ``vocab`` logits."""

    def __init__(self, batch: int, vocab: int, device, seed: int = 0, temperature: float = 0.9,
                 top_p: float = 0.95, rep_penalty: float = 1.15, rep_window: int = 64,
                 stop_ids: Optional[Iterable[int]] = None, history_cap: int = 0):
        if rep_window < 1:
            raise ValueError(f"rep_window must be >= 1, got {rep_window}")
        if not temperature > 0 or not rep_penalty > 0:
            raise ValueError("temperature and rep_penalty must be > 0")
        dev = torch.device(device)
        i32, i64 = torch.int32, torch.int64
        self.batch, self.vocab, self.device = batch, vocab, dev
        self.seed = int(seed) & (2**64 - 1)
        self.temperature, self.top_p, self.rep_penalty, self.rep_window = temperature, top_p, rep_penalty, rep_window
        self.seen = torch.zeros(batch, vocab, dtype=i32, device=dev)
        self.window = torch.zeros(batch, rep_window, dtype=i32, device=dev)
        self.window_state = torch.zeros(batch, 2, dtype=i32, device=dev)
        self.counter = torch.zeros(batch, dtype=i64, device=dev)
        self.done = torch.zeros(batch, dtype=i32, device=dev)
        self.token = torch.zeros(batch, dtype=i64, device=dev)
        self.stop = torch.tensor(sorted(set(int(s) for s in stop_ids or ())), dtype=i64, device=dev)
        self.history = torch.zeros(batch, history_cap, dtype=i64, device=dev) if history_cap > 0 else None
        # (key, mass) per entry, for vocabularies whose rows do not fit in shared memory
        self.scratch = torch.empty(batch, vocab, 2, dtype=torch.int32, device=dev) if vocab > 184320 else None

    def reset(self, recent: Sequence[Sequence[int]]):
        """Start every row's window from its last ``rep_window`` ids (``train.py:548-551``);
        clears the counters, done flags and history."""
        if len(recent) != self.batch:
            raise ValueError(f"need {self.batch} id lists, got {len(recent)}")
        seen = torch.zeros(self.batch, self.vocab, dtype=torch.int32)
        ring = torch.zeros(self.batch, self.rep_window, dtype=torch.int32)
        st = torch.zeros(self.batch, 2, dtype=torch.int32)
        for r, ids in enumerate(recent):
            w = [int(t) for t in ids][-self.rep_window:]
            for j, t in enumerate(w):
                ring[r, j] = t
                seen[r, t] += 1
            st[r, 0] = len(w)
        self.seen.copy_(seen)
        self.window.copy_(ring)
        self.window_state.copy_(st)
        self.counter.zero_()
        self.done.zero_()
        if self.history is not None:
            self.history.zero_()

    def _args(self, logits: torch.Tensor, update: bool, probs_out: Optional[torch.Tensor] = None):
        """The call's arguments and the logits tensor they point into (a converted copy when
        the input is not f32 / bf16 with unit column stride): the caller keeps that tensor
        alive until the call is enqueued, so its memory cannot be handed out before."""
        if logits.dim() != 2 or logits.shape[0] != self.batch or logits.shape[1] < self.vocab:
            raise ValueError(f"logits must be ({self.batch}, >= {self.vocab}), got {tuple(logits.shape)}")
        if logits.dtype not in (torch.float32, torch.bfloat16) or logits.stride(1) != 1:
            logits = logits.float().contiguous()
        T.require_cuda(logits)
        a = C.M3SampleArgs()
        a.batch, a.vocab = self.batch, self.vocab
        a.logits_dtype = C.M3_DTYPE_BF16 if logits.dtype == torch.bfloat16 else C.M3_DTYPE_F32
        a.logits_ld, a.logits = logits.stride(0), T.ptr(logits)
        a.temperature, a.top_p, a.rep_penalty, a.seed = self.temperature, self.top_p, self.rep_penalty, self.seed
        a.seen_count, a.scratch, a.out_token = T.ptr(self.seen), T.ptr(self.scratch), T.ptr(self.token)
        if update:
            a.counter, a.window, a.window_state, a.rep_window = (T.ptr(self.counter), T.ptr(self.window),
                                                                 T.ptr(self.window_state), self.rep_window)
            a.done = T.ptr(self.done)
            a.stop_ids, a.n_stop = T.ptr(self.stop), self.stop.numel()
            if self.history is not None:
                a.history, a.history_cap = T.ptr(self.history), self.history.shape[1]
        if probs_out is not None:
            a.probs_out, a.probs_ld = T.ptr(probs_out), probs_out.stride(0)
        return a, logits

    def pick(self, logits: torch.Tensor) -> torch.Tensor:
        """Draw one id per row from ``(batch, vocab)`` logits and advance the window; the
        result is `token` (a device buffer, updated in place, no host sync)."""
        a, keep = self._args(logits, update=True)
        C.check(C.lib().m3_sample_tokens(a, T.stream_handle(self.device)))
        del keep
        return self.token

    def filtered_probs(self, logits: torch.Tensor) -> torch.Tensor:
        """The distribution `pick` draws from (penalty, temperature and nucleus applied),
        without drawing or touching the window."""
        out = torch.empty(self.batch, self.vocab, dtype=torch.float32, device=self.device)
        a, keep = self._args(logits, update=False, probs_out=out)
        sink = torch.empty(self.batch, dtype=torch.int64, device=self.device)
        a.out_token = T.ptr(sink)
        C.check(C.lib().m3_sample_tokens(a, T.stream_handle(self.device)))
        del keep
        return out
