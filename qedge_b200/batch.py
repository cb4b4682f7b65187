"""Persistent per-row sampling parameters on the device.

Extends the reference's ``Batch._fill_sampling`` (``src/data/batch.py:149-175``):
the same structure-of-arrays on the device (``temperatures``, ``top_ps``,
``top_ks``, ``min_ps``), the same mapping of ``None``/<=0 top-k to the full
vocabulary (``:154-157``), reusable pinned host staging and a signature
cache that skips the upload when nothing changed (``:160-162``); plus the
repetition-penalty arrays and a fixed-width token-history buffer the B200
sampler reads.  The host flags ``all_greedy``/``use_top_p`` are computed as in
``:169-174``.
"""
from __future__ import annotations

import torch


class SamplingBatch:
    def __init__(self, *, max_bs: int, vocab_size: int, device: torch.device,
                 history_width: int = 0) -> None:
        self.max_bs = max_bs
        self.vocab_size = vocab_size
        self.device = torch.device(device)
        self.history_width = history_width
        d = self.device
        self.temperatures = torch.zeros(max_bs, dtype=torch.float32, device=d)
        self.top_ps = torch.zeros(max_bs, dtype=torch.float32, device=d)
        self.top_ks = torch.zeros(max_bs, dtype=torch.int32, device=d)
        self.min_ps = torch.zeros(max_bs, dtype=torch.float32, device=d)
        self.rep_penalties = torch.ones(max_bs, dtype=torch.float32, device=d)
        self.history = torch.zeros(max_bs, max(history_width, 1), dtype=torch.int32, device=d)
        self.history_lens = torch.zeros(max_bs, dtype=torch.int32, device=d)
        self.all_greedy = True
        self.any_greedy = False
        self.use_top_k = False
        self.use_top_p = False
        self.use_min_p = False
        self.use_penalty = False
        self.max_top_k = 0
        self._staging: dict[tuple[int, torch.dtype], torch.Tensor] = {}
        self._signature = None
        self._history_signature = None

    def _pinned(self) -> bool:
        return self.device.type == "cuda"

    def _cp(self, dst: torch.Tensor, data: list, dtype: torch.dtype) -> None:
        storage = dst.untyped_storage()
        key = (storage.data_ptr(), dtype)
        capacity = storage.nbytes() // torch.empty((), dtype=dtype).element_size()
        cpu = self._staging.get(key)
        if cpu is None or cpu.numel() < capacity:
            cpu = torch.empty(capacity, dtype=dtype, pin_memory=self._pinned())
            self._staging[key] = cpu
        cpu.numpy()[:len(data)] = data
        dst.copy_(cpu[:len(data)].view_as(dst), non_blocking=True)

    def fill(self, seqs) -> None:
        """Pack the sampling fields of ``seqs`` (objects with ``temperature``,
        ``top_p``, ``top_k``, ``min_p``; optionally ``repetition_penalty`` and
        ``token_ids``) into rows ``0..len(seqs)-1``."""
        bs = len(seqs)
        if bs > self.max_bs:
            raise ValueError(f"{bs} sequences exceed max_bs={self.max_bs}")
        vocab = self.vocab_size
        temps = [float(s.temperature) for s in seqs]
        top_ps = [1.0 if s.top_p is None else float(s.top_p) for s in seqs]
        top_ks = [vocab if (s.top_k is None or s.top_k <= 0) else min(int(s.top_k), vocab) for s in seqs]
        min_ps = [0.0 if s.min_p is None else float(s.min_p) for s in seqs]
        rps = [float(getattr(s, "repetition_penalty", 1.0) or 1.0) for s in seqs]
        signature = tuple(zip(temps, top_ps, top_ks, min_ps, rps))
        if signature != self._signature:
            self._cp(self.temperatures[:bs], temps, torch.float32)
            self._cp(self.top_ps[:bs], top_ps, torch.float32)
            self._cp(self.top_ks[:bs], top_ks, torch.int32)
            self._cp(self.min_ps[:bs], min_ps, torch.float32)
            self._cp(self.rep_penalties[:bs], rps, torch.float32)
            self.all_greedy = all(t <= 1e-5 for t in temps)
            self.any_greedy = any(t <= 1e-5 for t in temps)
            self.use_top_k = any(k < vocab for k in top_ks)
            self.use_top_p = any(p < 1.0 for p in top_ps)
            self.use_min_p = any(m > 0.0 for m in min_ps)
            self.use_penalty = any(r != 1.0 for r in rps)
            self.max_top_k = max(top_ks) if self.use_top_k else 0
            self._signature = signature
        if self.use_penalty and self.history_width > 0:
            self._fill_history(seqs)

    def _fill_history(self, seqs) -> None:
        """Copy the last ``history_width`` token ids of each sequence (the
        penalty is applied over the set of ids, so order is irrelevant)."""
        W = self.history_width
        sig = tuple((id(s), len(getattr(s, "token_ids", ()))) for s in seqs)
        if sig == self._history_signature:
            return
        flat, lens = [], []
        for s in seqs:
            ids = list(getattr(s, "token_ids", ()))[-W:]
            lens.append(len(ids))
            flat.extend(ids + [0] * (W - len(ids)))
        self._cp(self.history[:len(seqs)].reshape(-1), flat, torch.int32)
        self._cp(self.history_lens[:len(seqs)], lens, torch.int32)
        self._history_signature = sig

    def sampler_kwargs(self, bs: int) -> dict:
        """Keyword arguments for ``QESampler.forward`` for rows ``0..bs-1``."""
        kw = {"top_ks": self.top_ks[:bs]}
        if self.use_penalty and self.history_width > 0:
            kw.update(rep_penalties=self.rep_penalties[:bs], history=self.history[:bs],
                      history_lens=self.history_lens[:bs])
        return kw
