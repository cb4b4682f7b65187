"""Persistent per-row sampling parameters on the device.

Extends the reference's ``Batch._fill_sampling`` (``src/data/batch.py:149-175``):
the same structure-of-arrays on the device (``temperatures``, ``top_ps``,
``top_ks``, ``min_ps``), the same mapping of ``None``/<=0 top-k to the full
vocabulary (``:154-157``) and a signature cache that skips the upload when
nothing changed (``:160-162``); plus the repetition-penalty arrays and a
fixed-width token-history buffer the B200 sampler reads.  The parameters
live in one device block with a pinned host mirror, so a change is one
host-to-device copy.  The host flags ``all_greedy``/``use_top_p`` are computed as in
``:169-174``.
"""
from __future__ import annotations

import torch


class _Block:
    """Device tensors carved from one contiguous device buffer, with a pinned
    host mirror of the same layout: a whole block goes up in one copy.  An
    event recorded after each copy is waited on before the host mirror is
    written again, so a copy still in flight never sees new contents."""

    def __init__(self, fields, device: torch.device):
        self.device = device
        def size(n, dt):   # each field starts 16-byte aligned
            return (n * torch.empty((), dtype=dt).element_size() + 15) // 16 * 16
        nbytes = sum(size(n, dt) for _, n, dt in fields)
        self.dev = torch.zeros(max(nbytes, 16), dtype=torch.uint8, device=device)
        pinned = device.type == "cuda"
        self.host = torch.zeros(self.dev.numel(), dtype=torch.uint8, pin_memory=pinned)
        self.views, self.host_views = {}, {}
        off = 0
        for name, n, dt in fields:
            nb = n * torch.empty((), dtype=dt).element_size()
            self.views[name] = self.dev[off:off + nb].view(dt)
            self.host_views[name] = self.host[off:off + nb].view(dt).numpy()
            off += size(n, dt)
        self.used = off
        self._event = torch.cuda.Event() if pinned else None

    def host_ready(self) -> None:
        if self._event is not None:
            self._event.synchronize()

    def upload(self, nbytes: int | None = None) -> None:
        n = self.used if nbytes is None else nbytes
        self.dev[:n].copy_(self.host[:n], non_blocking=True)
        if self._event is not None:
            self._event.record()


class SamplingBatch:
    def __init__(self, *, max_bs: int, vocab_size: int, device: torch.device,
                 history_width: int = 0) -> None:
        self.max_bs = max_bs
        self.vocab_size = vocab_size
        self.device = torch.device(device)
        self.history_width = history_width
        W = max(history_width, 1)
        # per-row parameters in one block (one host-to-device copy per change)
        self._params = _Block([("temperatures", max_bs, torch.float32), ("top_ps", max_bs, torch.float32),
                               ("top_ks", max_bs, torch.int32), ("min_ps", max_bs, torch.float32),
                               ("rep_penalties", max_bs, torch.float32), ("seeds", max_bs, torch.int64)],
                              self.device)
        self._hist = _Block([("history_lens", max_bs, torch.int32), ("history", max_bs * W, torch.int32)],
                            self.device)
        v = self._params.views
        self.temperatures, self.top_ps, self.top_ks = v["temperatures"], v["top_ps"], v["top_ks"]
        self.min_ps, self.rep_penalties, self.seeds = v["min_ps"], v["rep_penalties"], v["seeds"]
        self.default_seed = 0
        self.rep_penalties.fill_(1.0)
        self.history_lens = self._hist.views["history_lens"]
        self.history = self._hist.views["history"].view(max_bs, W)
        self.all_greedy = True
        self.any_greedy = False
        self.use_top_k = False
        self.use_top_p = False
        self.use_min_p = False
        self.use_penalty = False
        self.use_seeds = False
        self.max_top_k = 0
        self._signature = None
        self._history_signature = None

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
        seeds = [getattr(s, "seed", None) for s in seqs]
        use_seeds = any(x is not None for x in seeds)
        # rows without a seed of their own keep the sampler's seed
        seeds = [self.default_seed if x is None else int(x) for x in seeds]
        signature = tuple(zip(temps, top_ps, top_ks, min_ps, rps, seeds))
        if signature != self._signature:
            blk = self._params
            blk.host_ready()
            hv = blk.host_views
            hv["temperatures"][:bs] = temps
            hv["top_ps"][:bs] = top_ps
            hv["top_ks"][:bs] = top_ks
            hv["min_ps"][:bs] = min_ps
            hv["rep_penalties"][:bs] = rps
            hv["seeds"][:bs] = [x - (1 << 64) if x >= (1 << 63) else x for x in seeds]
            blk.upload()
            self.all_greedy = all(t <= 1e-5 for t in temps)
            self.any_greedy = any(t <= 1e-5 for t in temps)
            self.use_top_k = any(k < vocab for k in top_ks)
            self.use_top_p = any(p < 1.0 for p in top_ps)
            self.use_min_p = any(m > 0.0 for m in min_ps)
            self.use_penalty = any(r != 1.0 for r in rps)
            self.use_seeds = use_seeds
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
        blk = self._hist
        blk.host_ready()
        lens = blk.host_views["history_lens"]
        rows = blk.host_views["history"].reshape(self.max_bs, W)
        for r, s in enumerate(seqs):
            ids = list(getattr(s, "token_ids", ()))[-W:]
            lens[r] = len(ids)
            rows[r, :len(ids)] = ids
        blk.upload()
        self._history_signature = sig

    def sampler_kwargs(self, bs: int) -> dict:
        """Keyword arguments for ``QESampler.forward`` for rows ``0..bs-1``."""
        kw = {"top_ks": self.top_ks[:bs]}
        if self.use_min_p:
            kw["min_ps"] = self.min_ps[:bs]
        if self.use_seeds:
            kw["seeds"] = self.seeds[:bs]
        if self.use_penalty and self.history_width > 0:
            kw.update(rep_penalties=self.rep_penalties[:bs], history=self.history[:bs],
                      history_lens=self.history_lens[:bs])
        return kw
