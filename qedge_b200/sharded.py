"""Vocab-sharded sampling: the lm_head output split over GPUs by vocabulary.

When QEdge's lm_head is tensor-parallel, each GPU holds ``logits[:, v0:v1]``
for its block of the vocabulary instead of the full ``[B, V]`` tensor that
``BatchSampler.forward`` (``src/compute/sampler.py:25-41``) samples.
``ShardedSampler`` samples such logits without gathering them: every GPU
reduces its shard to fixed-size per-(row, slice) records (max, softmax sum,
exact local race candidates, small top-k lists), the records are all-gathered
(NCCL over NVLink), and every GPU merges them identically.  Rows whose top-p
test needs the mass ahead of a candidate take one more, smaller all-gather.
Token ids equal the single-GPU ``QESampler`` ids under the same noise.

Shard ``s`` of ``n`` (``n`` divides 16) holds the canonical vocab slices
``[16s/n, 16(s+1)/n)``: ids ``shard_bounds(V, n, s)``.
"""
from __future__ import annotations

import ctypes
from typing import Callable

import torch

from . import _native as N
from .sampler import QESampler, _DTYPES, _ptr, _vec

NSLICE = 16


def slice_start(g: int, V: int) -> int:
    return V if g >= NSLICE else ((g * V) // (NSLICE * 8)) * 8


def shard_bounds(V: int, nshards: int, shard: int) -> tuple[int, int]:
    """Ids [start, end) of shard ``shard`` of ``nshards``."""
    if NSLICE % nshards:
        raise ValueError("nshards must divide 16")
    per = NSLICE // nshards
    return slice_start(shard * per, V), slice_start((shard + 1) * per, V)


def _torch_allgather(group=None) -> Callable[[torch.Tensor], torch.Tensor]:
    import torch.distributed as dist

    def gather(t: torch.Tensor) -> torch.Tensor:
        out = torch.empty(dist.get_world_size(group) * t.numel(), dtype=t.dtype, device=t.device)
        dist.all_gather_into_tensor(out, t.contiguous(), group=group)
        return out
    return gather


class _Calls:
    """The four C-ABI calls for one shard's logits and one set of row
    parameters (argument conversion as in ``QESampler.forward``)."""

    def __init__(self, lib, logits, vocab, temperatures, top_ps, *, all_greedy, use_top_p, top_ks,
                 rep_penalties, history, history_lens, seed, step, step_tensor, noise, row_offset,
                 out, out_status):
        B = logits.shape[0]
        dev = logits.device
        if logits.dtype not in _DTYPES:
            raise TypeError(f"unsupported logits dtype {logits.dtype}")
        if logits.stride(1) != 1:
            logits = logits.contiguous()
        self.keep = [logits]
        temps = _vec(temperatures, torch.float32, B, dev, "temperatures")
        tps = _vec(top_ps, torch.float32, B, dev, "top_ps")
        tks = _vec(top_ks, torch.int32, B, dev, "top_ks")
        rps = _vec(rep_penalties, torch.float32, B, dev, "rep_penalties")
        hist = hlen = None
        if history is not None and rps is not None:
            hist = history.to(device=dev, dtype=torch.int32).contiguous()
            hlen = _vec(history_lens, torch.int32, B, dev, "history_lens")
        if noise is not None:
            noise = noise.to(device=dev, dtype=torch.float32)
            if noise.stride(1) != 1:
                noise = noise.contiguous()
        self.keep += [temps, tps, tks, rps, hist, hlen, noise]
        a = N.QeSampleArgs()
        a.struct_size = ctypes.sizeof(N.QeSampleArgs)
        a.dtype = _DTYPES[logits.dtype]
        a.batch, a.vocab = B, vocab
        a.ld = logits.stride(0) if B > 1 else logits.shape[1]
        a.logits = _ptr(logits)
        a.temperatures = _ptr(temps)
        a.top_ps = _ptr(tps)
        a.top_ks = _ptr(tks)
        a.rep_penalties = _ptr(rps)
        a.history = _ptr(hist)
        a.history_lens = _ptr(hlen)
        a.history_ld = hist.stride(0) if hist is not None else 0
        a.noise = _ptr(noise)
        a.noise_ld = (noise.stride(0) if noise.shape[0] > 1 else noise.shape[1]) if noise is not None else 0
        a.seed = int(seed) & ((1 << 64) - 1)
        a.step = int(step or 0) & ((1 << 64) - 1)
        a.step_ptr = _ptr(step_tensor)
        a.row_offset = int(row_offset)
        a.flags = (N.QE_FLAG_ALL_GREEDY if all_greedy else 0) | (N.QE_FLAG_USE_TOP_P if use_top_p else 0)
        a.out_ids = _ptr(out)
        a.out_status = _ptr(out_status)
        self.a, self.lib = a, lib
        self.stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)

    def summarize(self, shard, nshards, records):
        N.check(self.lib.qe_shard_summarize(ctypes.byref(self.a), shard, nshards, _ptr(records), self.stream), self.lib)

    def merge(self, nshards, all_records, tests):
        N.check(self.lib.qe_shard_merge(ctypes.byref(self.a), nshards, _ptr(all_records), _ptr(tests), self.stream),
                self.lib)

    def test(self, shard, nshards, tests, partials):
        N.check(self.lib.qe_shard_test(ctypes.byref(self.a), shard, nshards, _ptr(tests), _ptr(partials),
                                       self.stream), self.lib)

    def decide(self, nshards, tests, all_partials):
        N.check(self.lib.qe_shard_decide(ctypes.byref(self.a), nshards, _ptr(tests), _ptr(all_partials),
                                         self.stream), self.lib)


class ShardedSampler:
    """Sampler for one GPU's vocab shard (``BatchSampler.forward`` semantics).

    ``allgather(t)`` concatenates a 1-D uint8 tensor over the shards in shard
    order; by default it is ``torch.distributed.all_gather_into_tensor`` on
    ``group`` (NCCL), with this process's rank as the shard index.
    """

    def __init__(self, seed: int = 0, *, nshards: int | None = None, shard: int | None = None,
                 group=None, allgather: Callable[[torch.Tensor], torch.Tensor] | None = None):
        self.lib = N.load()
        if nshards is None or shard is None:
            import torch.distributed as dist
            nshards = dist.get_world_size(group) if nshards is None else nshards
            shard = dist.get_rank(group) if shard is None else shard
        if NSLICE % nshards or not 0 <= shard < nshards:
            raise ValueError("nshards must divide 16 and 0 <= shard < nshards")
        self.nshards, self.shard = nshards, shard
        self.allgather = allgather or _torch_allgather(group)
        self.seed = int(seed) & ((1 << 64) - 1)
        self.step = 0
        self.rec_b = int(self.lib.qe_shard_record_bytes())
        self.test_b = int(self.lib.qe_shard_test_bytes())
        self.part_b = int(self.lib.qe_shard_partial_bytes())
        self.fallback_rows = 0

    @torch.no_grad()
    def forward(self, logits: torch.Tensor, vocab: int, temperatures, top_ps=None, *, all_greedy=False,
                use_top_p=False, top_ks=None, rep_penalties=None, history=None, history_lens=None,
                seed=None, step=None, step_tensor=None, noise=None, row_offset=0, out_status=None):
        """``logits``: this shard's ``[B, end - start]`` columns; ``vocab``:
        the full V; ``noise`` (parity mode): this shard's columns of the
        Exp(1) tensor.  Returns int64 ids ``[B]`` (global vocabulary ids)."""
        B = logits.shape[0]
        dev = logits.device
        n, s = self.nshards, self.shard
        v0, v1 = shard_bounds(vocab, n, s)
        if logits.shape[1] != v1 - v0:
            raise ValueError(f"shard {s} of {n} holds {v1 - v0} ids, logits have {logits.shape[1]}")
        if step is None and step_tensor is None:
            step = self.step
            self.step += 1
        out = torch.empty(B, dtype=torch.int64, device=dev)
        status = out_status if out_status is not None else torch.empty(B, dtype=torch.int32, device=dev)
        if B == 0:
            return out
        kw = dict(all_greedy=all_greedy, use_top_p=use_top_p, top_ks=top_ks, rep_penalties=rep_penalties,
                  history=history, history_lens=history_lens, seed=self.seed if seed is None else seed,
                  step=step, step_tensor=step_tensor, noise=noise, row_offset=row_offset)
        calls = _Calls(self.lib, logits, vocab, temperatures, top_ps, out=out, out_status=status, **kw)
        nsl = NSLICE // n
        rec = torch.empty(B * nsl * self.rec_b, dtype=torch.uint8, device=dev)
        calls.summarize(s, n, rec)
        all_rec = self.allgather(rec)
        tests = torch.empty(B * self.test_b, dtype=torch.uint8, device=dev)
        calls.merge(n, all_rec, tests)
        part = torch.empty(B * nsl * self.part_b, dtype=torch.uint8, device=dev)
        calls.test(s, n, tests, part)
        all_part = self.allgather(part)
        calls.decide(n, tests, all_part)
        # rows whose candidates all fell outside the kept set: gather the
        # full rows and finish them with the single-GPU sampler (identical
        # on every shard, so every shard takes the same collective steps)
        slow = torch.nonzero((status & N.QE_ROW_SLOW) != 0).flatten().tolist()
        if slow:
            self.fallback_rows += len(slow)
            idx = torch.tensor(slow, device=dev)
            full = self._gather_rows(logits.index_select(0, idx), vocab)
            nz = None
            if noise is not None:
                nz = self._gather_rows(noise.to(dev).index_select(0, idx), vocab)
            single = QESampler(self.seed if seed is None else seed)
            for j, r in enumerate(slow):
                sel = slice(r, r + 1)
                pick = lambda t: None if t is None else _vec(t, t.dtype, B, dev, "param")[sel]  # noqa: E731
                ids = single(full[j:j + 1], _vec(temperatures, torch.float32, B, dev, "t")[sel],
                             None if top_ps is None else _vec(top_ps, torch.float32, B, dev, "p")[sel],
                             all_greedy=all_greedy, use_top_p=use_top_p, top_ks=pick(top_ks),
                             rep_penalties=pick(rep_penalties),
                             history=None if history is None else history[sel],
                             history_lens=pick(history_lens), step=step, step_tensor=step_tensor,
                             noise=None if nz is None else nz[j:j + 1], row_offset=row_offset + r)
                out[r] = ids[0]
        return out

    __call__ = forward

    def _gather_rows(self, rows: torch.Tensor, vocab: int) -> torch.Tensor:
        """All-gather a [R, width] block of every shard's columns into [R, V]."""
        R = rows.shape[0]
        n = self.nshards
        widths = [shard_bounds(vocab, n, i)[1] - shard_bounds(vocab, n, i)[0] for i in range(n)]
        wmax = max(widths)
        pad = torch.zeros(R, wmax, dtype=rows.dtype, device=rows.device)
        pad[:, :rows.shape[1]] = rows
        flat = self.allgather(pad.contiguous().view(torch.uint8).flatten())
        blocks = flat.view(n, R, wmax * rows.element_size()).view(rows.dtype).view(n, R, wmax)
        return torch.cat([blocks[i, :, :widths[i]] for i in range(n)], dim=1)


def emulate(logits: torch.Tensor, nshards: int, temperatures, top_ps=None, *, seed: int = 0, **kw):
    """Run the sharded protocol for all ``nshards`` shards of a full
    ``[B, V]`` tensor inside one process (the all-gathers become
    concatenations).  Returns (ids, status); rows still marked QE_ROW_SLOW
    hold -1.  Used to check the sharded kernels on one GPU."""
    B, V = logits.shape
    samplers = []
    for s in range(nshards):
        v0, v1 = shard_bounds(V, nshards, s)
        samplers.append((ShardedSampler(seed, nshards=nshards, shard=s, allgather=lambda t: t), v0, v1))
    lib = samplers[0][0].lib
    rec_b, test_b, part_b = samplers[0][0].rec_b, samplers[0][0].test_b, samplers[0][0].part_b
    nsl = NSLICE // nshards
    dev = logits.device
    out = torch.empty(B, dtype=torch.int64, device=dev)
    status = torch.empty(B, dtype=torch.int32, device=dev)
    noise = kw.pop("noise", None)
    step = kw.pop("step", 0)
    step_tensor = kw.pop("step_tensor", None)
    calls = []
    for s, (_, v0, v1) in enumerate(samplers):
        calls.append(_Calls(lib, logits[:, v0:v1], V, temperatures, top_ps, out=out, out_status=status, seed=seed,
                            step=step, step_tensor=step_tensor,
                            noise=None if noise is None else noise[:, v0:v1],
                            **{k: kw.get(k) for k in ("all_greedy", "use_top_p", "top_ks", "rep_penalties",
                                                       "history", "history_lens")},
                            row_offset=kw.get("row_offset", 0)))
    recs = []
    for s in range(nshards):
        r = torch.empty(B * nsl * rec_b, dtype=torch.uint8, device=dev)
        calls[s].summarize(s, nshards, r)
        recs.append(r)
    all_rec = torch.cat(recs)
    tests = torch.empty(B * test_b, dtype=torch.uint8, device=dev)
    calls[0].merge(nshards, all_rec, tests)
    parts = []
    for s in range(nshards):
        p = torch.empty(B * nsl * part_b, dtype=torch.uint8, device=dev)
        calls[s].test(s, nshards, tests, p)
        parts.append(p)
    calls[0].decide(nshards, tests, torch.cat(parts))
    return out, status
