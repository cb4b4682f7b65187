"""Drop-in installation of the B200 sampler into QEdge's ``ModelRunner``.

The reference constructs ``BatchSampler()`` in ``ModelRunner.__init__``
(``src/compute/model_runner.py:28``) and calls it from ``_sample_gpu``
(``:77-93``) with the per-row arrays of ``Batch`` (``src/data/batch.py:57-60``).
:func:`install` swaps both on a live runner without editing the reference:

* ``runner.sampler`` becomes a :class:`~qedge_b200.sampler.QESampler`;
* ``runner._sample_gpu`` packs the sequences' sampling fields (temperature,
  top-p, top-k, repetition penalty, token history) into a
  :class:`~qedge_b200.batch.SamplingBatch` and calls the sampler with them;
  all-greedy batches go through the same kernel (argmax rows), so the call is
  a single launch on the current stream with no host synchronisation;
* the pinned host mirror ``runner.sample_cpu`` (256 entries in the
  reference, ``:31``) is grown to ``max_num_seqs`` so batches above 256 rows
  can be read back.

The decode step counter that keys the Philox noise advances once per call.
"""
from __future__ import annotations

import types

import torch

from .batch import SamplingBatch
from .sampler import QESampler


def _sample_gpu(self, logits: list[torch.Tensor], seqs) -> torch.Tensor:
    if not logits:
        return torch.empty(0, dtype=torch.long, device=self.device)
    merged = logits[0] if len(logits) == 1 else torch.cat(logits, dim=0)
    qb: SamplingBatch = self.qe_batch
    n = len(seqs)
    qb.fill(seqs)
    ids = self.sampler(merged, qb.temperatures[:n], qb.top_ps[:n], all_greedy=qb.all_greedy,
                       use_top_p=qb.use_top_p, step=self.qe_step, **qb.sampler_kwargs(n))
    self.qe_step += 1
    return ids


def install(runner, *, seed: int = 0, history_width: int = 2048) -> QESampler:
    """Replace ``runner``'s sampler and sampling call site; returns the sampler."""
    max_bs = int(getattr(runner.batch, "max_bs", 1))
    vocab = int(runner.batch.vocab_size)
    device = torch.device(runner.device)
    runner.qe_original = (runner.sampler, runner._sample_gpu)
    runner.sampler = QESampler(seed=seed)
    runner.qe_batch = SamplingBatch(max_bs=max_bs, vocab_size=vocab, device=device,
                                    history_width=history_width)
    runner.qe_batch.default_seed = int(seed) & ((1 << 64) - 1)
    runner.qe_step = 0
    runner._sample_gpu = types.MethodType(_sample_gpu, runner)
    cpu = getattr(runner, "sample_cpu", None)
    if cpu is not None and cpu.numel() < max_bs:
        runner.sample_cpu = torch.empty(max_bs, dtype=torch.int64, pin_memory=device.type == "cuda")
    return runner.sampler


def uninstall(runner) -> None:
    """Restore the runner's original sampler and call site."""
    sampler, fn = runner.qe_original
    runner.sampler = sampler
    runner._sample_gpu = fn
    del runner.qe_original
