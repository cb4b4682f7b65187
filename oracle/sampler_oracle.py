"""CPU restatement of QEdge's ``BatchSampler.forward`` (test infrastructure).

This is the checker for the CUDA sampler in ``qedge_b200``.  Only
``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` import it; the shipped sampler never calls it.

Reference algorithm (``src/compute/sampler.py:25-41``):

1. ``all_greedy`` -> ``logits.argmax(-1)`` on the raw logits (``:28-29``);
2. ``greedy = T <= 1e-5``; ``safe = where(greedy, 1, T)`` (``:30-31``);
3. ``probs = softmax(logits.float() / safe)`` in fp32 (``:32``);
4. if ``use_top_p`` (one flag for the whole batch, ``:34``): sort probs
   descending, ``remove = (cumsum - vals) > top_p``, zero the removed
   entries and draw with ``multinomial`` in sorted order (``:35-38``);
5. else draw with ``multinomial(probs, 1)`` (``:39-40``);
6. greedy rows take ``argmax`` of the logits (``:41``).

Restatement choices, each pinned by ``tests/golden`` (fixtures produced by
running the reference module itself):

* ``multinomial(w, 1)`` is replaced by the exponential race
  ``argmax_j w_j / E_j`` on a caller-supplied Exp(1) tensor ``E`` indexed by
  vocabulary id (in the top-p path the noise follows the token id, i.e.
  ``E.gather(1, idx)``).  ``torch.multinomial`` on CPU is the same race on
  noise from torch's generator.
* the sort is stable (ties keep lower ids first).
* ``cumsum`` accumulates in float64 and rounds each prefix to float32, which
  is what CPU torch does for float32 input.

Extensions the reference does not have (parity pinned by this oracle only):

* ``top_k`` (``SamplingParams.top_k``, packed by ``src/data/batch.py:154-157``
  but never applied by the reference sampler): ``remove |= rank >= k`` in the
  same stable order; the top-p mass is measured on the full distribution.
  Rows with an active ``top_k`` take the sorted path even when
  ``use_top_p`` is False.
* ``min_p`` (``SamplingParams.min_p``, packed by ``src/data/batch.py:60, 158``
  but never applied by the reference sampler): ``remove |= p < RN(min_p *
  p_max)`` in the same stable order (``p_max`` is the row's largest
  probability), so min-p, like top-k, removes a suffix of that order.  Rows
  with ``min_p > 0`` take the sorted path even when ``use_top_p`` is False.
* repetition penalty over the set of ids in the row's history, applied to
  ``logits.float()`` before temperature: ``x = x * rp if x < 0 else x / rp``
  (the rule of the Hugging Face repetition-penalty processor).  Greedy rows
  take the argmax of the penalised logits.
* a row whose probabilities are not finite (NaN/inf logits; the reference's
  ``multinomial`` raises on those) falls back to the greedy argmax.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

GREEDY_EPS = np.float32(1e-5)


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bfloat16 bit patterns (as torch does)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    r = ((u + np.uint64(0x7FFF) + ((u >> np.uint64(16)) & np.uint64(1))) >> np.uint64(16)).astype(np.uint16)
    r = np.where(nan, np.uint16(0x7FC0), r)
    return r


def f32_to_f16_bits(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, dtype=np.float32).astype(np.float16).view(np.uint16)


@dataclass
class RowResult:
    token: int
    fallback: bool          # non-finite row resolved as greedy
    kept: int               # size of the kept set (0 for greedy rows)


def _argmax_first(x: np.ndarray) -> int:
    # numpy argmax returns the first maximum and treats NaN as maximal,
    # matching torch.argmax.
    return int(np.argmax(x))


def penalise(x: np.ndarray, history, rp: float) -> np.ndarray:
    """Repetition penalty on the set of history ids (out-of-range ids are
    ignored)."""
    if history is None or rp == 1.0 or len(history) == 0:
        return x
    V = x.shape[0]
    ids = np.unique(np.asarray(history, dtype=np.int64))
    ids = ids[(ids >= 0) & (ids < V)]
    rpf = np.float32(rp)
    v = x[ids]
    x = x.copy()
    x[ids] = np.where(v < 0, (v * rpf).astype(np.float32), (v / rpf).astype(np.float32))
    return x


def softmax_f32(y: np.ndarray) -> np.ndarray:
    m = np.max(y)
    e = np.exp((y - m).astype(np.float32)).astype(np.float32)
    s = np.float32(np.sum(e, dtype=np.float32))
    return (e / s).astype(np.float32)


def sample_row(x: np.ndarray, T: float, top_p: float, top_k: int, noise: np.ndarray,
               *, use_top_p: bool, all_greedy: bool = False, min_p: float = 0.0) -> RowResult:
    """One row of the reference sampler on penalised float32 logits ``x``."""
    V = x.shape[0]
    if all_greedy or np.float32(T) <= GREEDY_EPS:
        return RowResult(_argmax_first(x), False, 0)
    y = (x / np.float32(T)).astype(np.float32)
    with np.errstate(invalid="ignore", over="ignore"):
        p = softmax_f32(y)
    if not np.all(np.isfinite(p)):
        return RowResult(_argmax_first(x), True, 0)
    k_active = 0 < top_k < V
    m_active = np.float32(min_p) > 0
    if use_top_p or k_active or m_active:
        order = np.argsort(-p, kind="stable")
        vals = p[order]
        remove = np.zeros(V, dtype=bool)
        if use_top_p:
            cs = np.cumsum(vals.astype(np.float64)).astype(np.float32)
            remove |= (cs - vals).astype(np.float32) > np.float32(top_p)
        if k_active:
            remove[top_k:] = True
        if m_active:
            remove |= vals < np.float32(np.float32(min_p) * vals[0])
        vals = np.where(remove, np.float32(0), vals)
        with np.errstate(divide="ignore", invalid="ignore"):
            r = (vals / noise[order]).astype(np.float32)
        pos = int(np.argmax(r))
        return RowResult(int(order[pos]), False, int(V - remove.sum()))
    with np.errstate(divide="ignore", invalid="ignore"):
        r = (p / noise).astype(np.float32)
    return RowResult(_argmax_first(r), False, V)


def sample(logits: np.ndarray, temperatures, top_ps, noise: np.ndarray, *,
           top_ks=None, rep_penalties=None, history=None, history_lens=None,
           all_greedy: bool = False, use_top_p: bool = False, details: bool = False,
           min_ps=None):
    """Batch restatement of ``BatchSampler.forward`` with the extensions.

    ``logits`` is float32 ``[B, V]`` (convert bf16/fp16 inputs first, exactly
    as ``logits.float()`` does).  ``noise`` is the Exp(1) tensor ``[B, V]``.
    Returns int64 token ids ``[B]`` (and per-row details if asked).
    """
    logits = np.asarray(logits, dtype=np.float32)
    B, V = logits.shape
    temps = np.asarray(temperatures, dtype=np.float32).reshape(B)
    tps = np.ones(B, np.float32) if top_ps is None else np.asarray(top_ps, dtype=np.float32).reshape(B)
    tks = np.zeros(B, np.int64) if top_ks is None else np.asarray(top_ks, dtype=np.int64).reshape(B)
    rps = np.ones(B, np.float32) if rep_penalties is None else np.asarray(rep_penalties, dtype=np.float32).reshape(B)
    mps = np.zeros(B, np.float32) if min_ps is None else np.asarray(min_ps, dtype=np.float32).reshape(B)
    out = np.empty(B, dtype=np.int64)
    rows = []
    for b in range(B):
        h = None
        if history is not None:
            n = history.shape[1] if history_lens is None else int(history_lens[b])
            h = history[b, :n]
        x = penalise(logits[b], h, float(rps[b]))
        res = sample_row(x, float(temps[b]), float(tps[b]), int(tks[b]), noise[b],
                         use_top_p=use_top_p, all_greedy=all_greedy, min_p=float(mps[b]))
        out[b] = res.token
        rows.append(res)
    return (out, rows) if details else out


def probs_f64(x: np.ndarray, T: float) -> np.ndarray:
    """Float64 softmax of ``x / T`` (x already penalised), used as the exact
    yardstick for the kernel's probabilities."""
    y = (x / np.float32(T)).astype(np.float32).astype(np.float64)
    m = y.max()
    e = np.exp(y - m)
    return e / e.sum()
