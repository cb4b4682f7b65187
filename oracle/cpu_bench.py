"""CPU-baseline worker: the oracle (CPU restatement of the reference
sampler, oracle/sampler_oracle.py) timed on host cores.  Test/bench
infrastructure only; used by bench.py's cpu_baseline leg."""
from __future__ import annotations

import numpy as np

from oracle import sampler_oracle as O

_cache = {}


def _row(cfg: int):
    if cfg not in _cache:
        from qedge_b200 import workloads as W
        kw = {} if cfg == 1 else {"B": 1}
        w = W.CONFIGS[cfg](**kw)
        _cache[cfg] = (w, W.exp_noise(1, w.V, 1))
    return _cache[cfg]


def warm(_i: int) -> int:
    for cfg in (1, 2, 3, 4, 5):
        pass
    return 0


def sample_rows(arg) -> int:
    cfg, _i = arg
    w, noise = _row(cfg)
    O.sample(w.logits_f32(), w.temperatures, w.top_ps, noise, top_ks=w.top_ks,
             rep_penalties=w.rep_penalties, history=w.history, history_lens=w.history_lens,
             use_top_p=w.use_top_p)
    return w.B
