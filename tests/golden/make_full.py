"""Generate ``full_configs.json``: oracle results for the five benchmark
configurations at their full sizes under shared Exp(1) noise.

The GPU parity tests (``tests/test_full_configs.py``) regenerate the same
seeded logits and noise on the GPU box and compare every row of the kernel
with these results, so the box needs no CPU oracle run at full size.  Per
row the fixture holds the oracle's token id, the size of its kept set, the
distance to ``top_p`` of the exclusive masses on either side of the top-p
boundary (how close the row is to a different kept-set decision), and the
float64 softmax normaliser ``sum_j exp((x_j - max x) / T)`` of the
penalised logits.

The oracle (``oracle/sampler_oracle.py``) is itself pinned against the
reference sampler's own outputs in ``golden.json``.

Usage: python tests/golden/make_full.py   (a few minutes on 8 cores)
"""
from __future__ import annotations

import json
import multiprocessing as mp
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle import sampler_oracle as O  # noqa: E402
from qedge_b200 import workloads as W  # noqa: E402

OUT = Path(__file__).resolve().parent / "full_configs.json"
NOISE_SEED = {1: 501, 2: 502, 3: 503, 4: 504, 5: 505}

_W = None
_N = None


def _row(b: int):
    w, noise = _W, _N
    x = w.logits_f32()[b]
    h = None
    if w.history is not None:
        h = w.history[b, :int(w.history_lens[b])]
    x = O.penalise(x, h, float(w.rep_penalties[b]))
    T = float(w.temperatures[b])
    res = O.sample_row(x, T, float(w.top_ps[b]), int(w.top_ks[b]), noise[b], use_top_p=w.use_top_p,
                       all_greedy=w.all_greedy)
    norm = float("nan")
    margin = float("inf")
    if T > 1e-5 and not res.fallback:
        y = (x / np.float32(T)).astype(np.float32).astype(np.float64)
        norm = float(np.exp(y - y.max()).sum())
        if w.use_top_p and w.top_ps[b] < 1.0:
            p = O.softmax_f32((x / np.float32(T)).astype(np.float32))
            vals = p[np.argsort(-p, kind="stable")]
            excl = (np.cumsum(vals.astype(np.float64)).astype(np.float32) - vals).astype(np.float64)
            tp = float(np.float32(w.top_ps[b]))
            n_p = int(np.argmax(excl > tp)) if np.any(excl > tp) else len(excl)
            lo = tp - excl[n_p - 1] if n_p > 0 else float("inf")
            hi = excl[n_p] - tp if n_p < len(excl) else float("inf")
            margin = float(min(lo, hi))
    return res.token, res.kept, margin, norm


def generate(cfg: int) -> dict:
    global _W, _N
    _W = W.CONFIGS[cfg]()
    _N = W.exp_noise(_W.B, _W.V, NOISE_SEED[cfg])
    with mp.get_context("fork").Pool(mp.cpu_count()) as pool:
        rows = pool.map(_row, range(_W.B), chunksize=4)
    return {"workload": _W.name, "B": _W.B, "V": _W.V, "noise_seed": NOISE_SEED[cfg],
            "ids": [int(r[0]) for r in rows], "kept": [int(r[1]) for r in rows],
            "top_p_margin": [r[2] for r in rows], "norm": [r[3] for r in rows]}


def main():
    import torch
    out = {"generator": "tests/golden/make_full.py", "numpy": np.__version__, "torch": torch.__version__,
           "configs": {}}
    for cfg in (1, 2, 3, 4, 5):
        out["configs"][str(cfg)] = generate(cfg)
        print("config", cfg, "done", flush=True)
    OUT.write_text(json.dumps(out, separators=(",", ":")) + "\n")


if __name__ == "__main__":
    main()
