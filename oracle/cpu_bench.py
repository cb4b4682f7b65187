"""CPU timing of the oracle (the CPU restatement of the reference sampler,
``oracle/sampler_oracle.py``) on the host cores.  Test/bench infrastructure
only: ``bench.py`` uses it for its ``cpu_baseline`` object and for the
``--impl reference`` arm.

The workload (logits and the shared Exp(1) noise of a benchmark
configuration) is generated once, before any timing, and placed in shared
memory; one spawn pool lives across every timed step and each task samples
one row by index, so a timed step is only the oracle's own work.
"""
from __future__ import annotations

import multiprocessing as mp
import os
import time
from multiprocessing import shared_memory

import numpy as np

from oracle import sampler_oracle as O

_G = {}


def _attach(spec):
    shms, arrays = [], {}
    for name, (shm_name, shape, dtype) in spec["arrays"].items():
        shm = shared_memory.SharedMemory(name=shm_name)
        shms.append(shm)
        arrays[name] = np.ndarray(shape, dtype=dtype, buffer=shm.buf)
    _G.update(arrays)
    _G["shms"] = shms
    _G["use_top_p"] = spec["use_top_p"]


def _sample_row(b: int) -> int:
    x = _G["logits"][b]
    hist = None
    if "history" in _G:
        hist = _G["history"][b, :int(_G["history_lens"][b])]
    x = O.penalise(x, hist, float(_G["rep_penalties"][b]))
    r = O.sample_row(x, float(_G["temperatures"][b]), float(_G["top_ps"][b]), int(_G["top_ks"][b]),
                     _G["noise"][b], use_top_p=_G["use_top_p"])
    return r.token


class CpuSampler:
    """The oracle over a whole configuration batch on `procs` host processes."""

    def __init__(self, cfg: int, procs: int | None = None, noise_seed: int = 1):
        from qedge_b200 import workloads as W
        w = W.CONFIGS[cfg]()
        self.cfg, self.B, self.V, self.name = cfg, w.B, w.V, w.name
        self.procs = procs or os.cpu_count() or 1
        arrays = {"logits": w.logits_f32(), "noise": W.exp_noise(w.B, w.V, noise_seed),
                  "temperatures": w.temperatures, "top_ps": w.top_ps, "top_ks": w.top_ks,
                  "rep_penalties": w.rep_penalties}
        if w.history is not None:
            arrays["history"] = w.history
            arrays["history_lens"] = w.history_lens
        self._shms = []
        spec = {"arrays": {}, "use_top_p": w.use_top_p}
        for name, a in arrays.items():
            a = np.ascontiguousarray(a)
            shm = shared_memory.SharedMemory(create=True, size=max(1, a.nbytes))
            np.ndarray(a.shape, dtype=a.dtype, buffer=shm.buf)[...] = a
            self._shms.append(shm)
            spec["arrays"][name] = (shm.name, a.shape, a.dtype.str)
        del arrays, w
        self.pool = mp.get_context("spawn").Pool(self.procs, initializer=_attach, initargs=(spec,))
        self.pool.map(_sample_row, range(min(self.procs, self.B)))   # import and attach in every worker

    def step(self, rows: int | None = None) -> float:
        """Sample the first `rows` rows (default all B); returns seconds."""
        n = self.B if rows is None else min(rows, self.B)
        t0 = time.perf_counter()
        self.pool.map(_sample_row, range(n), chunksize=1)
        return time.perf_counter() - t0

    def close(self):
        self.pool.close()
        self.pool.join()
        for shm in self._shms:
            shm.close()
            shm.unlink()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
