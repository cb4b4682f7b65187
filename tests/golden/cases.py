"""Golden-vector case definitions shared by ``make_golden.py`` and the tests.

Every case is rebuilt from seeds (numpy PCG64), so the fixture file only
stores the reference's token ids plus SHA-256 digests of the inputs.
"""
from __future__ import annotations

import hashlib

import numpy as np

from qedge_b200 import workloads as W
from oracle import noise as N


def _small(name, B, V, seed, *, sigma=2.0, dtype="bf16", temps=None, top_ps=None,
           use_top_p=False, mode="gauss"):
    g = np.random.Generator(np.random.PCG64(seed))
    if mode == "gauss":
        x = g.standard_normal((B, V), dtype=np.float32) * np.float32(sigma)
    elif mode == "ties":          # few distinct values: heavy ties everywhere
        x = g.integers(-3, 4, size=(B, V)).astype(np.float32) * np.float32(0.5)
    elif mode == "equal":         # all-equal rows
        x = np.zeros((B, V), np.float32)
    elif mode == "neginf":        # masked vocabulary entries
        x = g.standard_normal((B, V), dtype=np.float32) * np.float32(sigma)
        mask = g.random((B, V)) < 0.3
        x[mask] = -np.inf
        x[:, 0] = np.where(np.all(mask, axis=1), 0.0, x[:, 0])
    else:
        raise ValueError(mode)
    if temps is None:
        temps = g.choice(np.array([0.0, 0.5, 1.0, 1.3], np.float32), size=B)
    if top_ps is None:
        top_ps = g.uniform(0.3, 1.0, size=B).astype(np.float32)
    bits = W.to_bf16_bits(x) if dtype == "bf16" else x.astype(np.float32)
    return W.Workload(name, bits, dtype, np.asarray(temps, np.float32),
                      np.asarray(top_ps, np.float32), np.zeros(B, np.int32),
                      np.ones(B, np.float32), None, None, use_top_p=use_top_p)


def _with_penalty_only(w: W.Workload) -> W.Workload:
    """The reference has no top-k; golden cases drop it (the penalty is a
    logits transform and is applied before the reference is called)."""
    w.top_ks = np.zeros_like(w.top_ks)
    return w


def build_cases():
    """name -> (workload, noise_spec).  noise_spec is ("exp", seed) for a
    PCG64 Exp(1) tensor or ("philox", seed, step) for the kernel's noise."""
    cases = {}
    cases["cfg1"] = (W.config1(), ("exp", 1))
    cases["cfg1_philox"] = (W.config1(), ("philox", 42, 0))
    cases["cfg2_b8"] = (_with_penalty_only(W.config2(B=8)), ("exp", 12))
    cases["cfg3_b8"] = (W.config3(B=8), ("exp", 13))
    cases["cfg3_b8_philox"] = (W.config3(B=8), ("philox", 7, 123))
    cases["cfg4_b32"] = (_with_penalty_only(W.config4(B=32)), ("exp", 14))
    cases["cfg5_b8_topp"] = (_with_penalty_only(W.config5(B=8)), ("exp", 15))
    cases["small_v1"] = (_small("small_v1", 4, 1, 21, use_top_p=True), ("exp", 31))
    cases["small_v3"] = (_small("small_v3", 16, 3, 22, use_top_p=True), ("exp", 32))
    cases["small_v100"] = (_small("small_v100", 64, 100, 23, use_top_p=True), ("exp", 33))
    cases["small_v1000_nop"] = (_small("small_v1000_nop", 64, 1000, 24, use_top_p=False), ("exp", 34))
    cases["small_v5000_f32"] = (_small("small_v5000_f32", 32, 5000, 25, dtype="f32", use_top_p=True), ("exp", 35))
    cases["small_ties"] = (_small("small_ties", 32, 777, 26, mode="ties", use_top_p=True), ("exp", 36))
    cases["small_equal"] = (_small("small_equal", 8, 300, 27, mode="equal", use_top_p=True), ("exp", 37))
    cases["small_neginf"] = (_small("small_neginf", 32, 2000, 28, mode="neginf", use_top_p=True), ("exp", 38))
    cases["small_philox"] = (_small("small_philox", 64, 3001, 29, use_top_p=True), ("philox", 99, 5))
    cases["small_greedy_all"] = (_small("small_greedy_all", 16, 513, 30, temps=np.zeros(16)), ("exp", 39))
    return cases


def make_noise(spec, B, V) -> np.ndarray:
    if spec[0] == "exp":
        return W.exp_noise(B, V, spec[1])
    return N.philox_noise(B, V, spec[1], spec[2])


def penalised_f32(w: W.Workload) -> np.ndarray:
    """float32 logits after the repetition penalty (what the sampler sees)."""
    from oracle.sampler_oracle import penalise
    x = w.logits_f32().copy()
    if w.history is None:
        return x
    for b in range(w.B):
        x[b] = penalise(x[b], w.history[b, : int(w.history_lens[b])], float(w.rep_penalties[b]))
    return x


def digest(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()
