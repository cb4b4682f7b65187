"""Seeded synthetic sampler workloads (the five benchmark configurations).

The reference publishes no sampler benchmark; these inputs stand in for the
logits its decode loop produces (``src/compute/model_runner.py:201, 298``,
``vocab_size`` from the model config, V = 248,320 for Qwen3.5).  Everything
is generated with numpy's PCG64 so the same seed gives the same bits on any
host, and converted to bf16 with round-to-nearest-even (as torch does).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

VOCAB = 248_320


@dataclass
class Workload:
    name: str
    logits_bits: np.ndarray            # [B, V] uint16 (bf16/fp16 bits) or float32
    dtype: str                         # "bf16" | "f16" | "f32"
    temperatures: np.ndarray           # [B] float32
    top_ps: np.ndarray                 # [B] float32
    top_ks: np.ndarray                 # [B] int32 (0 = off)
    rep_penalties: np.ndarray          # [B] float32
    history: np.ndarray | None         # [B, H] int32
    history_lens: np.ndarray | None    # [B] int32
    use_top_p: bool
    all_greedy: bool = False
    meta: dict = field(default_factory=dict)

    @property
    def B(self) -> int:
        return self.logits_bits.shape[0]

    @property
    def V(self) -> int:
        return self.logits_bits.shape[1]

    def logits_f32(self) -> np.ndarray:
        if self.dtype == "f32":
            return np.asarray(self.logits_bits, dtype=np.float32)
        if self.dtype == "bf16":
            return (self.logits_bits.astype(np.uint32) << np.uint32(16)).view(np.float32)
        return self.logits_bits.view(np.float16).astype(np.float32)


def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = (u.astype(np.uint64) + 0x7FFF + ((u >> 16) & 1)) >> 16
    return r.astype(np.uint16)


def _rng(seed: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(seed))


def exp_noise(B: int, V: int, seed: int) -> np.ndarray:
    """Shared Exp(1) noise tensor for parity runs (the stand-in for the
    generator behind ``torch.multinomial``).

    Exact zeros (float32 draws can round to 0) are raised to the smallest
    normal float: the sampler contract is E > 0.  With E == 0 the reference's
    race divides 0/0 for a token removed by top-p and ``torch.argmax`` picks
    the NaN, i.e. it samples a token outside the nucleus.
    """
    e = _rng(seed).standard_exponential((B, V), dtype=np.float32)
    return np.maximum(e, np.float32(np.finfo(np.float32).tiny))


def config1(V: int = VOCAB, seed: int = 0) -> Workload:
    """B=1 fp32 logits ~ N(0, 2^2); T=0.7; no top-k/top-p (engine default
    single-sequence decode)."""
    x = _rng(seed).standard_normal((1, V), dtype=np.float32) * np.float32(2.0)
    return Workload("config1_b1_fp32", x.astype(np.float32), "f32",
                    np.array([0.7], np.float32), np.ones(1, np.float32),
                    np.zeros(1, np.int32), np.ones(1, np.float32), None, None,
                    use_top_p=False)


def config2(B: int = 64, V: int = VOCAB, seed: int = 2, H: int = 2048) -> Workload:
    """bf16 N(0, 3^2) with 8 spike ids per row SET to +12; T=0.8, top_k=50,
    top_p=0.9, repetition penalty 1.1 over H uniform history ids."""
    g = _rng(seed)
    x = g.standard_normal((B, V), dtype=np.float32) * np.float32(3.0)
    spikes = g.integers(0, V, size=(B, 8))
    np.put_along_axis(x, spikes, np.float32(12.0), axis=1)
    hist = g.integers(0, V, size=(B, H)).astype(np.int32)
    return Workload("config2_b64_topk50_topp09_rep", to_bf16_bits(x), "bf16",
                    np.full(B, 0.8, np.float32), np.full(B, 0.9, np.float32),
                    np.full(B, 50, np.int32), np.full(B, 1.1, np.float32),
                    hist, np.full(B, H, np.int32), use_top_p=True)


def config3(B: int = 256, V: int = VOCAB, seed: int = 3) -> Workload:
    """bf16 Zipf logits: -1.1*ln(rank) + N(0, 0.5^2), ranks under a random
    per-row permutation; top_p=0.95, T=1.0, no top-k (nucleus only)."""
    g = _rng(seed)
    ln_rank = np.log(np.arange(1, V + 1, dtype=np.float64)).astype(np.float32)
    x = np.empty((B, V), dtype=np.float32)
    for b in range(B):
        perm = g.permutation(V)
        x[b] = np.float32(-1.1) * ln_rank[perm]
    x += g.standard_normal((B, V), dtype=np.float32) * np.float32(0.5)
    return Workload("config3_b256_zipf_topp095", to_bf16_bits(x), "bf16",
                    np.ones(B, np.float32), np.full(B, 0.95, np.float32),
                    np.zeros(B, np.int32), np.ones(B, np.float32), None, None,
                    use_top_p=True)


def config4(B: int = 1024, V: int = VOCAB, seed: int = 4, H: int = 512) -> Workload:
    """bf16 N(0, 2.5^2) with mixed per-row params: T in {0,0.3,0.7,1,1.5},
    top_k in {off,1,20,1000}, top_p ~ U[0.5,1], repetition penalty 1.1 over
    512 history ids (the configuration gives no penalty value; 1.1 is used)."""
    g = _rng(seed)
    x = g.standard_normal((B, V), dtype=np.float32) * np.float32(2.5)
    temps = g.choice(np.array([0.0, 0.3, 0.7, 1.0, 1.5], np.float32), size=B)
    tks = g.choice(np.array([0, 1, 20, 1000], np.int32), size=B)
    tps = g.uniform(0.5, 1.0, size=B).astype(np.float32)
    hist = g.integers(0, V, size=(B, H)).astype(np.int32)
    return Workload("config4_b1024_mixed", to_bf16_bits(x), "bf16",
                    temps.astype(np.float32), tps, tks.astype(np.int32),
                    np.full(B, 1.1, np.float32), hist, np.full(B, H, np.int32),
                    use_top_p=True)


def config5(B: int = 512, V: int = VOCAB, seed: int = 5) -> Workload:
    """bf16 N(0, 2^2); T=0.8, top_k=64, top_p=0.9 (vocab-sharded case)."""
    x = _rng(seed).standard_normal((B, V), dtype=np.float32) * np.float32(2.0)
    return Workload("config5_b512_topk64_topp09", to_bf16_bits(x), "bf16",
                    np.full(B, 0.8, np.float32), np.full(B, 0.9, np.float32),
                    np.full(B, 64, np.int32), np.ones(B, np.float32), None, None,
                    use_top_p=True)


CONFIGS = {1: config1, 2: config2, 3: config3, 4: config4, 5: config5}


def to_device(w: Workload, device="cuda"):
    """Upload the logits of a workload as a torch tensor of its dtype."""
    import torch
    if w.dtype == "f32":
        return torch.from_numpy(np.ascontiguousarray(w.logits_bits, np.float32)).to(device)
    dt = {"bf16": torch.bfloat16, "f16": torch.float16}[w.dtype]
    t = torch.from_numpy(np.ascontiguousarray(w.logits_bits).view(np.int16)).to(device)
    return t.view(dt)
