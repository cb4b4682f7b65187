"""min-p (``SamplingParams.min_p``, ``src/sampling_params.py:11``; packed by
``src/data/batch.py:60, 158`` but never applied by the reference sampler) and
per-request seeds on the streaming path, against the oracle's documented
min-p rule and against one call per row with the row's own seed."""
import numpy as np
import pytest
import torch

from oracle import noise as ON
from oracle import sampler_oracle as O
from qedge_b200 import workloads as W
from tests.gpu_util import run

pytestmark = pytest.mark.gpu


def _flat_rows(B, V, seed, scale):
    g = np.random.Generator(np.random.PCG64(seed))
    x = g.standard_normal((B, V), dtype=np.float32) * np.float32(scale)
    return W.to_bf16_bits(x)


@pytest.mark.parametrize("mode", ["exp", "philox"])
def test_min_p_vs_oracle(mode):
    from qedge_b200.sampler import QESampler
    B, V = 32, 248_320
    bits = _flat_rows(B, V, 41, 2.5)
    g = np.random.Generator(np.random.PCG64(42))
    mps = g.choice(np.array([0.0, 0.01, 0.05, 0.2, 0.6], np.float32), size=B)
    tps = g.choice(np.array([1.0, 0.9, 0.5], np.float32), size=B)
    tks = g.choice(np.array([0, 40, 1000], np.int32), size=B)
    temps = g.choice(np.array([0.7, 1.0, 1.5], np.float32), size=B)
    w = W.Workload("minp", bits, "bf16", temps, tps, tks, np.ones(B, np.float32), None, None, use_top_p=True)
    mp_dev = torch.from_numpy(mps).cuda()
    if mode == "exp":
        noise = W.exp_noise(B, V, 43)
        ids = run(QESampler(seed=0), w, noise, min_ps=mp_dev)
    else:
        noise = ON.philox_noise(B, V, 44, 5)
        ids = run(QESampler(seed=0), w, None, seed=44, step=5, min_ps=mp_dev)
    want = O.sample(w.logits_f32(), temps, tps, noise, top_ks=tks, use_top_p=True, min_ps=mps)
    np.testing.assert_array_equal(ids, want)


def test_per_row_seeds_equal_single_row_calls():
    from qedge_b200.sampler import QESampler
    w = W.config3(B=8)
    seeds = np.array([3, 2**63 + 5, 0, 17, 2**64 - 1, 9, 123456789, 4], dtype=np.uint64)
    s = QESampler(seed=1)
    lg = W.to_device(w, "cuda")
    t = torch.from_numpy(w.temperatures).cuda()
    p = torch.from_numpy(w.top_ps).cuda()
    ids = s(lg, t, p, use_top_p=True, step=6, seeds=torch.from_numpy(seeds.view(np.int64)).cuda()).cpu().numpy()
    for r in range(8):
        one = s(lg[r:r + 1], t[r:r + 1], p[r:r + 1], use_top_p=True, step=6, seed=int(seeds[r]),
                row_offset=r).cpu().numpy()
        assert ids[r] == one[0], r
