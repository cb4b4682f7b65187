"""The call-site shim on a live (stub) runner with the real CUDA sampler:
``integration.install`` replaces ``ModelRunner.sampler`` and
``ModelRunner._sample_gpu`` (reference ``src/compute/model_runner.py:28,
77-93``); the ids it returns equal a direct ``QESampler`` call on the same
packed parameters and the oracle's on the same Philox noise."""
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from oracle import noise as ON
from oracle import sampler_oracle as O
from qedge_b200 import integration
from qedge_b200 import workloads as W
from qedge_b200.sampler import QESampler

pytestmark = pytest.mark.gpu


def _seq(t, p=None, k=None, rp=1.0, ids=()):
    return SimpleNamespace(temperature=t, top_p=p, top_k=k, min_p=None, repetition_penalty=rp,
                           token_ids=list(ids))


def test_installed_runner_matches_direct_call_and_oracle():
    V, B = 50_000, 6
    g = np.random.Generator(np.random.PCG64(31))
    x = g.standard_normal((B, V), dtype=np.float32) * np.float32(2.0)
    bits = W.to_bf16_bits(x)
    seqs = [_seq(0.0), _seq(1.0, 0.9), _seq(0.7, 0.5, 20), _seq(1.3, None, 5, 1.2, g.integers(0, V, 40)),
            _seq(0.9, 0.95, None, 1.1, g.integers(0, V, 300)), _seq(1.0)]
    runner = SimpleNamespace(batch=SimpleNamespace(max_bs=8, vocab_size=V), device="cuda",
                             sampler="orig", _sample_gpu="orig_fn",
                             sample_cpu=torch.empty(4, dtype=torch.int64))
    integration.install(runner, seed=21, history_width=512)
    logits = torch.from_numpy(bits.view(np.int16)).cuda().view(torch.bfloat16)
    ids = runner._sample_gpu([logits[:3], logits[3:]], seqs).cpu().numpy()
    assert runner.qe_step == 1 and runner.sample_cpu.numel() >= 8
    qb = runner.qe_batch
    direct = QESampler(seed=21)(logits, qb.temperatures[:B], qb.top_ps[:B], all_greedy=qb.all_greedy,
                                use_top_p=qb.use_top_p, step=0, **qb.sampler_kwargs(B)).cpu().numpy()
    np.testing.assert_array_equal(ids, direct)
    # oracle on the same packed parameters and the same Philox noise
    temps = np.array([s.temperature for s in seqs], np.float32)
    tps = np.array([1.0 if s.top_p is None else s.top_p for s in seqs], np.float32)
    tks = np.array([0 if s.top_k is None else s.top_k for s in seqs], np.int64)
    rps = np.array([s.repetition_penalty for s in seqs], np.float32)
    hist = np.zeros((B, 512), np.int32)
    hl = np.zeros(B, np.int32)
    for r, s in enumerate(seqs):
        hl[r] = len(s.token_ids[-512:])
        hist[r, :hl[r]] = s.token_ids[-512:]
    want = O.sample(W.Workload("x", bits, "bf16", temps, tps, tks, rps, None, None, True).logits_f32(),
                    temps, tps, ON.philox_noise(B, V, 21, 0), top_ks=tks, rep_penalties=rps,
                    history=hist, history_lens=hl, use_top_p=True)
    np.testing.assert_array_equal(ids, want)
    integration.uninstall(runner)
    assert runner.sampler == "orig"
