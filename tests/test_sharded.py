"""Vocab-sharded sampling (tensor-parallel lm_head) against the oracle.

* GPU, one process: ``sharded.emulate`` runs the whole protocol for 1, 2, 4
  and 8 shards of one logits tensor (the all-gathers become concatenations);
  the ids must equal the oracle's (and so the single-GPU sampler's) under the
  same noise, for small top-k rows (one all-gather), top-p race rows (the
  test round), unfiltered, greedy and penalised rows, in Philox and
  shared-noise mode.
* GPU, two processes over NCCL (needs two GPUs): ``ShardedSampler`` on each
  rank's shard gives the single-GPU ids.
* CPU, two ``gloo`` processes: the host plumbing (shard bounds, row gather
  for the exact fallback) on the collective the GPU path uses.
"""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import noise as ON
from oracle import sampler_oracle as O
from qedge_b200 import workloads as W
from qedge_b200.sharded import NSLICE, shard_bounds, slice_start


def _oracle(w, noise):
    return O.sample(w.logits_f32(), w.temperatures, w.top_ps, noise, top_ks=w.top_ks,
                    rep_penalties=w.rep_penalties, history=w.history, history_lens=w.history_lens,
                    all_greedy=bool(np.all(w.temperatures <= 1e-5)), use_top_p=w.use_top_p)


def _emulate(w, nshards, *, mode, seed=5, step=9):
    from qedge_b200 import sharded
    dev = "cuda"
    kw = dict(top_ks=torch.from_numpy(w.top_ks).to(dev), use_top_p=w.use_top_p,
              all_greedy=bool(np.all(w.temperatures <= 1e-5)))
    if w.history is not None:
        kw.update(rep_penalties=torch.from_numpy(w.rep_penalties).to(dev),
                  history=torch.from_numpy(w.history).to(dev),
                  history_lens=torch.from_numpy(w.history_lens).to(dev))
    if mode == "exp":
        noise = W.exp_noise(w.B, w.V, 300 + seed)
        kw["noise"] = torch.from_numpy(noise).to(dev)
    else:
        noise = ON.philox_noise(w.B, w.V, seed, step)
    ids, status = sharded.emulate(W.to_device(w, dev), nshards, torch.from_numpy(w.temperatures).to(dev),
                                  torch.from_numpy(w.top_ps).to(dev), seed=seed, step=step, **kw)
    torch.cuda.synchronize()
    return ids.cpu().numpy(), status.cpu().numpy(), noise


def _mixed(B=48, V=W.VOCAB, seed=11):
    """Rows of every kind: greedy, top-k 1/20/64, top-k 1000, top-p only,
    unfiltered, with a repetition penalty on every other row."""
    g = np.random.Generator(np.random.PCG64(seed))
    x = (g.standard_normal((B, V), dtype=np.float32) * np.float32(2.5))
    temps = g.choice(np.array([0.0, 0.5, 0.8, 1.0, 1.3], np.float32), size=B)
    tks = g.choice(np.array([0, 1, 20, 64, 1000], np.int32), size=B)
    tps = g.uniform(0.5, 1.0, size=B).astype(np.float32)
    hist = g.integers(0, V, size=(B, 256)).astype(np.int32)
    rps = np.where(np.arange(B) % 2 == 0, np.float32(1.1), np.float32(1.0)).astype(np.float32)
    return W.Workload("mixed", W.to_bf16_bits(x), "bf16", temps, tps, tks, rps, hist,
                      np.full(B, 256, np.int32), use_top_p=True)


# ---------------------------------------------------------------- CPU
def test_shard_bounds_partition_the_vocab():
    for V in (128, 1000, 151_936, 248_320, 262_144):
        for n in (1, 2, 4, 8, 16):
            b = [shard_bounds(V, n, s) for s in range(n)]
            assert b[0][0] == 0 and b[-1][1] == V
            assert all(b[i][1] == b[i + 1][0] for i in range(n - 1))
            # shard boundaries are canonical slice boundaries (noise tree intact)
            assert all(lo == slice_start(s * NSLICE // n, V) for s, (lo, _) in enumerate(b))
            assert all(lo % 8 == 0 for lo, _ in b)
    with pytest.raises(ValueError):
        shard_bounds(1000, 3, 0)


def _gloo_worker(rank, world, port, V, result):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from qedge_b200.sharded import ShardedSampler
        s = ShardedSampler(0, nshards=world, shard=rank)
        full = torch.arange(3 * V, dtype=torch.float32).view(3, V)
        v0, v1 = shard_bounds(V, world, rank)
        rows = full[[0, 2], v0:v1]
        got = s._gather_rows(rows, V)
        result[rank] = bool(torch.equal(got, full[[0, 2]]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_gloo_row_gather_for_exact_fallback(world):
    """Two gloo ranks rebuild full rows from their shards (the fallback path)."""
    import socket
    with socket.socket() as so:
        so.bind(("127.0.0.1", 0))
        port = so.getsockname()[1]
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        result = m.dict()
        procs = [ctx.Process(target=_gloo_worker, args=(r, world, port, 4099, result)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
        assert all(p.exitcode == 0 for p in procs)
        assert dict(result) == {r: True for r in range(world)}


# ---------------------------------------------------------------- GPU, one process
@pytest.mark.gpu
@pytest.mark.parametrize("nshards", [1, 2, 4, 8])
@pytest.mark.parametrize("mode", ["philox", "exp"])
def test_config5_sharded_vs_oracle(nshards, mode):
    """Config 5 (top-k 64, top-p 0.9, T 0.8): one all-gather decides every row."""
    w = W.config5(B=24)
    ids, status, noise = _emulate(w, nshards, mode=mode)
    np.testing.assert_array_equal(ids, _oracle(w, noise))
    assert np.all(status == 4)


@pytest.mark.gpu
@pytest.mark.parametrize("nshards", [2, 8])
def test_config3_sharded_top_p_rounds(nshards):
    """Nucleus-only rows go through the candidate-test round."""
    w = W.config3(B=24)
    ids, status, noise = _emulate(w, nshards, mode="philox")
    ok = (status & 8) == 0
    np.testing.assert_array_equal(ids[ok], _oracle(w, noise)[ok])
    assert ok.mean() > 0.8


@pytest.mark.gpu
@pytest.mark.parametrize("nshards", [1, 4])
@pytest.mark.parametrize("mode", ["philox", "exp"])
def test_mixed_rows_sharded_vs_oracle(nshards, mode):
    w = _mixed()
    ids, status, noise = _emulate(w, nshards, mode=mode)
    ok = (status & 8) == 0
    np.testing.assert_array_equal(ids[ok], _oracle(w, noise)[ok])
    assert np.all(ids[~ok] == -1)


@pytest.mark.gpu
def test_config1_unfiltered_sharded():
    w = W.config1()
    for n in (2, 16):
        ids, status, noise = _emulate(w, n, mode="philox")
        np.testing.assert_array_equal(ids, _oracle(w, noise))


@pytest.mark.gpu
def test_sharded_equals_single_gpu_sampler():
    """Same (seed, step): the sharded ids equal QESampler's on the full rows."""
    from qedge_b200.sampler import QESampler
    w = W.config5(B=32)
    dev = "cuda"
    ids, status, _ = _emulate(w, 4, mode="philox", seed=21, step=4)
    ref = QESampler(seed=21)(W.to_device(w, dev), torch.from_numpy(w.temperatures).to(dev),
                             torch.from_numpy(w.top_ps).to(dev), use_top_p=True,
                             top_ks=torch.from_numpy(w.top_ks).to(dev), step=4)
    np.testing.assert_array_equal(ids, ref.cpu().numpy())


# ---------------------------------------------------------------- GPU, two processes over NCCL
def _nccl_worker(rank, world, port, result):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    from datetime import timedelta
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        from qedge_b200.sampler import QESampler
        from qedge_b200.sharded import ShardedSampler
        w = W.config3(B=16)
        dev = torch.device("cuda", rank)
        full = W.to_device(w, dev)
        v0, v1 = shard_bounds(w.V, world, rank)
        temps = torch.from_numpy(w.temperatures).to(dev)
        tps = torch.from_numpy(w.top_ps).to(dev)
        s = ShardedSampler(13, nshards=world, shard=rank)
        ids = s(full[:, v0:v1].contiguous(), w.V, temps, tps, use_top_p=True, step=2)
        ref = QESampler(13)(full, temps, tps, use_top_p=True, step=2)
        torch.cuda.synchronize()
        result[rank] = bool(torch.equal(ids, ref))
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_nccl_two_gpus_match_single_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import socket
    with socket.socket() as so:
        so.bind(("127.0.0.1", 0))
        port = so.getsockname()[1]
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        result = m.dict()
        procs = [ctx.Process(target=_nccl_worker, args=(r, 2, port, result)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(300)
        assert all(p.exitcode == 0 for p in procs)
        assert dict(result) == {0: True, 1: True}


@pytest.mark.gpu
def test_sharded_sampler_finishes_slow_rows_exactly():
    """``ShardedSampler`` (one shard, identity all-gather) finishes the rows the
    candidate round could not decide by gathering them and running the
    single-GPU sampler: every id equals the oracle's."""
    from qedge_b200.sharded import ShardedSampler
    w = _mixed(B=64, seed=23)
    dev = "cuda"
    s = ShardedSampler(9, nshards=1, shard=0, allgather=lambda t: t)
    st = torch.zeros(w.B, dtype=torch.int32, device=dev)
    ids = s(W.to_device(w, dev), w.V, torch.from_numpy(w.temperatures).to(dev),
            torch.from_numpy(w.top_ps).to(dev), use_top_p=True, top_ks=torch.from_numpy(w.top_ks).to(dev),
            rep_penalties=torch.from_numpy(w.rep_penalties).to(dev), history=torch.from_numpy(w.history).to(dev),
            history_lens=torch.from_numpy(w.history_lens).to(dev), step=6, out_status=st)
    torch.cuda.synchronize()
    noise = ON.philox_noise(w.B, w.V, 9, 6)
    np.testing.assert_array_equal(ids.cpu().numpy(), _oracle(w, noise))
    assert s.fallback_rows > 0
