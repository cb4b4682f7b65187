"""Benchmark of the B200 token sampler on the headline configuration.

Metric: sampled rows/sec and us per decode-step sample at
B=256, V=248,320 (config 3: bf16 Zipf logits, top_p=0.95, T=1.0, Philox
noise), and the fraction of the HBM roofline.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config 3] [--mode philox|noise] [--vocab-sharded]

A step is one sampler call over one batch of B rows resident in HBM.  L2 is
not allowed to serve the logits: the timed loop rotates over enough distinct
logits buffers to exceed twice the L2 size.  Multi-GPU (torchrun, NCCL):
rows are sharded with no data-path collective (weak scaling: every rank
samples its own B rows, keyed on its global row offset); time is the max
over ranks.  ``--vocab-sharded`` (config 5 by default) instead splits the
vocabulary over the ranks (tensor-parallel lm_head): every rank holds
``[B, V/N]`` of the same rows and the shards are merged by NCCL all-gathers
of per-slice records (strong scaling).  ``--impl reference`` times the
reference algorithm's CPU restatement (oracle/) on the host cores, rank 0
only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "sampled rows/sec at B=256, V=248,320 (config 3: Zipf bf16, top_p=0.95)"
L2_BYTES = 126 * 1024 * 1024


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks/throttle sampling during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.samples = []
        self._stop = threading.Event()
        self._t = None

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                      "--format=csv,noheader,nounits"], capture_output=True,
                                     text=True, timeout=5).stdout.strip()
                if out:
                    self.samples.append([s.strip() for s in out.split(",")])
            except Exception:
                pass
            self._stop.wait(0.1)

    def __enter__(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        self._t.join(timeout=10)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4)
                          if len(s) > 5 + i and s[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(self.samples)}


def cpu_baseline(cfg: int, rows: int | None = None):
    """Time the oracle (CPU restatement of the reference sampler) on the host
    cores over a bounded sample of the workload: the first `rows` rows of
    configuration `cfg` (all B by default), one row per task on a spawn pool
    that holds the pre-generated workload in shared memory."""
    from oracle.cpu_bench import CpuSampler
    with CpuSampler(cfg) as cs:
        n = cs.B if rows is None else min(rows, cs.B)
        dt = cs.step(n)
        return {"value": n / dt, "unit": "rows/s", "cores": cs.procs, "kind": "port",
                "sample": f"{n} rows of {cs.name} (V={cs.V:,}) through oracle/sampler_oracle.py "
                          f"(numpy restatement of the reference sampler) on a {cs.procs}-process pool; "
                          f"workload generated before timing"}


def run_reference(args, rank: int, world: int):
    """The reference algorithm's CPU implementation (the oracle port) on the
    host cores, full config batches per step, rank 0 only."""
    if rank != 0:
        return
    from oracle.cpu_bench import CpuSampler
    with CpuSampler(args.config) as cs:
        for _ in range(args.warmup):
            cs.step()
        times = [cs.step() for _ in range(args.steps)]
    total = sum(times)
    v = cs.B * args.steps / total
    line = {"impl": "reference", "metric": METRIC if args.config == 3 else f"sampled rows/sec, config {args.config}",
            "value": v, "unit": "rows/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": {"workload": cs.name, "B": cs.B, "V": cs.V},
            "cpu_baseline": {"value": v, "unit": "rows/s", "cores": cs.procs, "kind": "port",
                             "sample": f"every step samples all {cs.B} rows of {cs.name} through "
                                       f"oracle/sampler_oracle.py on a {cs.procs}-process pool"},
            "e2e": {"value": v, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_vocab_sharded(args, rank: int, world: int, local: int):
    """Config 5: every rank samples the same B rows from its vocab shard."""
    import torch
    import torch.distributed as dist
    from qedge_b200 import workloads as W
    from qedge_b200.sharded import ShardedSampler, shard_bounds

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    w = W.CONFIGS[args.config]()
    B, V = w.B, w.V
    v0, v1 = shard_bounds(V, world, rank)
    esize = 4 if w.dtype == "f32" else 2
    shard_bytes = B * (v1 - v0) * esize
    nbuf = max(2, int(np.ceil(2 * L2_BYTES / shard_bytes)) + 1)
    full = W.to_device(w, dev)
    bufs = [full[:, v0:v1].roll(shifts=i * 997, dims=1).contiguous() for i in range(nbuf)]
    del full
    temps = torch.from_numpy(w.temperatures).to(dev)
    tps = torch.from_numpy(w.top_ps).to(dev)
    tks = torch.from_numpy(w.top_ks.astype(np.int32)).to(dev)
    if world > 1:
        sampler = ShardedSampler(1234, nshards=world, shard=rank)
    else:
        sampler = ShardedSampler(1234, nshards=1, shard=0, allgather=lambda t: t)
    stream = torch.cuda.current_stream(dev)

    def step(i, buf=None):
        return sampler(bufs[i % nbuf] if buf is None else buf, V, temps, tps, use_top_p=w.use_top_p,
                       top_ks=tks, step=i)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(local)
    with clocks:
        ev0.record(stream)
        for i in range(args.steps):
            step(args.warmup + i)
        ev1.record(stream)
        torch.cuda.synchronize()
    total_ms = ev0.elapsed_time(ev1)
    host = torch.empty_like(bufs[0], device="cpu").pin_memory()
    host.copy_(bufs[0])
    out_host = torch.empty(B, dtype=torch.int64).pin_memory()
    dbuf = torch.empty_like(bufs[0])
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(max(args.e2e_steps, 1)):
        dbuf.copy_(host, non_blocking=True)
        out_host.copy_(step(10_000 + i, dbuf), non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / max(args.e2e_steps, 1)
    if world > 1:
        t = torch.tensor([total_ms, e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms, e2e_ms = float(t[0].item()), float(t[1].item())
    ms = total_ms / args.steps
    hbm, peak_kind = peaks()
    alg = shard_bytes + 8 * B
    achieved = alg / (ms * 1e-3) / 1e9
    if rank == 0:
        line = {
            "metric": f"sampled rows/sec, config {args.config} vocab-sharded over {world} GPU(s)",
            "value": B / (ms * 1e-3), "unit": "rows/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": w.dtype + " in, f32 math", "data": "synthetic",
            "config": {"workload": w.name, "B": B, "V": V, "noise": "philox",
                       "parallelism": f"vocab x{world} (NCCL all-gather of slice records)",
                       "l2": f"rotating {nbuf} shard buffers per rank"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                         "frac": achieved / hbm, "peak_kind": peak_kind, "traffic": None,
                         "alg_bytes_per_launch": alg, "note": "per rank, whole step incl. collectives"},
            "e2e": {"value": B / (e2e_ms * 1e-3), "unit": "rows/s", "h2d_bytes_per_step": shard_bytes,
                    "d2h_bytes_per_step": 8 * B},
            "gpu_launches": args.steps * 4,
            "fallback_rows": sampler.fallback_rows,
            "clocks": clocks.summary(),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


LAUNCHES_PER_CALL = 6   # scan, decide, count, retry, count, finish (qe_sample_stream.cu)


def prepare_config(cfg: int, dev, mode: str = "philox"):
    """Device inputs of a configuration: rotating logits buffers (together
    more than 2x L2, so that L2 never serves the logits between steps) and
    the per-row parameters."""
    import torch
    from qedge_b200 import workloads as W
    w = W.CONFIGS[cfg]()
    esize = 4 if w.dtype == "f32" else 2
    bytes_per_batch = w.B * w.V * esize
    nbuf = max(2, int(np.ceil(2 * L2_BYTES / bytes_per_batch)) + 1)
    base = W.to_device(w, dev)
    bufs = [base] + [base.roll(shifts=i * 997, dims=1).contiguous() for i in range(1, nbuf)]
    kw = {"top_ks": torch.from_numpy(w.top_ks.astype(np.int32)).to(dev)}
    hist_bytes = 0
    if w.history is not None:
        kw.update(rep_penalties=torch.from_numpy(w.rep_penalties).to(dev),
                  history=torch.from_numpy(w.history).to(dev),
                  history_lens=torch.from_numpy(w.history_lens).to(dev))
        hist_bytes = int(w.history_lens.sum()) * 4
    if mode == "noise":
        kw["noise"] = torch.from_numpy(W.exp_noise(w.B, w.V, 1)).to(dev)
    temps = torch.from_numpy(w.temperatures).to(dev)
    tps = torch.from_numpy(w.top_ps).to(dev)
    alg = bytes_per_batch + hist_bytes + 8 * w.B + (w.B * w.V * 4 if mode == "noise" else 0)
    return {"w": w, "bufs": bufs, "nbuf": nbuf, "kw": kw, "temps": temps, "tps": tps,
            "bytes_per_batch": bytes_per_batch, "alg": alg}


def time_steps(sampler, c, stream, steps: int, warmup: int, row_offset: int = 0, step0: int = 0):
    """Warm-up, then `steps` sampler calls, each bracketed by CUDA events on
    the launching stream.  Returns (total ms, per-call ms list)."""
    import torch
    w = c["w"]

    def step(i):
        return sampler(c["bufs"][i % c["nbuf"]], c["temps"], c["tps"], use_top_p=w.use_top_p, step=step0 + i,
                       row_offset=row_offset, **c["kw"])

    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    per = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    ev0.record(stream)
    for i in range(steps):
        per[i][0].record(stream)
        step(warmup + i)
        per[i][1].record(stream)
    ev1.record(stream)
    torch.cuda.synchronize()
    return ev0.elapsed_time(ev1), [a.elapsed_time(b) for a, b in per]


def stats(ms_list):
    v = np.asarray(ms_list) * 1e3
    return {"median": float(np.median(v)), "p10": float(np.percentile(v, 10)), "p90": float(np.percentile(v, 90))}


def traffic_record(cfg: int, mode: str):
    """DRAM bytes per call measured by ncu for this configuration (a committed
    summary, tagged with the kernels and the commit it was measured on)."""
    prof = ROOT / "profiles" / f"traffic_config{cfg}_{mode}.json"
    if not prof.exists():
        return None, None
    d = json.loads(prof.read_text())
    return d.get("dram_bytes_per_call"), {k: d.get(k) for k in ("commit", "kernels", "source")}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", type=int, default=3)
    ap.add_argument("--mode", default="philox", choices=["philox", "noise"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra-configs", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--vocab-sharded", action="store_true")
    args = ap.parse_args()
    if args.vocab_sharded and "--config" not in sys.argv:
        args.config = 5
    args.warmup = max(args.warmup, 3)

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if "--steps" not in sys.argv:
            args.steps, args.warmup = 5, 3
        return run_reference(args, rank, world)
    if args.vocab_sharded:
        return run_vocab_sharded(args, rank, world, local)

    import torch
    import torch.distributed as dist
    from qedge_b200.sampler import QESampler

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    c = prepare_config(args.config, dev, args.mode)
    w = c["w"]
    B, V = w.B, w.V
    row_offset = rank * B
    sampler = QESampler(seed=1234)
    stream = torch.cuda.current_stream(dev)
    if world > 1:
        dist.barrier()
    clocks = ClockSampler(local)
    with clocks:
        total_ms, launch_ms = time_steps(sampler, c, stream, args.steps, args.warmup, row_offset)
    if world > 1:
        t = torch.tensor([total_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
        dist.barrier()
    ms = total_ms / args.steps

    # end to end through the public API: pinned host logits -> device, sample,
    # ids -> host, every step
    host = torch.empty_like(c["bufs"][0], device="cpu").pin_memory()
    host.copy_(c["bufs"][0])
    out_host = torch.empty(B, dtype=torch.int64).pin_memory()
    dbuf = torch.empty_like(c["bufs"][0])
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(max(args.e2e_steps, 1)):
        dbuf.copy_(host, non_blocking=True)
        ids = sampler(dbuf, c["temps"], c["tps"], use_top_p=w.use_top_p, step=10_000 + i,
                      row_offset=row_offset, **c["kw"])
        out_host.copy_(ids, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / max(args.e2e_steps, 1)
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())

    hbm, peak_kind = peaks()
    st = stats(launch_ms)
    achieved = c["alg"] / (st["median"] * 1e-6) / 1e9
    traffic, traffic_src = traffic_record(args.config, args.mode)
    line = None
    if rank == 0:
        line = {
            "metric": METRIC if args.config == 3 else f"sampled rows/sec, config {args.config}",
            "value": world * B / (ms * 1e-3), "unit": "rows/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "us_per_sample_step": ms * 1e3, "us_per_call": st,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": {"bf16": "bf16", "f16": "f16", "f32": "f32"}[w.dtype] + " in, f32 math",
            "data": "synthetic",
            "config": {"workload": w.name, "B": B, "V": V, "noise": args.mode,
                       "parallelism": f"rows x{world} (no collective)",
                       "l2": f"rotating {c['nbuf']} logits buffers "
                             f"({c['nbuf'] * c['bytes_per_batch'] / 2**20:.0f} MiB > 2x L2)"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                         "frac": achieved / hbm, "peak_kind": peak_kind,
                         "frac_of_8tbs": achieved / 8000.0, "traffic": traffic,
                         "traffic_source": traffic_src,
                         "alg_bytes_per_launch": c["alg"],
                         "note": "achieved = algorithmic bytes / median time of one whole sampler call "
                                 f"({LAUNCHES_PER_CALL} launches); the scan kernel is the dominant one"},
            "e2e": {"value": world * B / (e2e_ms * 1e-3), "unit": "rows/s",
                    "h2d_bytes_per_step": c["bytes_per_batch"], "d2h_bytes_per_step": 8 * B},
            "gpu_launches": args.steps * LAUNCHES_PER_CALL,
            "clocks": clocks.summary(),
        }
    del c
    torch.cuda.empty_cache()
    if world == 1 and not args.no_extra_configs:
        # the other benchmark configurations: per-call time over >= 100 calls
        extra = {}
        for cfg in (1, 2, 4, 5):
            if cfg == args.config:
                continue
            ce = prepare_config(cfg, dev, args.mode)
            _, lm = time_steps(sampler, ce, stream, max(args.steps, 100), 10, 0, step0=50_000)
            se = stats(lm)
            ach = ce["alg"] / (se["median"] * 1e-6) / 1e9
            extra[f"config{cfg}"] = {"workload": ce["w"].name, "B": ce["w"].B, "us_per_call": se,
                                     "rows_per_s": ce["w"].B / (se["median"] * 1e-6),
                                     "roofline_frac": ach / hbm, "alg_bytes_per_launch": ce["alg"]}
            del ce
            torch.cuda.empty_cache()
            if not args.no_cpu_baseline:
                extra[f"config{cfg}"]["cpu_baseline"] = cpu_baseline(cfg, rows=64)
        line["configs"] = extra
    if rank == 0:
        if not args.no_cpu_baseline and world == 1:
            line["cpu_baseline"] = cpu_baseline(args.config)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
