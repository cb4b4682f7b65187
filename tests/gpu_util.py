"""Helpers for the GPU tests: move a workload to the device and sample it
through the C ABI (QESampler -> libqesample.so)."""
from __future__ import annotations

import numpy as np
import torch

from qedge_b200 import workloads as W

TORCH_DT = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}


def device_logits(w: W.Workload, dev="cuda") -> torch.Tensor:
    return W.to_device(w, dev)


def run(sampler, w: W.Workload, noise=None, *, seed=None, step=None, top_k=True,
        all_greedy=None, out_probs=None, out_status=None, logits=None, **extra):
    dev = "cuda"
    lg = device_logits(w, dev) if logits is None else logits
    kw = {}
    if top_k:
        kw["top_ks"] = torch.from_numpy(w.top_ks.astype(np.int32)).to(dev)
    if w.history is not None:
        kw["rep_penalties"] = torch.from_numpy(w.rep_penalties).to(dev)
        kw["history"] = torch.from_numpy(w.history).to(dev)
        kw["history_lens"] = torch.from_numpy(w.history_lens).to(dev)
    if noise is not None:
        kw["noise"] = torch.from_numpy(noise).to(dev)
    if all_greedy is None:
        all_greedy = bool(np.all(w.temperatures <= 1e-5))
    ids = sampler(lg, torch.from_numpy(w.temperatures).to(dev), torch.from_numpy(w.top_ps).to(dev),
                  all_greedy=all_greedy, use_top_p=w.use_top_p, seed=seed, step=step,
                  out_probs=out_probs, out_status=out_status, **kw, **extra)
    torch.cuda.synchronize()
    return ids.cpu().numpy()
