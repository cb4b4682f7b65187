"""Generate ``golden.json`` by running QEdge's own sampler module.

Run in a container where the reference checkout is mounted (its path is
given with ``--reference``); the GPU box does not have it, which is why the
results are committed.  The reference's ``src/compute/sampler.py`` is loaded
file-by-file with ``importlib`` (the pattern of the reference's
``tests/test_host.py:13-18``), so none of its accelerator imports run.

Shared-noise adapter: while the reference runs, ``torch.multinomial(w, 1)``
is replaced by ``argmax(w / E')`` where ``E'`` is the case's Exp(1) tensor in
the tensor's own index order (gathered through the indices of the preceding
``torch.sort`` in the top-p path), and ``torch.sort`` is made stable.  The
script also checks that the default (unstable) sort gives the same ids and
records the outcome.

Usage: python tests/golden/make_golden.py --reference <path-to-QEdge>
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from tests.golden import cases as C  # noqa: E402


class SharedNoise:
    def __init__(self, noise: torch.Tensor, stable: bool = True):
        self.noise = noise
        self.stable = stable
        self.last_idx = None

    def __enter__(self):
        self._sort, self._mult = torch.sort, torch.multinomial

        def sort(inp, *a, **k):
            if self.stable:
                k["stable"] = True
            vals, idx = self._sort(inp, *a, **k)
            self.last_idx = idx
            return vals, idx

        def multinomial(w, n, *a, **k):
            assert n == 1
            e = self.noise if self.last_idx is None else self.noise.gather(1, self.last_idx)
            return torch.argmax(w / e, dim=1, keepdim=True)

        torch.sort, torch.multinomial = sort, multinomial
        return self

    def __exit__(self, *exc):
        torch.sort, torch.multinomial = self._sort, self._mult


def load_reference_sampler(ref: Path):
    spec = importlib.util.spec_from_file_location("qedge_ref_sampler", ref / "src/compute/sampler.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.BatchSampler()


def run_case(sampler, w, noise, stable=True):
    x = C.penalised_f32(w)
    if w.history is None and w.dtype == "bf16":
        logits = torch.from_numpy(w.logits_bits.view(np.int16).copy()).view(torch.bfloat16)
    else:
        logits = torch.from_numpy(x)
    temps = torch.from_numpy(w.temperatures.copy())
    top_ps = torch.from_numpy(w.top_ps.copy())
    all_greedy = bool(np.all(w.temperatures <= 1e-5))
    with SharedNoise(torch.from_numpy(noise), stable=stable):
        ids = sampler(logits, temps, top_ps, all_greedy=all_greedy, use_top_p=w.use_top_p)
    return ids.numpy().astype(np.int64), all_greedy


def check_multinomial_is_race():
    """torch.multinomial(p, 1) == argmax(p / Exp(1)) on the same generator."""
    g = torch.Generator().manual_seed(0)
    p = torch.softmax(torch.randn(4, 248_320, generator=g) * 2, dim=-1)
    torch.manual_seed(11)
    a = torch.multinomial(p, 1).squeeze(1)
    torch.manual_seed(11)
    q = torch.empty_like(p).exponential_(1)
    b = torch.argmax(p / q, dim=-1)
    return bool(torch.equal(a, b))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, type=Path)
    ap.add_argument("--out", type=Path, default=Path(__file__).with_name("golden.json"))
    args = ap.parse_args()
    sampler = load_reference_sampler(args.reference)
    out = {"torch": torch.__version__, "numpy": np.__version__,
           "multinomial_is_exponential_race": check_multinomial_is_race(), "cases": {}}
    for name, (w, spec) in C.build_cases().items():
        noise = C.make_noise(spec, w.B, w.V)
        ids, all_greedy = run_case(sampler, w, noise, stable=True)
        ids_unstable, _ = run_case(sampler, w, noise, stable=False)
        out["cases"][name] = {
            "B": w.B, "V": w.V, "dtype": w.dtype, "noise": list(spec),
            "use_top_p": w.use_top_p, "all_greedy": all_greedy,
            "logits_sha256": C.digest(w.logits_bits), "noise_sha256": C.digest(noise),
            "ids": ids.tolist(), "unstable_sort_same_ids": bool(np.array_equal(ids, ids_unstable)),
        }
        print(name, ids[:8].tolist(), "unstable-same:", out["cases"][name]["unstable_sort_same_ids"])
    args.out.write_text(json.dumps(out, indent=1) + "\n")


if __name__ == "__main__":
    main()
