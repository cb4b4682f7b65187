"""``QESampler``: drop-in replacement for QEdge's ``BatchSampler``.

Reference interface (``src/compute/sampler.py:25-28``)::

    BatchSampler.forward(logits, temperatures, top_ps, *,
                         all_greedy=False, use_top_p=False) -> LongTensor[B]

``QESampler.forward`` keeps that signature (same positional arguments, same
keyword flags, same int64 output on ``logits.device``) and adds optional
keywords for the fields the reference's ``SamplingParams``/``Batch`` carry
but its sampler ignores (``top_ks``, ``min_ps``, ``src/data/batch.py:59-60``),
the repetition penalty, the Philox noise key (seed or per-row seeds, step)
and a parity mode that consumes a caller-supplied Exp(1) noise tensor.  Work
runs on the current CUDA stream with no host synchronisation; every call goes
through ``libqesample.so`` and raises if it is missing.
"""
from __future__ import annotations

import ctypes

import torch
from torch import nn

from . import _native as N

_DTYPES = {torch.float32: N.QE_DTYPE_F32, torch.bfloat16: N.QE_DTYPE_BF16,
           torch.float16: N.QE_DTYPE_F16}


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _vec(t, dtype, B, device, name):
    if t is None:
        return None
    if not isinstance(t, torch.Tensor):
        t = torch.as_tensor(t)
    if t.device != device or t.dtype != dtype or not t.is_contiguous():
        t = t.to(device=device, dtype=dtype).contiguous()
    if t.numel() < B:
        raise ValueError(f"{name} has {t.numel()} entries for {B} rows")
    return t


class QESampler(nn.Module):
    """Batch greedy / temperature / top-k / top-p sampler on sm_100a.

    ``seed`` keys the Philox noise stream; each call without an explicit
    ``step`` uses the next value of an internal step counter, so repeated
    calls draw fresh noise and ``(seed, step, row)`` always reproduces the
    same token.
    """

    PATHS = {"stream": 0, "multi": N.QE_FLAG_MULTI_KERNEL}

    def __init__(self, seed: int = 0, path: str = "stream") -> None:
        super().__init__()
        if path not in self.PATHS:
            raise ValueError(f"path must be one of {sorted(self.PATHS)}")
        self.seed = int(seed) & ((1 << 64) - 1)
        self.step = 0
        self.path = path
        self._ws: dict[int, torch.Tensor] = {}
        self._lib = N.load()

    def workspace(self, batch: int, vocab: int, device: torch.device) -> torch.Tensor:
        need = int(self._lib.qe_sample_workspace_size(batch, vocab))
        key = device.index if device.index is not None else torch.cuda.current_device()
        ws = self._ws.get(key)
        if ws is None or ws.numel() < need:
            ws = torch.empty(max(need, 256), dtype=torch.uint8, device=device)
            self._ws[key] = ws
        return ws

    def device_errors(self, device=None) -> int:
        """Error bits the last call on ``device`` left on the GPU (4: a race
        found no candidate; that row's id is -1).  Waits for the current
        stream."""
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        key = dev.index if dev.index is not None else torch.cuda.current_device()
        ws = self._ws.get(key)
        if ws is None:
            return 0
        flags = ctypes.c_uint32(0)
        stream = torch.cuda.current_stream(dev).cuda_stream
        N.check(self._lib.qe_sample_errors(ctypes.c_void_p(ws.data_ptr()), ctypes.c_void_p(stream),
                                           ctypes.byref(flags)), self._lib)
        return int(flags.value)

    def check(self, device=None) -> None:
        """Raise if the last call on ``device`` reported a device-side error."""
        bits = self.device_errors(device)
        if bits:
            raise N.NativeError(f"sampler kernel reported device error bits {bits:#x} "
                                f"(4: a race found no candidate; affected rows have id -1)")

    @torch.no_grad()
    def forward(self, logits: torch.Tensor, temperatures: torch.Tensor,
                top_ps: torch.Tensor | None, *, all_greedy: bool = False,
                use_top_p: bool = False, top_ks: torch.Tensor | None = None,
                min_ps: torch.Tensor | None = None,
                rep_penalties: torch.Tensor | None = None,
                history: torch.Tensor | None = None,
                history_lens: torch.Tensor | None = None,
                seed: int | None = None, seeds: torch.Tensor | None = None,
                step: int | None = None,
                step_tensor: torch.Tensor | None = None,
                noise: torch.Tensor | None = None, row_offset: int = 0,
                out_probs: torch.Tensor | None = None,
                out_status: torch.Tensor | None = None,
                out_kept: torch.Tensor | None = None,
                out_norm: torch.Tensor | None = None,
                wait_polls: int = 0) -> torch.Tensor:
        if logits.dim() != 2:
            raise ValueError("logits must be [B, V]")
        if not logits.is_cuda:
            raise ValueError("QESampler runs on CUDA tensors only")
        if logits.dtype not in _DTYPES:
            raise TypeError(f"unsupported logits dtype {logits.dtype}")
        B, V = logits.shape
        dev = logits.device
        out = torch.empty(B, dtype=torch.int64, device=dev)
        if B == 0:
            return out
        if logits.stride(1) != 1 or (B > 1 and logits.stride(0) < V):
            logits = logits.contiguous()
        temps = _vec(temperatures, torch.float32, B, dev, "temperatures")
        tps = _vec(top_ps, torch.float32, B, dev, "top_ps")
        tks = _vec(top_ks, torch.int32, B, dev, "top_ks")
        mps = _vec(min_ps, torch.float32, B, dev, "min_ps")
        sds = _vec(seeds, torch.int64, B, dev, "seeds")
        rps = _vec(rep_penalties, torch.float32, B, dev, "rep_penalties")
        hist = hlen = None
        if history is not None and rps is not None:
            hist = history.to(device=dev, dtype=torch.int32)
            if hist.dim() != 2 or hist.shape[0] < B:
                raise ValueError("history must be [B, H]")
            if hist.stride(1) != 1:
                hist = hist.contiguous()
            hlen = _vec(history_lens, torch.int32, B, dev, "history_lens")
        if noise is not None:
            if noise.shape[0] < B or noise.shape[1] < V or noise.dtype != torch.float32:
                raise ValueError("noise must be float32 [B, V]")
            if noise.device != dev or noise.stride(1) != 1:
                noise = noise.to(dev).contiguous()
        if out_probs is not None and (out_probs.dtype != torch.float32 or out_probs.stride(1) != 1
                                      or out_probs.shape[0] < B or out_probs.shape[1] < V):
            raise ValueError("out_probs must be float32 [B, V] with unit column stride")
        for name, t, dt in (("out_kept", out_kept, torch.int64), ("out_norm", out_norm, torch.float64),
                            ("out_status", out_status, torch.int32)):
            if t is not None and (t.dtype != dt or not t.is_cuda or t.numel() < B or not t.is_contiguous()):
                raise ValueError(f"{name} must be a contiguous CUDA {dt} tensor with >= {B} entries")
        if step_tensor is not None and (step_tensor.dtype not in (torch.int64, torch.uint64)
                                        or not step_tensor.is_cuda):
            raise ValueError("step_tensor must be a CUDA int64 scalar")
        if step is None and step_tensor is None:
            step = self.step
            self.step += 1
        ws = self.workspace(B, V, dev)
        a = N.QeSampleArgs()
        a.struct_size = ctypes.sizeof(N.QeSampleArgs)
        a.dtype = _DTYPES[logits.dtype]
        a.batch, a.vocab = B, V
        a.ld = logits.stride(0) if B > 1 else V
        a.logits = _ptr(logits)
        a.temperatures = _ptr(temps)
        a.top_ps = _ptr(tps)
        a.top_ks = _ptr(tks)
        a.min_ps = _ptr(mps)
        a.rep_penalties = _ptr(rps)
        a.history = _ptr(hist)
        a.history_lens = _ptr(hlen)
        a.history_ld = hist.stride(0) if hist is not None else 0
        a.noise = _ptr(noise)
        a.noise_ld = noise.stride(0) if noise is not None else 0
        a.seed = (self.seed if seed is None else int(seed)) & ((1 << 64) - 1)
        a.seeds = _ptr(sds)
        a.step = int(step or 0) & ((1 << 64) - 1)
        a.step_ptr = _ptr(step_tensor)
        a.row_offset = int(row_offset)
        a.flags = ((N.QE_FLAG_ALL_GREEDY if all_greedy else 0) | (N.QE_FLAG_USE_TOP_P if use_top_p else 0)
                   | self.PATHS[self.path])
        a.wait_polls = int(wait_polls)
        a.out_ids = _ptr(out)
        a.out_probs = _ptr(out_probs)
        a.probs_ld = out_probs.stride(0) if out_probs is not None else 0
        a.out_status = _ptr(out_status)
        a.out_kept = _ptr(out_kept)
        a.out_norm = _ptr(out_norm)
        a.workspace = _ptr(ws)
        a.workspace_bytes = ws.numel()
        stream = torch.cuda.current_stream(dev).cuda_stream
        N.check(self._lib.qe_sample(ctypes.byref(a), ctypes.c_void_p(stream)), self._lib)
        return out
