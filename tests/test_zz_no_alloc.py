"""qe_sample_noalloc: sampling for callers that cannot allocate device memory.

Some hosts of this library cannot hand it a workspace: a plugin running inside
an engine that owns all device memory and exposes no allocator, or a language
binding without a device-memory API.  For them the library carries one fixed
scratch array (QE_NOALLOC_SCRATCH_BYTES).  These tests call the entry point
through the C ABI and check that it returns exactly the ids of qe_sample with
a caller workspace, on two calls in a row (the shared array keeps the previous
call's contents, which must not leak into the next result).  This file is
collected last on purpose.
"""
import ctypes
import os

import numpy as np
import pytest

from qedge_b200 import _native as N
from qedge_b200 import workloads as W


def _args(B=4, V=248_320):
    a = N.QeSampleArgs()
    a.struct_size = ctypes.sizeof(a)
    a.dtype = N.QE_DTYPE_BF16
    a.batch, a.vocab, a.ld = B, V, V
    a.logits = a.temperatures = a.out_ids = ctypes.c_void_p(0x1000)
    return a


def test_noalloc_exported_and_rejects_oversize_before_touching_the_gpu():
    lib = N.load()
    assert hasattr(lib, "qe_sample_noalloc")
    big = _args(B=1024)
    assert lib.qe_sample_workspace_size(1024, 248_320) > N.QE_NOALLOC_SCRATCH_BYTES
    assert lib.qe_sample_noalloc(ctypes.byref(big), None) == -4
    assert b"built-in scratch" in lib.qe_last_error()
    assert lib.qe_sample_noalloc(None, None) == -1


def _call(lib, fn, w, dev_tensors, out, step, ws=None, flags=0):
    import torch
    lg, temps, tps, tks, rps, hist, hlen = dev_tensors
    a = N.QeSampleArgs()
    a.struct_size = ctypes.sizeof(N.QeSampleArgs)
    a.dtype = {"bf16": N.QE_DTYPE_BF16, "f16": N.QE_DTYPE_F16, "f32": N.QE_DTYPE_F32}[w.dtype]
    a.batch, a.vocab, a.ld = w.B, w.V, lg.stride(0)
    a.logits = lg.data_ptr()
    a.temperatures = temps.data_ptr()
    a.top_ps = tps.data_ptr()
    a.top_ks = tks.data_ptr()
    if hist is not None:
        a.rep_penalties = rps.data_ptr()
        a.history = hist.data_ptr()
        a.history_lens = hlen.data_ptr()
        a.history_ld = hist.stride(0)
    a.seed = 31
    a.step = step
    a.flags = (N.QE_FLAG_USE_TOP_P if w.use_top_p else 0) | flags
    a.out_ids = out.data_ptr()
    if ws is not None:
        a.workspace = ws.data_ptr()
        a.workspace_bytes = ws.numel()
    stream = torch.cuda.current_stream().cuda_stream
    N.check(fn(ctypes.byref(a), ctypes.c_void_p(stream)), lib)
    torch.cuda.synchronize()
    return out.cpu().numpy().copy()


@pytest.mark.gpu
@pytest.mark.parametrize("path", ["stream", "multi"])
def test_noalloc_matches_workspace_entry_point_twice(path):
    import torch
    flags = N.QE_FLAG_MULTI_KERNEL if path == "multi" else 0
    lib = N.load()
    dev = torch.device("cuda", 0)
    for w in (W.config2(B=16), W.config3(B=8)):
        tensors = (W.to_device(w, dev), torch.from_numpy(w.temperatures).to(dev),
                   torch.from_numpy(w.top_ps).to(dev), torch.from_numpy(w.top_ks).to(dev),
                   torch.from_numpy(w.rep_penalties).to(dev),
                   None if w.history is None else torch.from_numpy(w.history).to(dev),
                   None if w.history_lens is None else torch.from_numpy(w.history_lens).to(dev))
        ws = torch.zeros(lib.qe_sample_workspace_size(w.B, w.V), dtype=torch.uint8, device=dev)
        out = torch.empty(w.B, dtype=torch.int64, device=dev)
        for step in (0, 1):
            want = _call(lib, lib.qe_sample, w, tensors, out, step, ws=ws, flags=flags)
            got = _call(lib, lib.qe_sample_noalloc, w, tensors, out, step, flags=flags)
            np.testing.assert_array_equal(got, want)
