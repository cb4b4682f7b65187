"""The C ABI library loads, exports every declared symbol and rejects bad
arguments on the host (no GPU needed: validation runs before any CUDA call)."""
import ctypes
import re
from pathlib import Path

import pytest

from qedge_b200 import _native as N

ROOT = Path(__file__).resolve().parents[1]


def declared_functions():
    text = (ROOT / "include" / "qedge_sample.h").read_text()
    return sorted(set(re.findall(r"^\w[\w\s\*]*?\b(qe_\w+)\s*\(", text, flags=re.M)))


def test_header_and_binding_agree():
    assert sorted(N.EXPORTED) == declared_functions()


def test_library_exports_all_symbols():
    lib = N.load()
    for name in declared_functions():
        assert hasattr(lib, name), name
    assert lib.qe_abi_version() == N.QE_ABI_VERSION


def test_struct_layout_matches_header():
    # sizeof(qe_sample_args) as compiled into the library is checked by
    # qe_sample; a mismatch is reported as QE_ERR_INVALID.
    lib = N.load()
    a = N.QeSampleArgs()
    a.struct_size = ctypes.sizeof(a) + 8
    assert lib.qe_sample(ctypes.byref(a), None) == -1
    assert b"struct_size" in lib.qe_last_error()


def _args(**kw):
    a = N.QeSampleArgs()
    a.struct_size = ctypes.sizeof(a)
    a.dtype = N.QE_DTYPE_BF16
    a.batch, a.vocab, a.ld = 4, 100, 100
    a.logits = a.temperatures = a.out_ids = ctypes.c_void_p(0x1000)
    a.workspace = ctypes.c_void_p(0x10000)
    a.workspace_bytes = 1 << 20
    for k, v in kw.items():
        setattr(a, k, v)
    return a


@pytest.mark.parametrize("kw,code", [
    (dict(vocab=0), -1),
    (dict(vocab=1 << 24), -1),
    (dict(ld=50), -1),
    (dict(dtype=7), -1),
    (dict(logits=None), -1),
    (dict(out_ids=None), -1),
    (dict(workspace_bytes=16), -3),
    (dict(workspace=None), -3),
    (dict(workspace=ctypes.c_void_p(0x10010)), -1),
    (dict(batch=-1), -1),
])
def test_invalid_arguments_rejected(kw, code):
    lib = N.load()
    assert lib.qe_sample(ctypes.byref(_args(**kw)), None) == code
    assert lib.qe_last_error()


def test_null_args_and_empty_batch():
    lib = N.load()
    assert lib.qe_sample(None, None) == -1
    assert lib.qe_sample(ctypes.byref(_args(batch=0)), None) == 0


def test_workspace_size_monotone():
    lib = N.load()
    assert lib.qe_sample_workspace_size(0, 10) == 0
    assert 0 < lib.qe_sample_workspace_size(1, 248320) <= lib.qe_sample_workspace_size(1024, 248320)


def test_missing_library_fails_loudly(tmp_path):
    with pytest.raises(N.NativeError):
        N.load(tmp_path / "nope.so")


def test_workspace_sizes_and_noalloc_capacity():
    """The workspace grows linearly with the batch, and the built-in scratch
    of qe_sample_noalloc holds 314 rows at V = 248,320 (the documented limit)."""
    from qedge_b200 import _native as N
    lib = N.load()
    V = 248_320
    w1, w2 = lib.qe_sample_workspace_size(1, V), lib.qe_sample_workspace_size(2, V)
    assert 0 < w1 < w2 and w2 - w1 < 120_000
    assert lib.qe_sample_workspace_size(314, V) <= N.QE_NOALLOC_SCRATCH_BYTES
    assert lib.qe_sample_workspace_size(315, V) > N.QE_NOALLOC_SCRATCH_BYTES
    assert lib.qe_sample_workspace_size(0, V) == 0
