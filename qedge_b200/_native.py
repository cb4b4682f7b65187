"""ctypes binding of ``libqesample.so`` (the C ABI in ``include/qedge_sample.h``).

The library is built in-tree by ``qedge_b200.build``.  There is no fallback:
if the library cannot be loaded, every sampler call raises.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libqesample.so"

QE_ABI_VERSION = 2
QE_DTYPE_F32, QE_DTYPE_BF16, QE_DTYPE_F16 = 0, 1, 2
QE_FLAG_ALL_GREEDY, QE_FLAG_USE_TOP_P, QE_FLAG_MULTI_KERNEL = 1, 2, 4
QE_ROW_GREEDY, QE_ROW_NONFINITE, QE_ROW_GATHERED, QE_ROW_SLOW, QE_ROW_TIMEOUT = 1, 2, 4, 8, 16
STATUS_NAMES = {0: "QE_OK", -1: "QE_ERR_INVALID", -2: "QE_ERR_CUDA",
                -3: "QE_ERR_WORKSPACE", -4: "QE_ERR_UNSUPPORTED"}

# Every symbol the header declares; tests check the library exports them.
EXPORTED = ("qe_abi_version", "qe_sample_workspace_size", "qe_sample", "qe_last_error", "qe_sample_errors",
            "qe_sample_noalloc", "qe_shard_record_bytes", "qe_shard_test_bytes", "qe_shard_partial_bytes",
            "qe_shard_summarize", "qe_shard_merge", "qe_shard_test", "qe_shard_decide")
QE_NOALLOC_SCRATCH_BYTES = 32 << 20

_vp = ctypes.c_void_p


class QeSampleArgs(ctypes.Structure):
    _fields_ = [
        ("struct_size", ctypes.c_uint32),
        ("dtype", ctypes.c_int32),
        ("batch", ctypes.c_int64),
        ("vocab", ctypes.c_int64),
        ("ld", ctypes.c_int64),
        ("logits", _vp),
        ("temperatures", _vp),
        ("top_ps", _vp),
        ("top_ks", _vp),
        ("min_ps", _vp),
        ("rep_penalties", _vp),
        ("history", _vp),
        ("history_lens", _vp),
        ("history_ld", ctypes.c_int64),
        ("noise", _vp),
        ("noise_ld", ctypes.c_int64),
        ("seed", ctypes.c_uint64),
        ("seeds", _vp),
        ("step", ctypes.c_uint64),
        ("step_ptr", _vp),
        ("row_offset", ctypes.c_int64),
        ("flags", ctypes.c_uint32),
        ("wait_polls", ctypes.c_uint32),
        ("out_ids", _vp),
        ("out_probs", _vp),
        ("probs_ld", ctypes.c_int64),
        ("out_status", _vp),
        ("out_kept", _vp),
        ("out_norm", _vp),
        ("workspace", _vp),
        ("workspace_bytes", ctypes.c_size_t),
    ]


class NativeError(RuntimeError):
    pass


_lock = threading.Lock()
_lib = None


def load(path: Path | str | None = None) -> ctypes.CDLL:
    """Load the sampler library (once) and declare its signatures."""
    global _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = Path(path) if path else LIB_PATH
        if not p.exists():
            raise NativeError(f"{p} is missing: build it with `python -m qedge_b200.build`")
        lib = ctypes.CDLL(str(p))
        lib.qe_abi_version.restype = ctypes.c_int
        lib.qe_abi_version.argtypes = []
        lib.qe_sample_workspace_size.restype = ctypes.c_size_t
        lib.qe_sample_workspace_size.argtypes = [ctypes.c_int64, ctypes.c_int64]
        lib.qe_sample.restype = ctypes.c_int
        lib.qe_sample.argtypes = [ctypes.POINTER(QeSampleArgs), _vp]
        lib.qe_sample_noalloc.restype = ctypes.c_int
        lib.qe_sample_noalloc.argtypes = [ctypes.POINTER(QeSampleArgs), _vp]
        lib.qe_last_error.restype = ctypes.c_char_p
        lib.qe_last_error.argtypes = []
        lib.qe_sample_errors.restype = ctypes.c_int
        lib.qe_sample_errors.argtypes = [_vp, _vp, ctypes.POINTER(ctypes.c_uint32)]
        for name in ("qe_shard_record_bytes", "qe_shard_test_bytes", "qe_shard_partial_bytes"):
            getattr(lib, name).restype = ctypes.c_size_t
            getattr(lib, name).argtypes = []
        _a = ctypes.POINTER(QeSampleArgs)
        lib.qe_shard_summarize.restype = ctypes.c_int
        lib.qe_shard_summarize.argtypes = [_a, ctypes.c_int, ctypes.c_int, _vp, _vp]
        lib.qe_shard_merge.restype = ctypes.c_int
        lib.qe_shard_merge.argtypes = [_a, ctypes.c_int, _vp, _vp, _vp]
        lib.qe_shard_test.restype = ctypes.c_int
        lib.qe_shard_test.argtypes = [_a, ctypes.c_int, ctypes.c_int, _vp, _vp, _vp]
        lib.qe_shard_decide.restype = ctypes.c_int
        lib.qe_shard_decide.argtypes = [_a, ctypes.c_int, _vp, _vp, _vp]
        ver = lib.qe_abi_version()
        if ver != QE_ABI_VERSION:
            raise NativeError(f"libqesample ABI {ver} != expected {QE_ABI_VERSION}")
        if path is None:
            _lib = lib
        return lib


def check(rc: int, lib=None) -> None:
    if rc != 0:
        lib = lib or load()
        msg = lib.qe_last_error().decode(errors="replace")
        raise NativeError(f"{STATUS_NAMES.get(rc, rc)}: {msg}")
