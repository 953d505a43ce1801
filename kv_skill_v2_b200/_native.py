"""ctypes binding of libxencb.so, the C ABI declared in include/xencb.h.

The library is built in-tree (kv_skill_v2_b200/csrc/build.py). Loading it needs no GPU; calling its compute
entry points needs a CUDA device. There is no fallback: if the library is missing, every product call
raises, naming the build command.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().with_name("libxencb.so")

# element type codes, status codes and flags (include/xencb.h)
F32, F16, BF16 = 0, 1, 2
OK, EINVAL, ECUDA, ENOTSUP = 0, 1, 2, 3
DEV_TIMEOUT, DEV_CLAMPED, DEV_BADPAGE = 1, 2, 4
PIN_RMS, PIN_L2 = 1, 2
NOALLOC_SCRATCH_BYTES = 16 << 20
ABI_VERSION = 6

_p, _i, _i64, _f, _sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t

# name -> (restype, argtypes); mirrors include/xencb.h one to one
SIGNATURES: dict = {
    "xencb_abi_version": (_i, []),
    "xencb_last_error": (ctypes.c_char_p, []),
    "xencb_launch_count": (ctypes.c_ulonglong, []),
    "xencb_device_status": (_i, [_p, _i, ctypes.POINTER(ctypes.c_uint)]),
    "xencb_project_in_workspace": (_sz, [_i64, _i, _i]),
    "xencb_project_in": (_i, [_p, _i, _i64, _i, _p, _p, _p, _i, _i, _p, _f, _p, _p, _p, _i, _f, _p, _p, _p, _p,
                              _p, _sz, _p]),
    "xencb_project_in_route": (_i, [_p, _i, _i64, _i, _p, _p, _p, _i, _i, _p, _f, _p, _p, _p, _i, _f, _p, _p, _p,
                                    _p, _p, _i, _p, _i64, _i64, _f, _i, _p, _p, _p, _p, _p, _p, _sz, _p]),
    "xencb_project_in_route_lse": (_i, [_p, _i, _i64, _i, _p, _p, _p, _i, _i, _p, _f, _p, _f, _p, _p, _p, _p, _i, _p,
                                        _i64, _i64, _f, _p, _p, _p, _sz, _p]),
    "xencb_rms_norm": (_i, [_p, _i, _i64, _i, _f, _p, _p]),
    "xencb_route_k": (_i, [_i, _i]),
    "xencb_route": (_i, [_p, _i64, _i, _p, _i, _p, _i64, _i64, _f, _i, _p, _p, _p, _p, _p, _p]),
    "xencb_read_decode_workspace": (_sz, [_i64, _i, _i, _i, _i]),
    "xencb_read_decode_sparse_workspace": (_sz, [_i64, _i, _i, _i, _i]),
    "xencb_read_decode": (_i, [_p, _i64, _i, _p, _p, _i, _i64, _i64, _i, _p, _p, _i, _i64, _i64, _p, _p, _i, _f,
                               _i, _p, _p, _sz, _p]),
    "xencb_read_decode_sparse": (_i, [_p, _i64, _i, _p, _p, _i, _i64, _i64, _i, _p, _p, _i, _i64, _i64, _p, _p, _i, _f,
                               _i, _p, _p, _sz, _p]),
    "xencb_read_decode_noalloc": (_i, [_p, _i64, _i, _p, _i, _i64, _i64, _i, _p, _p, _i, _i64, _i64, _p, _p, _i,
                                       _f, _i, _p, _p]),
    "xencb_read_attn": (_i, [_p, _i64, _i, _p, _i, _i64, _i64, _i, _p, _p, _i, _i64, _i64, _p, _p, _i, _f, _i, _p,
                             _p]),
    "xencb_read_forced_workspace": (_sz, [_i, _i]),
    "xencb_read_forced": (_i, [_p, _i, _p, _p, _i, _i64, _i64, _i, _p, _p, _i, _p, _i64, _i, _p, _p, _p, _sz, _p]),
    "xencb_read_multi_workspace": (_sz, [_i64, _i64, _i, _i, _i, _i]),
    "xencb_read_multi": (_i, [_p, _i64, _i, _p, _p, _i, _i64, _i64, _i, _p, _p, _i, _p, _i64, _i64, _p, _f, _i, _p,
                              _p, _sz, _p]),
    "xencb_read_prefill_workspace": (_sz, [_i64, _i, _i, _i]),
    "xencb_read_prefill": (_i, [_p, _i64, _i, _p, _p, _i, _i64, _i64, _i, _p, _p, _i, _p, _i64, _i64, _p, _f, _i,
                                _p, _p, _sz, _p]),
    "xencb_route_lse": (_i, [_p, _i64, _i, _p, _i, _p, _i64, _i64, _f, _p, _p, _p]),
    "xencb_shard_merge": (_i, [_p, _i, _i64, _i, _p, _p]),
    "xencb_exch_bytes": (_sz, [_i, _i64]),
    "xencb_exch_alloc": (_i, [_sz, ctypes.POINTER(ctypes.c_void_p), _p]),
    "xencb_exch_open": (_i, [_p, ctypes.POINTER(ctypes.c_void_p)]),
    "xencb_exch_close": (_i, [_p]),
    "xencb_exch_free": (_i, [_p]),
    "xencb_shard_push": (_i, [_p, _i64, _p, _i, _i, _p, _p]),
    "xencb_shard_merge_wait": (_i, [_p, _i, _i64, _i, _p, _p, _p]),
    "xencb_project_out_workspace": (_sz, [_i64, _i, _i]),
    "xencb_project_out": (_i, [_p, _i64, _i, _p, _p, _p, _i, _f, _p, _p, _p, _f, _p, _p, _p, _i, _p, _p, _p, _p,
                               _sz, _p]),
    "xencb_selector_weights": (_i, [_p, _i64, _i, _i, _i, _p, _p]),
    "xencb_selector_logits": (_i, [_p, _i, _i64, _i, _p, _p, _i, _i, _f, _p, _p]),
    "xencb_selector_apply": (_i, [_p, _i, _p, _i, _i64, _i, _p, _i, _i, _f, _p, _p]),
    "xencb_summaries": (_i, [_p, _i, _i64, _i64, _i, _p, _p, _i64, _i, _i, _p, _p]),
    "xencb_library_build_workspace": (_sz, [_i, _i, _i]),
    "xencb_library_build": (_i, [_p, _i, _i64, _p, _i, _i, _p, _p, _i, _i64, _i64, _i, _p, _p, _p, _p, _sz, _p]),
    "xencb_select_scores": (_i, [_p, _i64, _i, _i, _i, _i, _p, _i, _i64, _i, _i, _p, _p, _i64, _i64, _i, _i, _p, _p]),
    "xencb_select_topk": (_i, [_p, _i64, _i, _i, _p, _p, _p]),
    "xencb_topk_read": (_i, [_p, _i64, _i, _p, _p, _i, _i64, _i64, _i, _p, _i, _i64, _p, _i, _i, _f, _i, _p, _p, _p]),
    "xencb_wait_selftest": (_i, [ctypes.c_longlong, _p, _p]),
    "xencb_read_kernel_events": (_i, [_p, _p]),
    "xencb_weights_prep_bytes": (_sz, [_i, _i]),
    "xencb_weights_prep": (_i, [_p, _i, _i, _p, _sz, _p]),
}

_lib = None
_lock = threading.Lock()


class NativeMissing(RuntimeError):
    """libxencb.so is not built or cannot be loaded."""


def lib() -> ctypes.CDLL:
    """The loaded library (loaded once, thread-safe)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not LIB_PATH.exists():
                    raise NativeMissing(
                        f"{LIB_PATH.name} is not built; run `python -m kv_skill_v2_b200.csrc.build` "
                        "(the Library read has no CPU path)")
                try:
                    L = ctypes.CDLL(str(LIB_PATH))
                except OSError as e:  # pragma: no cover - depends on the host
                    raise NativeMissing(f"cannot load {LIB_PATH}: {e}") from e
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(L, name)
                    fn.restype, fn.argtypes = res, args
                if L.xencb_abi_version() != ABI_VERSION:
                    raise NativeMissing(f"{LIB_PATH.name} ABI {L.xencb_abi_version()} != {ABI_VERSION}; rebuild")
                _lib = L
    return _lib


def check(rc: int, what: str = "") -> None:
    """Raise the Python exception for a non-zero xencb status (ValueError for XENCB_EINVAL)."""
    if rc == OK:
        return
    msg = lib().xencb_last_error().decode(errors="replace")
    text = f"xencb{': ' + what if what else ''}: {msg}"
    if rc == EINVAL:
        raise ValueError(text)
    if rc == ENOTSUP:
        raise NotImplementedError(text)
    raise RuntimeError(text)


def call(name: str, *args) -> int:
    """Call entry point `name` and raise on a non-zero status."""
    rc = getattr(lib(), name)(*args)
    check(rc, name)
    return rc


def exported_symbols() -> list:
    return sorted(SIGNATURES)


def launch_count() -> int:
    """Kernels launched (or captured into a CUDA graph) by libxencb.so in this process so far."""
    return int(lib().xencb_launch_count())
