"""Loader of the sm_100a C-ABI library (``include/dsv41_b200.h``) through ctypes.

The library is built in-tree (``sgl_amd_mono_b200/deepseek_v41/sm100a/build.py``). There is
no fallback: a missing or unloadable library raises ``ExtError`` at the first call.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parents[1] / "deepseek_v41" / "sm100a" / "libdsv41_b200.so"
STATUS = {0: "ok", -1: "invalid argument", -2: "CUDA launch failed", -3: "scratch too small",
          -4: "device guard fired"}

_lock = threading.Lock()
_lib = None


class ExtError(RuntimeError):
    pass


def lib() -> ctypes.CDLL:
    """The loaded library (loaded once per process)."""
    global _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise ExtError(
                    f"{LIB_PATH} is not built; run python -m sgl_amd_mono_b200.deepseek_v41.sm100a.build"
                )
            _lib = ctypes.CDLL(str(LIB_PATH))
        return _lib


def struct(name: str, fields: list[str]) -> type:
    """A ctypes mirror of a header struct whose fields are all int64_t."""
    return type(name, (ctypes.Structure,), {"_fields_": [(f, ctypes.c_int64) for f in fields]})


def check(rc: int, what: str) -> int:
    if rc < 0:
        raise ExtError(f"{what}: {STATUS.get(rc, rc)}")
    return rc


def call(fn: str, args: ctypes.Structure, stream: int) -> None:
    """``fn(&args, stream)``, raising on a negative status."""
    f = getattr(lib(), fn)
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
    check(f(ctypes.byref(args), ctypes.c_void_p(stream)), fn)


def query(fn: str, args: ctypes.Structure) -> int:
    """An int64 query ``fn(&args)`` (scratch sizes), raising on a negative status."""
    f = getattr(lib(), fn)
    f.restype = ctypes.c_int64
    f.argtypes = [ctypes.c_void_p]
    return check(int(f(ctypes.byref(args))), fn)


def launch_count() -> int:
    """Kernels the library has launched in this process."""
    f = lib().dsv41_launch_count
    f.restype = ctypes.c_int64
    f.argtypes = []
    return int(f())


def set_option(name: str, value: int) -> None:
    """``dsv41_set_option``: a launch-sequence tuning switch ("attn_tc", "attn_pair",
    "dense_min_m", "pdl"), raising on an unknown name or value."""
    f = lib().dsv41_set_option
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_char_p, ctypes.c_int64]
    check(f(name.encode(), int(value)), f"dsv41_set_option({name!r}, {value})")
