"""ctypes binding of libjeffb200.so (include/jeffb200.h). Loading fails loudly when the library is missing: the
package has no CPU fallback. `call` raises on a non-zero status with the library's message."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libjeffb200.so"
HEADER = HERE.parent / "include" / "jeffb200.h"

_P = ctypes.c_void_p
_I = ctypes.c_int
_L = ctypes.c_int64



def parse_header(text: str) -> dict[str, tuple[str, str]]:
    """{entry point: (return kind, argument kinds)} from the header: "p" pointer, "i" int, "l" int64_t."""
    out: dict[str, tuple[str, str]] = {}
    for ret, name, params in re.findall(r"^\s*(int|const char\*)\s+(jb_\w+)\(([^)]*)\);", text, flags=re.M | re.S):
        kinds = ""
        for param in (x.strip() for x in params.split(",")):
            if not param or param == "void":
                continue
            kinds += "p" if "*" in param else ("l" if "int64_t" in param else "i")
        out[name] = ("s" if ret.startswith("const char") else "i", kinds)
    return out


_CT = {"p": _P, "i": _I, "l": _L}


class JbError(RuntimeError):
    """A libjeffb200 call returned a non-zero status."""


class ArgumentError(JbError, ValueError):
    """The library refused an argument before any launch (JB_EINVAL)."""


_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise ImportError(f"{LIB_PATH} is missing: build it with `python -m jeff_b200.build` (nvcc, sm_100a). The "
                          "package has no CPU fallback.")
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (ret, sig) in parse_header(HEADER.read_text()).items():
        fn = getattr(lib, name)
        fn.argtypes = [_CT[c] for c in sig]
        fn.restype = ctypes.c_char_p if ret == "s" else _I
    _lib = lib
    return lib


def header_symbols() -> list[str]:
    """Every entry point include/jeffb200.h declares."""
    return list(parse_header(HEADER.read_text()))


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_ptr(stream: torch.cuda.Stream | None = None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


# Kernel launches each entry point makes (the product with LoRA makes two: shrink, then the fused GEMM); counted
# by `call` so a caller can report how many of this library's kernels a recorded pass launches.
_NO_LAUNCH = {"jb_abi_version", "jb_last_error", "jb_device_status"}
launches = 0


def call(name: str, *args) -> None:
    global launches
    lib = load()
    if name not in _NO_LAUNCH:
        products = ("jb_int4_lora_product", "jb_int4_lora_product_static", "jb_int4_lora_product_split")
        launches += 2 if (name in products and args[11]) else 1   # args[11]: rank
    status = getattr(lib, name)(*args)
    if status != 0:
        msg = lib.jb_last_error().decode(errors="replace")
        if status == -1:
            raise ArgumentError(f"{name}: {msg}")
        raise JbError(f"{name} failed ({status}): {msg}")


def device_status(reset: bool = True) -> int:
    """The device status word kernels set when a bounded wait gave up (0: none). Synchronises the stream."""
    out = ctypes.c_int(0)
    call("jb_device_status", ctypes.addressof(out), 1 if reset else 0, stream_ptr())
    return out.value
