"""ctypes binding of the C ABI in include/proteus_atlas.h (libproteus_atlas.so, built in-tree).

The library is the only compute path: there is no CPU or torch fallback, and importing a kernel
wrapper on a machine without the built library or without a CUDA device raises.
"""
from __future__ import annotations

import ctypes as C
import os
import re
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libproteus_atlas.so"

ATLAS_F32, ATLAS_BF16, ATLAS_F16 = 0, 1, 2
DTYPE_CODE = {torch.float32: ATLAS_F32, torch.bfloat16: ATLAS_BF16, torch.float16: ATLAS_F16}

_P = C.c_void_p
_I = C.c_int
_L = C.c_int64

HEADER = Path(__file__).resolve().parents[1] / "include" / "proteus_atlas.h"


def parse_header(path: Path = HEADER) -> dict:
    """name -> (restype, argtypes) for every function declared in include/proteus_atlas.h.

    Pointers map to c_void_p, int64_t to c_int64, int to c_int, double to c_double, so the binding
    cannot drift from the header."""
    text = re.sub(r"/\*.*?\*/", " ", path.read_text(), flags=re.S)
    sigs = {}
    for m in re.finditer(r"(const\s+char\s*\*|int64_t|int)\s+(atlas_\w+)\s*\(([^)]*)\)\s*;", text):
        ret, name, params = m.groups()
        rtype = C.c_char_p if "char" in ret else (_L if ret == "int64_t" else _I)
        args = []
        for prm in params.split(","):
            prm = prm.strip()
            if not prm or prm == "void":
                continue
            if "*" in prm:
                args.append(_P)
            elif prm.startswith("int64_t"):
                args.append(_L)
            elif prm.startswith("int "):
                args.append(_I)
            elif prm.startswith("double "):
                args.append(C.c_double)
            else:
                raise ValueError(f"unparsed parameter {prm!r} of {name}")
        sigs[name] = (rtype, args)
    return sigs


SIGNATURES = parse_header() if HEADER.exists() else {}

_lib = None


class AtlasKernelError(RuntimeError):
    pass


def load(path: str | os.PathLike | None = None):
    """Load the kernel library (once). Raises if it is missing: there is no fallback path."""
    global _lib
    if _lib is not None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise AtlasKernelError(f"{p} is missing: build it with `python -m proteus_b200.build` (needs nvcc)")
    lib = C.CDLL(str(p))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


# kernels launched per call (predicated kernels that exit early on the device still count)
_KERNELS = {"atlas_grouped_merge": 6, "atlas_last_error": 0, "atlas_abi_version": 0, "atlas_device_status": 0,
            "atlas_device_status_set": 0, "atlas_stats_enrich_supported": 0}
LAUNCHES = {"count": 0}


_KERNELS.update({"atlas_ctx_rows": 4, "atlas_ctx_annotations": 2})


def _n_kernels(name: str, args) -> int:
    if name == "atlas_dense_select":
        return 3  # row-major count (+ keys in key order), row-major emit, hard columns
    if name == "atlas_admit":  # candidates, plus the bulk-row kernel when there are bulk rows
        return 2 if (args[6] and args[20]) else 1
    if name.endswith("_bytes") or name.endswith("_i32"):
        return 0
    return _KERNELS.get(name, 1)


def call(name: str, *args):
    """Call an entry point and raise AtlasKernelError on a non-zero status."""
    lib = load()
    LAUNCHES["count"] += _n_kernels(name, args)
    rc = getattr(lib, name)(*args)
    if rc != 0:
        msg = lib.atlas_last_error().decode(errors="replace")
        raise AtlasKernelError(f"{name} failed (status {rc}): {msg}")
    return rc


def ptr(t):
    """Device pointer of a tensor (None -> NULL)."""
    if t is None:
        return None
    return t.data_ptr()


def stream_ptr(device=None):
    return torch.cuda.current_stream(device).cuda_stream


def dtype_code(dt: torch.dtype) -> int:
    if dt not in DTYPE_CODE:
        raise TypeError(f"unsupported activation dtype {dt} (bf16, fp16, fp32)")
    return DTYPE_CODE[dt]


def require_cuda(t: torch.Tensor, what: str):
    if not t.is_cuda:
        raise AtlasKernelError(f"{what} must be a CUDA tensor: the B200 kernels are the only compute path")
