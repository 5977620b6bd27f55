"""ctypes binding of libekv_b200.so (include/ekv_kernels.h, include/ekv_vmm.h).

The library is the only compute path: nothing here falls back to PyTorch or
to the CPU.  If the shared object is missing, every kernel call raises.
"""

from __future__ import annotations

import ctypes as ct
import functools
import os
from pathlib import Path

import torch

LIBRARY_PATH = Path(__file__).resolve().parent / "lib" / "libekv_b200.so"
MAX_PLANES = 256  # EKV_MAX_PLANES
MAX_LAYERS = 128  # EKV_MAX_LAYERS
SHARED_INLINE_MAX = 512  # EKV_SHARED_INLINE_MAX
SHADOW_MAX_LAYERS = 128  # EKV_SHADOW_MAX_LAYERS

_p = ct.c_void_p
_i32 = ct.c_int
_i64 = ct.c_int64
_u64p = ct.POINTER(ct.c_uint64)
_i64p = ct.POINTER(ct.c_int64)

# name -> argtypes (every kernel entry point returns int).
_KERNELS = {
    "ekv_resolve_resident": [
        _p, _i32, _i64, _i64, _i64,
        _p, _i32, _i64, _i64,
        _p, _i32, _i64,
        _p, _i32, _i64,
        _p, _i32, _i64,
        _p, _i32, _i64, _i64,
        _p, _i64, _i64,
        _i64, _i32, _p,
    ],
    "ekv_lookup_slots": [
        _p, _i32, _i64, _i64,
        _p, _i32, _i64,
        _p, _i32,
        _i64, _i64,
        _p, _i64,
        _p, _i64,
        _p, _i64,
        _p,
        _i32, _p,
    ],
    "ekv_gather_rows": [
        _p, _p, _i64,
        _p, _i32, _p, _i32, _p, _i32, _p, _i32, _p, _i32,
        _i64, _i64, _i64, _i64, _i64, _i64,
        _i32, _i32, _p,
    ],
    "ekv_gather_rows_planes": [
        _u64p, _u64p, _i32, _i64,
        _p, _i32, _p, _i32, _p, _i32, _p, _i32, _p, _i32,
        _i64, _i64, _i64, _i64, _i64, _i64,
        _i32, _i32, _p,
    ],
    "ekv_lookup_gather_planes": [
        _u64p, _u64p, _i32, _i64,
        _p, _i32, _p, _i32, _p, _i32, _p, _i32, _i64,
        _i64, _i64, _i64, _i64, _i64,
        _p, _p,
        _i32, _i32, _p,
    ],
    "ekv_compact_misses": [
        _p, _i64, _p, _i32, _i64,
        _i64, _i64,
        _p, _i64, _p,
        _i32, _p,
    ],
    "ekv_gather_layers": [
        _u64p, _u64p, _i32, _i32, _i64,
        _u64p, _i32, _p, _i32, _p, _i32, _u64p, _i32, _p, _i32,
        _i64, _i64, _i64, _i64, _i64, _i64,
        _i32, _i32, _p,
    ],
    "ekv_pack_rows": [
        _u64p, _i32, _i64,
        _p, _p, _i32, _i64,
        _p, _i32,
        _p, _i64, _i64,
        _i32, _p,
    ],
    "ekv_unpack_rows": [
        _u64p, _i32, _i64,
        _p, _p, _i32, _i64,
        _p, _i32,
        _p, _i64, _i64,
        _i32, _p,
    ],
    "ekv_pack_rows_staged": [
        _u64p, _i32, _i64,
        _p, _p, _i32, _i64,
        _i64p, _i64,
        _p, _i64,
        _p, _i64,
        _i32, _p, _p,
    ],
    "ekv_unpack_rows_staged": [
        _u64p, _i32, _i64,
        _p, _p, _i32, _i64,
        _i64p, _i64,
        _p, _i64,
        _p, _i64,
        _i32, _p, _p,
    ],
    "ekv_pack_rows_staged_noalloc": [
        _u64p, _i32, _i64,
        _p, _p, _i32, _i64,
        _i64p, _i64,
        _p, _i64,
        _i32, _p, _p,
    ],
    "ekv_swap_select": [
        _p, _i64, _i64,
        _p, _i64, _i64,
        _p,
        _p, _i64, _i64,
        _p, _i64, _p,
        _p, _i64,
        _i64, _i32, _p,
    ],
    "ekv_promote_rows": [
        _u64p, _u64p, _i32, _i64,
        _i64, _i64, _i64,
        _p, _i64, _p,
        _p, _i64,
        _i64, _i64, _i32, _p,
    ],
    "ekv_chunk_counts": [
        _p, _i32, _i64,
        _i64p, _i64p, _i32,
        _i64, _i64,
        _p, _i64, _i32, _p,
        _i32, _p,
    ],
    "ekv_freeable_bitmap": [_p, _p, _p, _i64, _p, _i32, _p],
    "ekv_bitmap_and": [_p, _i32, _i64, _p, _i32, _p],
    "ekv_freeable_and_peers": [_p, _p, _p, _p, _i64, _u64p, _i32, _i32, ct.c_uint32, ct.c_uint32,
                               _p, _p, _p, _i32, _p],
    "ekv_resolve_shared_blocks": [
        _p, _i32, _i64, _i64, _i64, _i64,
        _p, _i64, _p, _i64,
        _p, _i32, _i64, _i64,
        _p, _i32, _i64, _i64, _i64, _i64,
        _p, _i32, _i64, _i64,
        _i32, _p, _p, _p, _i32, _i32, _p,
    ],
    "ekv_shadow_check": [
        _p, _i32, _i64, _i64, _i64, _i64,
        _p, _i32, _i64, _p, _i32, _i64,
        _p, _i32, _i64, _i64, _i64,
        _p, _i64, _i64, _p, _i64,
        _p, _p, _i64, _i64, _i64,
        _p, _p, _p, _i64,
        _i64, _i64, _i64, _i64,
        _i64, _i64, _p, _p, _p,
        _i32, _p,
    ],
    "ekv_shadow_check_complete": [
        _p, _i32, _p, _i32, _i64,
        _i64, _i64, _i64, _p, _i64,
        _u64p, _u64p, _u64p, _u64p,
        _u64p, _i32, _i64, _i64,
        _i64, _i64, _i64, _i64, _p,
        _i32, _p,
    ],
    "ekv_shadow_write": [
        _p, _p, _p, _i64, _i64,
        _i64, _p, _p, _i64, _i64,
        _i64, _i64, _p, _i32, _i64, _i32,
        _p,
    ],
    "ekv_shadow_reset": [_u64p, _i32, _i64, _p, _i32, _i64, _i32, _p],
}

_VMM = {
    "ev_create": ([_i32, ct.c_uint64, ct.c_uint64], ct.c_void_p),
    "ev_ensure": ([_p, _u64p, ct.c_size_t], ct.c_int),
    "ev_precommit": ([_p, _u64p, ct.c_size_t], ct.c_int),
    "ev_drop": ([_p, _u64p, ct.c_size_t], ct.c_int),
    "ev_base": ([_p], ct.c_uint64),
    "ev_backed": ([_p], ct.c_uint64),
    "ev_reserved": ([_p], ct.c_uint64),
    "ev_granularity": ([_p], ct.c_uint64),
    "ev_poisoned": ([_p], ct.c_int),
    "ev_close": ([_p], ct.c_int),
    "ev_set_spare": ([_p, ct.c_uint64], ct.c_int),
    "ev_spare": ([_p], ct.c_uint64),
    "ev_error": ([], ct.c_char_p),
}

ABI_VERSION = 2  # EKV_ABI_VERSION of include/ekv_kernels.h

EXPORTS = tuple(_KERNELS) + ("ekv_error", "ekv_abi_version") + tuple(_VMM)


class KernelError(RuntimeError):
    """A libekv_b200 entry point returned an error status."""


@functools.lru_cache(maxsize=None)
def library(path: str | None = None) -> ct.CDLL:
    """Load and type the shared library (once per path)."""
    path = path or os.environ.get("EKV_B200_LIBRARY") or str(LIBRARY_PATH)
    try:
        lib = ct.CDLL(path)
    except OSError as exc:
        raise RuntimeError(
            f"libekv_b200.so could not be loaded from {path}; build it with "
            "`python -m ekv_b200.build` (nvcc, sm_100a). There is no fallback path."
        ) from exc
    def entry(name):
        try:
            return getattr(lib, name)
        except AttributeError:
            raise RuntimeError(
                f"{path} does not export {name}: it is older than this package (its ABI is "
                "outdated); rebuild it with `python -m ekv_b200.build`") from None

    for name, argtypes in _KERNELS.items():
        fn = entry(name)
        fn.argtypes = argtypes
        fn.restype = ct.c_int
    entry("ekv_error").argtypes = []
    lib.ekv_error.restype = ct.c_char_p
    entry("ekv_abi_version").argtypes = []
    lib.ekv_abi_version.restype = ct.c_int
    if lib.ekv_abi_version() != ABI_VERSION:
        raise RuntimeError(
            f"{path} has ABI version {lib.ekv_abi_version()}, this package needs {ABI_VERSION}; "
            "rebuild it with `python -m ekv_b200.build`")
    for name, (argtypes, restype) in _VMM.items():
        fn = entry(name)
        fn.argtypes = argtypes
        fn.restype = restype
    return lib


TORCH_BINDING_PATH = LIBRARY_PATH.parent / "_ekv_torch.so"


@functools.lru_cache(maxsize=None)
def torch_binding():
    """The compiled pybind11 binding of the per-call lookups and gathers, or None.

    It calls the same C entry points of the library loaded above (their
    addresses are handed over here), reading tensor pointers and strides in C++
    instead of Python; a call it does not handle (unusual arguments) reports so
    and the ctypes path runs.  EKV_B200_NO_TORCH_BINDING=1 disables it.
    """
    if os.environ.get("EKV_B200_NO_TORCH_BINDING") or not TORCH_BINDING_PATH.exists():
        return None
    import importlib.util

    try:
        spec = importlib.util.spec_from_file_location("_ekv_torch", TORCH_BINDING_PATH)
        module = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(module)
    except (ImportError, OSError):
        return None
    lib = library()
    module.bind(ct.cast(lib.ekv_resolve_resident, ct.c_void_p).value,
                ct.cast(lib.ekv_lookup_slots, ct.c_void_p).value,
                ct.cast(lib.ekv_resolve_shared_blocks, ct.c_void_p).value,
                ct.cast(lib.ekv_gather_rows, ct.c_void_p).value,
                ct.cast(lib.ekv_gather_rows_planes, ct.c_void_p).value)
    return module


def last_error(name: str) -> KernelError:
    """KernelError carrying the library's message for the last failed call of this thread."""
    return KernelError(f"{name}: {library().ekv_error().decode('utf-8', 'replace')}")


def call(name: str, *args) -> None:
    """Invoke a kernel entry point; raise KernelError with its message on failure."""
    lib = library()
    if getattr(lib, name)(*args) != 0:
        raise KernelError(f"{name}: {lib.ekv_error().decode('utf-8', 'replace')}")


def u64_array(values) -> ct.Array:
    values = [int(v) for v in values]
    return (ct.c_uint64 * max(1, len(values)))(*values)


def i64_array(values) -> ct.Array:
    values = [int(v) for v in values]
    return (ct.c_int64 * max(1, len(values)))(*values)


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_handle(device: torch.device) -> int:
    """Raw cudaStream_t of torch's current stream on `device` (0 = legacy default)."""
    if _raw_stream is not None:
        return _raw_stream(device.index)
    return torch.cuda.current_stream(device).cuda_stream


_INDEX_SIZES = {torch.int32: 4, torch.int64: 8}


def index_esize(tensor: torch.Tensor, name: str) -> int:
    try:
        return _INDEX_SIZES[tensor.dtype]
    except KeyError:
        raise TypeError(f"{name} must be an int32 or int64 tensor, got {tensor.dtype}") from None


def require_cuda(tensors: dict, device: torch.device | None = None) -> torch.device:
    """All named tensors must be CUDA tensors on one device; return it."""
    for name, tensor in tensors.items():
        if tensor is None:
            continue
        if not isinstance(tensor, torch.Tensor) or not tensor.is_cuda:
            raise ValueError(f"{name} must be a CUDA tensor")
        here = tensor.device
        if device is None:
            device = here
        elif here != device:
            raise ValueError("all tensors must be on the same CUDA device")
    if device is None:
        raise ValueError("no CUDA tensor given")
    return device


def ptr(tensor: torch.Tensor | None) -> int | None:
    return None if tensor is None else tensor.data_ptr()
