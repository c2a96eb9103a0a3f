"""ctypes binding of the in-tree C ABI library (include/suffixgpu.h).

The library is built by ``python -m suffixgpu_b200.build``. There is no
fallback: if it is missing or a call fails, an exception is raised.
"""

from __future__ import annotations

import ctypes
import os
from ctypes import (POINTER, Structure, c_char_p, c_float, c_int, c_int32,
                    c_int64, c_size_t, c_void_p)

import torch

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libsuffixgpu_b200.so")

_lib: ctypes.CDLL | None = None


class DraftParams(Structure):
    _fields_ = [
        ("batch", c_int32),
        ("seq_len", c_int32),
        ("row_stride", c_int64),
        ("k", c_int32),
        ("max_pattern_len", c_int32),
        ("max_occurrences", c_int32),
        ("num_backoff", c_int32),
        ("min_match_len", c_int32),
        ("has_spec_factor", c_int32),
        ("spec_factor", c_float),
        ("spec_offset", c_float),
        ("min_token_prob", c_float),
        ("vote_alpha", c_float),
    ]


class LocalInputs(Structure):
    _fields_ = [
        ("num_tokens", c_void_p),
        ("token_ids", c_void_p),
        ("sampled", c_void_p),
        ("sampled_cols", c_int32),
        ("host_ids", c_int32),
        ("valid_count", c_void_p),
        ("mask", c_void_p),
        ("limit", c_int64),
    ]


class LocalOutputs(Structure):
    _fields_ = [
        ("draft", c_void_p),
        ("num_valid", c_void_p),
        ("new_counts", c_void_p),
        ("best_score", c_void_p),
        ("best_len", c_void_p),
        ("best_occ", c_void_p),
        ("row_mask", c_void_p),
    ]


# name -> (argtypes); every entry point returns int status
_SIGS: dict[str, list] = {
    "sg_local_draft": [POINTER(DraftParams), POINTER(LocalInputs),
                       POINTER(LocalOutputs), c_void_p],
    "sg_mapped_host_ptr": [c_void_p, POINTER(c_void_p)],
    "sg_scatter_append": [c_void_p, c_int64, c_int32, c_int32, c_void_p,
                          c_void_p, c_void_p, c_int32, c_void_p, c_void_p],
    "sg_match_back": [c_void_p, c_int64, c_int64, c_void_p, c_int32, c_int32,
                      c_int64, c_void_p, c_void_p],
    "sg_first_occurrences": [c_void_p, c_int64, c_void_p, c_int32, c_int32,
                             c_int32, c_void_p, c_void_p, c_void_p],
    "sg_expand_chain": [c_void_p, c_int32, c_int32, c_int32, c_void_p,
                        c_void_p, c_float, c_float, c_void_p, c_void_p,
                        c_void_p, c_void_p, c_void_p],
    "sg_build_suffix_array": [c_void_p, c_int64, c_void_p, c_void_p,
                              c_size_t, POINTER(c_int32), c_void_p],
    "sg_build_suffix_array_noalloc": [c_void_p, c_int64, c_void_p,
                                      POINTER(c_int32), c_void_p],
    "sg_suffix_array_append": [c_void_p, c_int64, c_void_p, c_int64, c_int64,
                               c_int64, c_int32, c_void_p, c_void_p, c_size_t,
                               POINTER(c_int32), c_void_p],
    "sg_sa_search": [c_void_p, c_void_p, c_int64, c_void_p, c_int32, c_int32,
                     c_void_p, c_void_p, c_void_p, c_void_p],
    "sg_suffix_match_backoff": [c_void_p, c_void_p, c_int64, c_void_p,
                                c_int32, c_int32, c_void_p, c_int32,
                                c_void_p, c_int32, c_void_p, c_void_p,
                                c_void_p, c_void_p, c_void_p],
    "sg_delta_match_backoff": [c_void_p, c_int64, c_void_p, c_void_p,
                               c_int32, c_int32, c_void_p, c_int32, c_void_p,
                               c_int32, c_int32, c_void_p, c_void_p,
                               c_void_p, c_void_p, c_void_p],
    "sg_gather_tails_update": [c_void_p, c_int64, c_int32, c_void_p, c_void_p,
                               c_int32, c_void_p, c_int64, c_void_p, c_int32,
                               c_int32, c_void_p, c_void_p, c_void_p,
                               c_void_p],
    "sg_gather_tails": [c_void_p, c_int64, c_int32, c_void_p, c_int32,
                        c_int32, c_void_p, c_void_p, c_void_p],
    "sg_global_candidates": [c_void_p, c_void_p, c_void_p, c_void_p,
                             c_void_p, c_void_p, c_void_p, c_void_p, c_int64,
                             c_void_p, c_int64, c_void_p, c_int32, c_int32,
                             c_int32, c_int32, c_int32, c_float, c_float,
                             c_void_p, c_void_p, c_void_p, c_void_p,
                             c_void_p],
    "sg_append_documents": [c_void_p, c_int64, c_int64, c_void_p, c_void_p,
                            c_int32, c_void_p, c_void_p],
    "sg_delta_compact": [c_void_p, c_int64, c_int64, c_int64, c_void_p,
                         c_void_p],
    "sg_device_error": [POINTER(ctypes.c_uint32), c_int, c_void_p],
    "sg_shard_extract": [c_void_p, c_int64, c_int64, c_int64, c_void_p,
                         c_void_p, c_void_p, c_size_t, c_void_p],
    "sg_shard_pack_rows": [c_void_p, c_void_p, c_void_p, c_int32, c_int32,
                           c_void_p, c_void_p],
    "sg_shard_longest": [c_void_p, c_int64, c_void_p, c_int64, c_void_p,
                         c_int32, c_int32, c_void_p, c_void_p],
    "sg_shard_bounds": [c_void_p, c_int64, c_void_p, c_int64, c_void_p,
                        c_int32, c_int32, c_void_p, c_void_p, c_int32,
                        c_void_p, c_void_p],
    "sg_shard_resolve": [c_void_p, c_void_p, c_void_p, c_int32, c_int32,
                         c_void_p, c_int32, c_int32, c_void_p, c_void_p,
                         c_void_p, c_int32, c_int32, c_void_p, c_void_p,
                         c_void_p, c_void_p],
    "sg_global_draft_samples": [c_void_p, c_void_p, c_void_p, c_void_p,
                                c_void_p, c_void_p, c_void_p, c_int64,
                                c_void_p, c_int64, c_void_p, c_int64,
                                c_void_p, c_int32, c_int32, c_int32, c_int32,
                                c_int32, c_float, c_float, c_float, c_float,
                                c_void_p, c_void_p, c_void_p, c_void_p,
                                c_void_p],
    "sg_global_combine": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                          c_void_p, c_void_p, c_int32, c_int32, c_int32,
                          c_void_p],
    "sg_global_draft": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                        c_void_p, c_void_p, c_void_p, c_int64, c_void_p,
                        c_int64, c_void_p, c_int32, c_int32, c_int32,
                        c_int32, c_int32, c_float, c_float, c_float,
                        c_float, c_void_p, c_void_p, c_void_p, c_void_p,
                        c_void_p],
}


def lib() -> ctypes.CDLL:
    """Load the kernel library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"SuffixGPU CUDA library not found at {LIB_PATH}; build it "
                "with `python -m suffixgpu_b200.build`")
        L = ctypes.CDLL(LIB_PATH)
        L.sg_status_string.restype = c_char_p
        L.sg_status_string.argtypes = [c_int]
        L.sg_last_cuda_error.restype = c_int
        L.sg_abi_version.restype = c_int
        for name, args in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = c_int
            fn.argtypes = args
        for name in list(_SIGS_EXTRA):
            fn = getattr(L, name)
            fn.restype, fn.argtypes = _SIGS_EXTRA[name]
        _lib = L
    return _lib


# entry points with non-int return types: name -> (restype, argtypes)
_SIGS_EXTRA: dict[str, tuple] = {
    "sg_suffix_array_workspace_size": (c_size_t, [c_int64]),
    "sg_set_wait_polls": (c_int, [c_int]),
    "sg_suffix_array_append_workspace_size": (c_size_t, [c_int64]),
    "sg_shard_extract_workspace_size": (c_size_t, [c_int64]),
}


def register(name: str, argtypes: list, restype=c_int) -> None:
    """Declare another entry point's signature (used by submodules)."""
    if restype is c_int:
        _SIGS[name] = argtypes
    else:
        _SIGS_EXTRA[name] = (restype, argtypes)
    if _lib is not None:
        fn = getattr(_lib, name)
        fn.restype = restype
        fn.argtypes = argtypes


_ops = None


def torch_ops():
    """The torch operators of libsuffixgpu_b200_torch.so (loaded once;
    raises if it has not been built)."""
    global _ops
    if _ops is None:
        path = os.path.join(os.path.dirname(os.path.abspath(__file__)),
                            "libsuffixgpu_b200_torch.so")
        if not os.path.exists(path):
            raise RuntimeError(f"{path} is missing: run python -m "
                               "suffixgpu_b200.build")
        lib()  # the kernel library first (the operator links to it)
        torch.ops.load_library(path)
        _ops = torch.ops.suffixgpu_b200
    return _ops


def call(name: str, *args) -> None:
    """Call an entry point; raise on a non-zero status."""
    check(name, getattr(lib(), name)(*args))


def check(name: str, st: int) -> None:
    """Raise for a non-zero status returned by entry point ``name``."""
    if st != 0:
        L = lib()
        msg = L.sg_status_string(st).decode()
        cerr = L.sg_last_cuda_error()
        raise RuntimeError(f"{name} failed: {msg} (status {st}, "
                           f"cuda error {cerr})")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_of(device: torch.device) -> int:
    """Handle of the current CUDA stream of ``device`` (torch's raw-stream
    accessor when present: the Stream-object path costs several
    microseconds per call)."""
    if _raw_stream is not None:
        return _raw_stream(device.index if device.index is not None
                           else torch.cuda.current_device())
    return torch.cuda.current_stream(device).cuda_stream


__all__ = ["DraftParams", "LocalInputs", "LocalOutputs", "lib", "call",
           "check", "ptr", "stream_of", "register", "c_size_t"]
