"""ctypes binding of librgpt_kernels.so (the C ABI declared in include/rgpt.h).

This is the only place Python touches the native library. Every wrapper takes
torch tensors, checks devices/dtypes/contiguity on the host, passes raw device
pointers plus the current CUDA stream, and raises RuntimeError with the
library's message on a non-zero status. There is no CPU or torch fallback: a
missing library or a non-CUDA tensor is an error.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "librgpt_kernels.so")

_c_int = ctypes.c_int
_c_ll = ctypes.c_longlong
_c_float = ctypes.c_float
_c_vp = ctypes.c_void_p

# name -> argtypes (restype is always c_int)
_SIGNATURES: dict[str, list] = {
    "rgpt_last_error": [ctypes.c_char_p, ctypes.c_ulonglong],
    "rgpt_device_error": [],
    "rgpt_version": [],
    "rgpt_gemm_bf16": [
        _c_vp, _c_int, _c_ll, _c_ll,  # A, a_mn_major, lda, a_bstride
        _c_vp, _c_int, _c_ll, _c_ll,  # B, b_mn_major, ldb, b_bstride
        _c_int, _c_int, _c_int, _c_int,  # M, N, K, batch
        _c_int, _c_int, _c_float, _c_float,  # epi, act, alpha, beta
        _c_vp, _c_ll, _c_ll,  # D, ldd, d_bstride
        _c_vp, _c_ll, _c_ll,  # D2, ldd2, d2_bstride
        _c_vp, _c_ll, _c_ll,  # C, ldc, c_bstride
        _c_vp, _c_int, _c_vp, _c_vp,  # colscale, splitk, alpha_dev, stream
    ],
    "rgpt_gemm_bf16_dropout": [
        _c_vp, _c_int, _c_ll, _c_ll, _c_vp, _c_int, _c_ll, _c_ll, _c_int, _c_int, _c_int, _c_int,
        _c_int, _c_int, _c_float, _c_float, _c_vp, _c_ll, _c_ll, _c_vp, _c_ll, _c_ll, _c_vp, _c_ll, _c_ll,
        _c_vp, _c_int, _c_vp,  # colscale, splitk, alpha_dev
        _c_vp, _c_ll, _c_float,  # drop_mask, drop_ldm, drop_p
        _c_vp,
    ],
    "rgpt_gemm_argmax": [_c_vp, _c_ll, _c_vp, _c_ll, _c_int, _c_int, _c_int, _c_vp, _c_vp, _c_ll, _c_vp, _c_vp],
    "rgpt_drop_mask": [_c_vp, _c_ll, _c_vp, ctypes.c_uint, _c_float, _c_int, _c_int, _c_vp],
    "rgpt_attn_drop_mask": [_c_vp, _c_vp, ctypes.c_uint, _c_float, _c_int, _c_int, _c_int, _c_vp],
    "rgpt_rownorm_fwd": [_c_vp, _c_vp, _c_vp, _c_vp, _c_float, _c_int, _c_float, _c_float, _c_int, _c_int,
                         _c_vp, _c_vp, _c_vp, _c_vp],
    "rgpt_rownorm_bwd": [_c_vp, _c_vp, _c_vp, _c_float, _c_int, _c_float, _c_float, _c_int, _c_int,
                         _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp,
                         _c_vp, _c_vp, _c_float, _c_vp],
    "rgpt_qkv_prep_fwd": [_c_vp, _c_vp, _c_vp, _c_vp, _c_int, _c_float, _c_float, _c_vp, _c_vp, _c_float, _c_float,
                          _c_float, _c_float, _c_int, _c_int, _c_int, _c_vp],
    "rgpt_qkv_prep_bwd": [_c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp,
                          _c_int, _c_float, _c_float, _c_vp, _c_vp, _c_float, _c_float, _c_float, _c_float,
                          _c_int, _c_int, _c_int, _c_vp],
    "rgpt_embedding_fwd": [_c_vp, _c_vp, _c_vp, _c_int, _c_int, _c_int, _c_vp, _c_vp, ctypes.c_uint, _c_float, _c_vp],
    "rgpt_embedding_bwd": [_c_vp, _c_vp, _c_vp, _c_int, _c_int, _c_int, _c_vp, _c_float, _c_vp],
    "rgpt_cross_entropy": [_c_vp, _c_ll, _c_int, _c_int, _c_vp, _c_int, _c_float, _c_vp, _c_vp, _c_vp, _c_vp,
                           _c_int, _c_vp],
    "rgpt_cross_entropy_noalloc": [_c_vp, _c_ll, _c_int, _c_int, _c_vp, _c_int, _c_float, _c_vp, _c_vp, _c_int,
                                   _c_vp],
    "rgpt_halt_losses": [_c_vp, _c_vp, _c_vp, _c_int, _c_int, _c_float, _c_vp, _c_vp, _c_vp],
    "rgpt_adamw": [_c_vp, _c_vp, _c_vp, _c_int, _c_int, _c_float, _c_float, _c_float, _c_float, _c_float, _c_int,
                   _c_vp, _c_vp],
    "rgpt_muon_prep": [_c_vp, _c_int, _c_int, _c_int, _c_vp, _c_ll, _c_int, _c_float, _c_int, _c_vp, _c_vp, _c_vp],
    "rgpt_ns_scale": [_c_vp, _c_ll, _c_int, _c_int, _c_int, _c_int, _c_vp, _c_vp],
    "rgpt_ns_sumsq": [_c_vp, _c_int, _c_ll, _c_ll, _c_ll, _c_int, _c_int, _c_int, _c_vp, _c_vp],
    "rgpt_ns_split": [_c_vp, _c_int, _c_ll, _c_ll, _c_ll, _c_int, _c_int, _c_int, _c_vp, _c_vp, _c_ll, _c_ll,
                      _c_vp, _c_ll, _c_ll, _c_int, _c_ll, ctypes.c_uint, _c_vp],
    "rgpt_muon_apply": [_c_vp, _c_int, _c_int, _c_int, _c_vp, _c_ll, _c_int, _c_float, _c_float, _c_float,
                        _c_float, _c_vp, _c_vp],
    "rgpt_ns_chain": [_c_vp, _c_vp, _c_vp, _c_vp, _c_int, _c_int, _c_int, _c_ll, _c_ll, _c_ll, _c_ll, _c_int, _c_float,
                      _c_float, _c_float, _c_vp, _c_vp],
    "rgpt_segment_copy": [_c_vp, _c_vp, _c_vp, _c_int, _c_int, _c_vp, _c_int, _c_int, _c_float, _c_int, _c_vp],
    "rgpt_rownorm_any_fwd": [_c_vp, _c_vp, _c_vp, _c_int, _c_float, _c_float, _c_ll, _c_int, _c_vp],
    "rgpt_rownorm_any_bwd": [_c_vp, _c_vp, _c_vp, _c_int, _c_float, _c_float, _c_ll, _c_int, _c_vp, _c_vp, _c_vp,
                             _c_vp],
    "rgpt_rope": [_c_vp, _c_ll, _c_ll, _c_ll, _c_vp, _c_vp, _c_int, _c_int, _c_int, _c_int, _c_int, _c_vp],
    "rgpt_attn_fwd": [_c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_int, _c_int, _c_int, _c_int,
                      _c_vp, _c_float, _c_vp],
    "rgpt_attn_bwd_prep": [_c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_int, _c_int, _c_int, _c_int, _c_vp],
    "rgpt_attn_bwd": [_c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_ll, _c_vp, _c_ll,
                      _c_int, _c_int, _c_int, _c_int, _c_vp, _c_float, _c_vp],
}

_lock = threading.Lock()
_lib = None


def load() -> ctypes.CDLL:
    """Load (once) and return the native library; raises if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with `make -C rgpt_b200/csrc` "
                    "(there is no CPU fallback)")
            lib = ctypes.CDLL(LIB_PATH)
            for name, argtypes in _SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = argtypes
                fn.restype = _c_int
            _lib = lib
    return _lib


def register(name: str, argtypes: list) -> None:
    """Declare another entry point's signature (used by op modules)."""
    _SIGNATURES[name] = argtypes
    if _lib is not None:
        fn = getattr(_lib, name)
        fn.argtypes = argtypes
        fn.restype = _c_int


def last_error() -> str:
    buf = ctypes.create_string_buffer(1024)
    load().rgpt_last_error(buf, 1024)
    return buf.value.decode(errors="replace")


# Kernels each entry point enqueues (rgpt_cross_entropy: up to 3, counted by its wrapper).
_KERNELS_PER_CALL = {"rgpt_last_error": 0, "rgpt_device_error": 0, "rgpt_version": 0,
                     "rgpt_cross_entropy_noalloc": 3}
launch_count = 0  # native kernels enqueued by this process (read by the benchmark)


def call(name: str, *args, kernels: int | None = None) -> None:
    """Invoke entry point `name`; raise RuntimeError on a non-zero status."""
    global launch_count
    rc = getattr(load(), name)(*args)
    if rc != 0:
        raise RuntimeError(f"{name} failed (status {rc}): {last_error()}")
    launch_count += _KERNELS_PER_CALL.get(name, 1) if kernels is None else kernels


def device_error() -> int:
    """Synchronise and return/clear the device-side error word (0 = none)."""
    rc = load().rgpt_device_error()
    if rc != 0:
        raise RuntimeError(f"device error: {last_error()}")
    return 0


def stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    if t is None:
        return None
    if not t.is_cuda:
        raise RuntimeError("librgpt_kernels only takes CUDA tensors (no CPU path)")
    return t.data_ptr()
