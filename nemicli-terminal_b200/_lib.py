"""ctypes binding of libnemiqmv.so (the C ABI of include/nemicli_qmv.h).

The library is built in-tree by build.py.  There is no fallback: if it is missing or a call
returns a non-zero status, a RuntimeError names the failure.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

from . import build as _build

_lock = threading.Lock()
_lib = None

P, I, LL = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong

_SIGNATURES = {
    "qmv_abi_version": ([], I),
    "qmv_status_string": ([I], ctypes.c_char_p),
    "qmv_last_cuda_error": ([], I),
    "qmv_block_values": ([I], I),
    "qmv_block_bytes": ([I], I),
    "qmv_unit_values": ([I], I),
    "qmv_supported": ([I, I], I),
    "qmv_quant_q8": ([P, I, P, P, P, P, LL, P], I),
    "qmv_mv": ([I, P, I, I, P, P, P, P, I, P, P], I),
    "qmv_mv_experts": ([I, P, LL, LL, P, I, P, P, P, P, I, P, I, I, P], I),
    "qmv_block_sums": ([I, P, I, I, P, P, P, P, P], I),
    "qmv_mv_multi": ([I, I, P, P, P, I, P, P, P, P, P], I),
    "qmv_mv_x": ([I, I, P, P, P, I, P, I, P], I),
    "qmv_mv_multi_tok": ([I, I, P, P, P, I, P, P, P, P, I, P], I),
    "qmv_mv_multi_ep": ([I, I, P, P, P, I, P, P, P, P, I, I, I, P, P, P, P, P, P, P], I),
    "qmv_mv_norm": ([I, I, P, P, P, I, P, P, ctypes.c_float, P, P, ctypes.c_float, P], I),
    "qmv_set_pdl": ([I], I),
    "qmv_chain": ([P, I, P, P], I),
    "qmv_chain_noalloc": ([P, I, P], I),
    "qmv_chain_workspace_bytes": ([], LL),
    "qmv_device_status": ([I, P, P], I),
    "qmv_norm_q8": ([P, P, ctypes.c_float, P, P, ctypes.c_float, P, P, P, P, P, I, P], I),
    "qmv_act_q8": ([P, P, I, P, P, P, P, P, I, P], I),
    "qmv_unpack": ([I, P, LL, P, I, P], I),
    "qmv_moe_workspace_bytes": ([I, I, I, I], LL),
    "qmv_mm_tc_workspace_bytes": ([I, I, I, I], LL),
    "qmv_expert_dispatch": ([P, I, I, LL, I, P, I, I, P, I, P, P, P], I),
    "qmv_expert_combine": ([P, I, P, P, I, I, I, P, P], I),
    "qmv_mm_tc": ([I, P, I, I, P, I, I, P, P, LL, P], I),
    "qmv_moe_ffn": ([I, P, P, LL, I, P, LL, LL, P, P, I, I, P, I, LL, I, I, P, P, P], I),
}

ABI_VERSION = 2


def lib_path() -> str:
    return _build.LIB_PATH


def load() -> ctypes.CDLL:
    """Load the CUDA library (raises if it was not built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            path = lib_path()
            if not os.path.exists(path):
                raise RuntimeError(f"CUDA library missing: {path} (build it with nemicli_terminal_b200.build.build())")
            L = ctypes.CDLL(path)
            for name, (args, res) in _SIGNATURES.items():
                fn = getattr(L, name)
                fn.argtypes = args
                fn.restype = res
            if L.qmv_abi_version() != ABI_VERSION:
                raise RuntimeError(f"{path}: ABI version {L.qmv_abi_version()} != {ABI_VERSION}")
            _lib = L
    return _lib


def exported_symbols() -> list:
    return list(_SIGNATURES)


def check(status: int, what: str) -> None:
    if status:
        L = load()
        msg = L.qmv_status_string(status).decode()
        extra = f" (cudaError {L.qmv_last_cuda_error()})" if status == 5 else ""
        raise RuntimeError(f"{what}: {msg}{extra}")


def on_gpu(x) -> bool:
    """A CUDA tensor or CUDA device: the one device question the mirrors ask before calling the library."""
    if isinstance(x, torch.Tensor):
        return x.is_cuda
    return torch.device(x).type == "cuda"


def ptr(t) -> ctypes.c_void_p:
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def stream_ptr(device=None) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def device_status(clear: bool = True, device=None) -> int:
    """The device status word (bit 1: a refused expert id or address); synchronises the stream."""
    out = ctypes.c_int(0)
    check(load().qmv_device_status(int(clear), ctypes.byref(out), stream_ptr(device)), "qmv_device_status")
    return out.value
