"""ctypes binding of the C ABI in include/deltaattn_b200.h.

The library is the in-tree ``lib/libdeltaattn_b200.so`` built by ``build.py``. There is
no fallback: if it is missing or a call fails, a RuntimeError is raised (its text contains
"CUDA" for CUDA failures, as the reference's error classifier expects).
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libdeltaattn_b200.so")

P = ctypes.c_void_p
I32 = ctypes.c_int
I64 = ctypes.c_int64
F32 = ctypes.c_float
SZ = ctypes.c_size_t
PI64 = ctypes.POINTER(ctypes.c_int64)
PI32 = ctypes.POINTER(ctypes.c_int)

# name -> (restype, argtypes); mirrors include/deltaattn_b200.h
SIGNATURES = {
    "dab_last_error": (ctypes.c_char_p, []),
    "dab_abi_version": (I32, []),
    "dab_set_device": (I32, [I32]),
    "dab_workspace_error": (I32, [P, PI32, P]),
    "dab_chunked_eval": (I32, [P, I32, PI64, P, PI64, P, PI64, F32, I64, I64, I64, I64, I64, I64, I64, I32, P]),
    "dab_parallel_scatter_pack_kv": (I32, [P, P, P, P, P, P, P, I32, PI64, PI64, PI64, PI64, PI64, PI64, PI64,
                                           I64, I64, I64, I64, I64, I64, I64, P]),
    "dab_hybrid_flash_workspace_size": (SZ, [I64, I64, I64, I64]),
    "dab_hybrid_flash": (I32, [I32, P, P, P, P, P, P, P, I32, P, I32, PI64, F32, I64, I64, I64, I64, I64, I64,
                               I64, I64, I64, I64, I64, I64, P, SZ, I32, P]),
    "dab_hybrid_flash_devlen": (I32, [I32, P, P, P, P, P, P, P, I32, P, P, I32, PI64, F32, I64, I64, I64, I64, I64,
                                      I64, I64, I64, I64, I64, I64, I64, P, SZ, P]),
    "dab_hybrid_flash_noalloc": (I32, [I32, P, P, P, P, P, P, P, I32, P, I32, PI64, F32, I64, I64, I64, I64, I64,
                                       I64, I64, I64, I64, I64, I64, I64, I32, P]),
    "dab_noalloc_error": (I32, [PI32, P]),
    "dab_attn_fwd_flat": (I32, [P, P, P, F32, P, I32, PI64, I64, I64, I64, I64, I64, I64, I32, I64, I64, I64, P,
                                SZ, I32, P]),
    "dab_decode_update": (I32, [P, P, P, P, P, P, P, P, P, I64, I64, F32, I64, I32, PI64, PI64, PI64, PI64, I64,
                                I64, I64, I32, I64, I64, P, P]),
    "dab_decode_attention_workspace_size": (SZ, [I64, I64, I64, I64, I64]),
    "dab_decode_attention": (I32, [P, P, P, P, P, P, P, P, I32, PI64, F32, I64, I64, I64, I64, I64, I64, P, SZ,
                                   P]),
    "dab_decode_update_dev": (I32, [P, P, P, P, P, P, P, P, P, P, F32, I64, I32, PI64, PI64, PI64, PI64, I64,
                                    I64, I64, I32, I64, I64, P, P]),
    "dab_decode_attention_dev": (I32, [P, P, P, P, P, P, P, P, I32, PI64, F32, P, I32, I64, I64, I64, I64, I64, I64,
                                       P, SZ, P]),
    "dab_decode_advance": (I32, [P, I64, P]),
    "dab_rope": (I32, [P, PI64, P, PI64, P, P, PI64, I32, I64, I64, I64, I64, P]),
    "dab_proj_rope": (I32, [P, I64, P, I64, P, P, I64, P, I64, I32, I64, I64, I64, I64, I64, I64, P, SZ, P]),
    "dab_dpxa_compact": (I32, [P, PI64, P, PI64, P, P, P, I32, I64, I64, I64, I64, P]),
    "dab_dpxa_score": (I32, [P, P, P, P, P, P, P, P, F32, I32, I64, I64, I64, I64, I64, P]),
    "dab_dpxa_select": (I32, [P, P, P, F32, I64, I64, I64, I64, P]),
    "dab_block_sparse_attention": (I32, [P, P, P, P, P, I32, PI64, F32, I64, I64, I64, I64, I64, P, SZ, P]),
    "dab_periodic_meta": (I32, [P, P, P, I64, I64, I64, I64, P]),
    "dab_pack_from_keep_workspace_size": (SZ, [I64, I64, I64]),
    "dab_nm_select": (I32, [P, PI64, P, PI64, I32, I64, I64, I64, I64, I64, I64, I64, P]),
    "dab_nm_num_packed": (I64, [I64, I64, I64, I64]),
    "dab_delta_compress_workspace_size": (SZ, [I64, I64, I64, I64]),
    "dab_delta_compress": (I32, [P, PI64, P, PI64, P, P, PI64, P, PI64, P, PI64, P, P, PI64, P, P, P, PI64, P, I32,
                                 I64, I64, I64, I64, F32, I32, I64, I64, P, SZ, P]),
    "dab_pack_from_keep": (I32, [P, PI64, P, PI64, P, PI64, P, P, PI64, P, P, PI64, P, I32, I64, I64, I64, I64,
                                 I64, P, P, P, SZ, P]),
}

_lib = None
_lock = threading.Lock()
_dev = threading.local()


def load():
    """Load the library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(
                        f"deltaattention_b200: CUDA library {LIB_PATH} is not built; run "
                        "`python -m deltaattention_b200.build` (no CPU fallback exists)")
                lib = ctypes.CDLL(LIB_PATH)
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(lib, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = lib
    return _lib


def exported_symbols():
    return list(SIGNATURES)


def check(status: int, what: str) -> None:
    if status != 0:
        msg = load().dab_last_error().decode(errors="replace")
        raise RuntimeError(f"deltaattention_b200.{what} failed: {msg}")


def dtype_code(t: torch.Tensor) -> int:
    try:
        return {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {t.dtype}") from None


def ptr(t):
    if t is None:
        return None
    return ctypes.c_void_p(t.data_ptr())


def strides(vals) -> ctypes.Array:
    vals = [int(v) for v in vals]
    return (ctypes.c_int64 * len(vals))(*vals)


def stream_of(t: torch.Tensor):
    """Current torch stream of t's device, made current for the library as well."""
    dev = t.device.index if t.device.index is not None else torch.cuda.current_device()
    if getattr(_dev, "idx", None) != dev:
        check(load().dab_set_device(dev), "set_device")
        _dev.idx = dev
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def require_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError("deltaattention_b200 kernels take CUDA tensors (there is no CPU path)")


_ws_cache: dict = {}


def workspace(device: torch.device, stream: int, nbytes: int, tag: str = "attn") -> torch.Tensor:
    """Zero-initialised scratch per (tag, device, stream), grown on demand and reused.

    Attention workspaces ("attn") start with the device error word that bounded in-kernel
    waits write on timeout (read it with ``workspace_errors``)."""
    key = (tag, device.index, stream)
    buf = _ws_cache.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.zeros(max(nbytes, 4096), dtype=torch.uint8, device=device)
        _ws_cache[key] = buf
    return buf


def workspace_errors() -> list:
    """Read and clear the error word of every attention, key-compression, projection and
    packing workspace (synchronises)."""
    codes = []
    for (tag, dev, st), buf in list(_ws_cache.items()):
        if tag not in ("attn", "compress", "proj", "pack"):
            continue
        code = ctypes.c_int(0)
        check(load().dab_workspace_error(ptr(buf), ctypes.byref(code), ctypes.c_void_p(st)), "workspace_error")
        codes.append(code.value)
    return codes
