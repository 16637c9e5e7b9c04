"""ctypes binding of libfathom_b200.so (C ABI in include/fathom_b200.h).

There is no fallback: if the shared library is missing or fails to load, every
operation raises.  Build it with `python -m fathom_b200.build`.
"""
import ctypes
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libfathom_b200.so")

FATHOM_OK = 0
FATHOM_ERR_NULL = -1
FATHOM_ERR_SHAPE = -2
FATHOM_ERR_UNSUPPORTED = -3
FATHOM_ERR_CUDA = -4
FATHOM_ERR_WORKSPACE = -5

HOST_HUGEPAGES = 1

DTYPE_CODE = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}

P = ctypes.c_void_p
I64 = ctypes.c_int64
I32 = ctypes.c_int
SZ = ctypes.c_size_t

# name -> (restype, argtypes); the complete exported surface of include/fathom_b200.h
SIGNATURES = {
    "fathom_last_error": (ctypes.c_char_p, []),
    "fathom_abi_version": (I32, []),
    "fathom_quantise_pack": (I32, [P, I32, I64, I64, I64, I64, I32, P, P, I32, P, P, P]),
    "fathom_pack_codes": (I32, [P, I64, I64, I64, P, P]),
    "fathom_unpack_planes": (I32, [P, I64, I64, I64, P, P]),
    "fathom_relayout": (I32, [P, P, I64, I64, I64, P, P, I64, P]),
    "fathom_dequant_planes": (I32, [P, P, I32, I64, I64, P, I64, P, P]),
    "fathom_scan_planes_reference": (I32, [P, I64, I32, I64, P, P, I32, P, P, P]),
    "fathom_scan_chan4_reference": (I32, [P, I64, I32, I64, P, P, I32, P, P, P]),
    "fathom_make_plan": (I32, [P, P, I64, I32, I32, P, P, P, P, P, P, P, P]),
    "fathom_scan": (I32, [P, I64, I32, I64, I64, P, P, I32, P, P, I64, I64, P, P]),
    "fathom_wait_timeouts": (I32, [P, I32]),
    "fathom_pack_chan4": (I32, [P, I64, I64, I64, P, P]),
    "fathom_channel_list": (I32, [P, I64, P, P, P]),
    "fathom_scan_chan4": (I32, [P, I64, I32, I64, I64, P, P, P, P, I64, I64, P, P]),
    "fathom_klt_quantise_pack": (I32, [P, I32, I64, I64, I64, P, P, I64, I32, P, P, I32, P, P, P, P]),
    "fathom_klt_query": (I32, [P, I64, I32, P, P, P, P, P]),
    "fathom_scan_select_workspace_bytes": (SZ, [I64, I32, I64, I64]),
    "fathom_scan_select": (I32, [P, I64, I32, I64, I64, P, P, I32, P, P, I64, I64, I64, I64, I64, I64, P, P, I64, P,
                                 P, SZ, P, P]),
    "fathom_select_workspace_bytes": (SZ, [I64, I64, I64]),
    "fathom_select_topk": (I32, [P, I64, I64, I64, I64, I64, I64, I64, P, I64, P, P, SZ, P]),
    "fathom_sink_local_topk": (I32, [P, I64, I64, I64, I64, I64, P, P, SZ, P]),
    "fathom_sink_local_topk_static": (I32, [P, I64, I64, I64, I64, I64, P, P]),
    "fathom_merge_topk": (I32, [P, P, I64, I64, I64, P, P, P]),
    "fathom_gather_rows": (I32, [P, I64, P, I64, I64, I64, P, P]),
    "fathom_decode_workspace_bytes": (SZ, [I64, I32, I64]),
    "fathom_decode_attention": (I32, [P, I64, I32, P, I64, P, P, I64, I64, I64, P, P, I64, P, P, P, SZ, P]),
    "fathom_decode_partial_workspace_bytes": (SZ, [I64, I32, I64]),
    "fathom_decode_attention_partial": (I32, [P, I64, I32, P, I64, P, P, I64, I64, I64, I64, P, P, SZ, P]),
    "fathom_attention_combine": (I32, [P, I64, I64, P, P, P]),
    "fathom_gather_runs": (I32, [P, P, P, P, P, I64, I64, I64, P]),
    "fathom_stage_planes": (I32, [P, P, P, I64, I64, I64, I64, P, P, P]),
    "fathom_host_alloc_mapped": (I32, [SZ, ctypes.POINTER(P), ctypes.POINTER(P)]),
    "fathom_host_alloc_mapped_ex": (I32, [SZ, I32, ctypes.POINTER(P), ctypes.POINTER(P)]),
    "fathom_host_free": (I32, [P]),
}

_lib = None


class FathomError(RuntimeError):
    """A libfathom_b200 call returned a negative status."""

    def __init__(self, status, what, message):
        super().__init__(f"{what} failed (status {status}): {message}")
        self.status = status


def lib():
    """The loaded library (loads and declares signatures on first use)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m fathom_b200.build` "
                               "(fathom_b200 has no CPU or eager fallback)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(status, what):
    if status != FATHOM_OK:
        msg = lib().fathom_last_error().decode(errors="replace")
        if status in (FATHOM_ERR_SHAPE, FATHOM_ERR_NULL, FATHOM_ERR_UNSUPPORTED):
            raise ValueError(f"{what}: {msg}")
        raise FathomError(status, what, msg)


def ptr(x):
    """Device address of a tensor or of any object exposing data_ptr() (e.g. a mapped host alias); None -> NULL."""
    if x is None:
        return None
    return x.data_ptr()


def stream_of(device):
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(*tensors):
    for t in tensors:
        if isinstance(t, torch.Tensor) and not t.is_cuda:
            raise ValueError("fathom_b200 operates on CUDA tensors only (no CPU path); got a tensor on "
                             f"{t.device}")


_ws_cache = {}


def workspace(device, nbytes, tag="ws"):
    """A cached, 256-byte aligned device scratch buffer of at least nbytes for `device`."""
    key = (torch.device(device), tag)
    buf = _ws_cache.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)
        _ws_cache[key] = buf
    return buf
