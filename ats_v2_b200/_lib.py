"""ctypes binding of ``libats_b200.so`` (the C ABI in include/ats_b200.h).

The library is loaded on first use from this package's directory.  If it is
missing the import of any op fails with an error that says how to build it:
there is no fallback implementation behind these entry points.
"""

from __future__ import annotations

import contextlib
import ctypes
import os
import threading
from ctypes import POINTER, c_char_p, c_float, c_int, c_int64, c_size_t, c_void_p
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libats_b200.so"

ATS_OK = 0
ATS_EBADARG = -1
ATS_EUNSUPPORTED = -2
ATS_ECUDA = -3
ATS_ETIMEOUT = -4

ATS_F32 = 0
ATS_BF16 = 1

ATS_MOE_PACKED = 0
ATS_MOE_SLOTS = 1
ATS_ROUTER_BWD_DW, ATS_ROUTER_BWD_DX, ATS_ROUTER_BWD_ALL = 1, 2, 3  # stages of ats_moe_router_bwd_staged

_I64x3 = c_int64 * 3

# name -> (restype, argtypes); mirrors include/ats_b200.h
SIGNATURES: dict[str, tuple] = {
    "ats_abi_version": (c_int, []),
    "ats_strerror": (c_char_p, [c_int]),
    "ats_last_error_message": (c_char_p, []),
    "ats_kernel_launches": (ctypes.c_uint64, []),
    "ats_set_gemm_sm_limit": (c_int, [c_int]),
    "ats_gemm_supported": (c_int, [c_int, c_int64, c_int64, c_int64]),
    "ats_gemm_workspace_bytes": (c_size_t, []),
    "ats_gemm_fwd": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int64, c_int64, c_int64, c_void_p, c_size_t,
                             c_void_p]),
    "ats_gemm_bwd": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int64, c_int64, c_int64,
                             c_void_p, c_size_t, c_void_p]),
    "ats_gemm_rope_fwd": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int64, c_int64, c_int64, c_void_p,
                                  c_void_p, c_int64, c_void_p, c_size_t, c_void_p]),
    "ats_ipc_handle_bytes": (c_size_t, []),
    "ats_ipc_export": (c_int, [c_void_p, c_void_p, POINTER(ctypes.c_uint64), POINTER(ctypes.c_uint64)]),
    "ats_ipc_open": (c_int, [c_void_p, POINTER(c_void_p)]),
    "ats_ipc_close": (c_int, [c_void_p]),
    "ats_peer_copies": (c_int, [c_int, POINTER(c_void_p), POINTER(c_void_p), POINTER(ctypes.c_uint64), c_void_p]),
    "ats_gemm_sm_limit": (c_int, []),
    "ats_set_gemm_pairs": (c_int, [c_int]),
    "ats_gemm_pairs": (c_int, []),
    "ats_device_status": (c_int, [POINTER(c_int)]),
    "ats_set_wait_budget": (c_int, [c_int64]),
    "ats_rmsnorm_fwd": (c_int, [c_void_p, c_int64, c_int, c_void_p, c_int, c_void_p, c_int64, c_void_p,
                                c_int64, c_int64, c_float, c_void_p]),
    "ats_rmsnorm_bwd_workspace_bytes": (c_size_t, [c_int64, c_int64]),
    "ats_rmsnorm_bwd": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p, c_void_p,
                                c_size_t, c_int64, c_int64, c_float, c_void_p]),
    "ats_rmsnorm_status": (c_int, [POINTER(c_int)]),
    "ats_rmsnorm_bwd_noalloc": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p,
                                        c_int64, c_int64, c_float, c_void_p]),
    "ats_rmsnorm_residual_fwd": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p, c_int64,
                                         c_int64, c_float, c_void_p]),
    "ats_rmsnorm_residual_bwd": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p,
                                         c_void_p, c_void_p, c_size_t, c_int64, c_int64, c_float, c_void_p]),
    "ats_add_rmsnorm_fwd": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p, c_int64, c_int64,
                                    c_float, c_void_p]),
    "ats_add_rmsnorm_bwd_workspace_bytes": (c_size_t, [c_int64, c_int64]),
    "ats_add_rmsnorm_bwd": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p,
                                    c_void_p, c_size_t, c_int64, c_int64, c_float, c_void_p]),
    "ats_rope_apply": (c_int, [c_void_p, c_void_p, c_int64, POINTER(c_int64), POINTER(c_int64),
                               c_void_p, c_void_p, c_int64, POINTER(c_int64), POINTER(c_int64),
                               c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_int, c_int, c_void_p]),
    "ats_moe_status": (c_int, [c_void_p, c_size_t, c_int64, c_int, c_int, c_int64, c_int, POINTER(c_int)]),
    "ats_moe_plan_export": (c_int, [c_void_p, c_size_t, c_int64, c_int, c_int, c_int64, c_int, c_void_p, c_void_p,
                                    c_void_p, c_void_p]),
    "ats_moe_uses_tensor_cores": (c_int, [c_int, c_int64, c_int64]),
    "ats_moe_topk": (c_int, [c_void_p, c_int64, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p]),
    "ats_moe_max_rows": (c_int64, [c_int64, c_int, c_int, c_int64, c_int]),
    "ats_moe_workspace_bytes": (c_size_t, [c_int64, c_int, c_int, c_int64, c_int]),
    "ats_moe_route_plan": (c_int, [c_void_p, c_int64, c_int, c_int, c_int64, c_int, c_float, c_void_p, c_void_p,
                                   c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    "ats_moe_gather": (c_int, [c_void_p, c_void_p, c_int, c_int64, c_int64, c_int, c_int, c_int64, c_int,
                               c_void_p, c_size_t, c_void_p]),
    "ats_moe_experts_fwd": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int,
                                    c_int64, c_int, c_int, c_int64, c_int, c_int64, c_int64, c_void_p, c_size_t,
                                    c_void_p]),
    "ats_moe_combine": (c_int, [c_void_p, c_void_p, c_int, c_int64, c_int64, c_int, c_int, c_int64, c_int,
                                c_void_p, c_size_t, c_void_p]),
    "ats_moe_combine_bwd": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int64, c_int64, c_int,
                                    c_int, c_int64, c_int, c_void_p, c_size_t, c_void_p]),
    "ats_moe_experts_bwd": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                    c_void_p, c_void_p, c_void_p, c_int, c_int64, c_int, c_int, c_int64, c_int,
                                    c_int64, c_int64, c_void_p, c_size_t, c_void_p]),
    "ats_moe_scatter_grad": (c_int, [c_void_p, c_void_p, c_int, c_int64, c_int64, c_int, c_int, c_int64, c_int,
                                     c_void_p, c_size_t, c_void_p]),
    "ats_moe_route_bwd": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64,
                                  c_int, c_int, c_int64, c_int, c_float, c_void_p, c_size_t, c_void_p]),
    "ats_moe_ep_segments_bytes": (c_size_t, [c_int, c_int]),
    "ats_moe_ep_segments": (c_int, [c_void_p, c_int, c_int, c_int64, c_int, c_void_p, c_size_t, c_void_p]),
    "ats_moe_ep_experts_fwd": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int,
                                       c_int, c_int64, c_int64, c_int64, c_void_p, c_size_t, c_void_p]),
    "ats_moe_ep_experts_fwd_sources": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int,
                                               c_int, c_int, c_int64, c_int64, c_int64, c_void_p, c_size_t, c_int,
                                               c_int, c_void_p]),
    "ats_moe_ep_experts_bwd": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                       c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int64, c_int64,
                                       c_int64, c_void_p, c_size_t, c_void_p]),
    "ats_moe_ep_status": (c_int, [c_void_p, c_size_t, c_int, c_int, POINTER(c_int)]),
    "ats_moe_ep_counts_ints": (c_size_t, [c_int]),
    "ats_moe_ep_push": (c_int, [c_void_p, c_void_p, c_int64, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int,
                                c_void_p, c_int64, c_int64, c_int, c_int, c_void_p]),
    "ats_moe_ep_push_split": (c_int, [c_void_p, c_void_p, c_int64, c_void_p, c_int, c_int, c_int, c_int, c_int,
                                      c_int, c_void_p, c_int64, c_int64, c_int, c_int, c_int, c_void_p]),
    "ats_moe_ep_pull": (c_int, [c_void_p, c_int64, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_void_p,
                                c_int64, c_int64, c_int, c_int, c_void_p]),
    "ats_moe_ep_experts_bwd_staged": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                              c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int64, c_int64,
                                              c_int64, c_void_p, c_size_t, c_int, c_void_p]),
    "ats_moe_ep_combine": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_int, c_int64, c_void_p, c_size_t,
                                   c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_int64, c_int64, c_int,
                                   c_void_p]),
    "ats_moe_ep_zero_padding": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_int64,
                                        c_int64, c_int, c_void_p]),
    "ats_swiglu_supported": (c_int, [c_int, c_int64, c_int64, c_int64]),
    "ats_swiglu_workspace_bytes": (c_size_t, []),
    "ats_swiglu_rows": (c_int64, [c_int64]),
    "ats_swiglu_fwd": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int64, c_int64,
                               c_int64, c_void_p, c_size_t, c_void_p]),
    "ats_swiglu_bwd": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                               c_void_p, c_void_p, c_int, c_int64, c_int64, c_int64, c_void_p, c_size_t, c_void_p]),
    "ats_swiglu_status": (c_int, [c_void_p, c_size_t, POINTER(c_int)]),
    "ats_moe_router_supported": (c_int, [c_int, c_int64, c_int64, c_int]),
    "ats_moe_router_workspace_bytes": (c_size_t, [c_int64, c_int64, c_int]),
    "ats_moe_router_fwd": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int, c_void_p,
                                   c_size_t, c_void_p]),
    "ats_moe_router_bwd": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_int, c_int64,
                                   c_int, c_void_p, c_void_p, c_int64, c_int64, c_int, c_void_p, c_size_t,
                                   c_void_p]),
    "ats_moe_router_bwd_staged": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_int,
                                          c_int64, c_int, c_void_p, c_void_p, c_int64, c_int64, c_int, c_void_p,
                                          c_size_t, c_int, c_void_p]),
    "ats_moe_router_status": (c_int, [c_void_p, c_size_t, c_int64, c_int64, c_int, POINTER(c_int)]),
}

_lib = None
_lock = threading.Lock()


class AtsError(RuntimeError):
    """A non-zero status from the C ABI."""

    def __init__(self, fn: str, status: int, detail: str):
        super().__init__(f"{fn} failed: {detail} (status {status})")
        self.status = status


def load() -> ctypes.CDLL:
    """Load (once) and return the library; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise ImportError(
                    f"{LIB_PATH} is missing. Build it with `python -m ats_v2_b200._build` "
                    "(nvcc for sm_100a); ats_v2_b200 has no implementation without it.")
            lib = ctypes.CDLL(os.fspath(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


# ATS_CHECK_STATUS=1: after every call, wait for the device and raise if a
# bounded device wait gave up in it (a debugging mode: it synchronises).
_CHECK_EACH_CALL = os.environ.get("ATS_CHECK_STATUS", "0") not in ("", "0")


def call(name: str, *args) -> None:
    """Call a status-returning entry point; raise AtsError on failure."""
    lib = load()
    st = getattr(lib, name)(*args)
    if st != ATS_OK:
        detail = lib.ats_last_error_message().decode(errors="replace") or lib.ats_strerror(st).decode()
        raise AtsError(name, st, detail)
    if _CHECK_EACH_CALL and not name.endswith("_status"):
        check_device_status(name)


def check_device_status(after: str = "an earlier call") -> None:
    """Raise AtsError if a bounded wait of a tensor-core GEMM or an RMSNorm ring
    kernel on the current device gave up since the last check (the status word
    is cleared by reading it).  Synchronous: the modules call it only where the
    host waits for the device anyway."""
    lib = load()
    code = c_int(0)
    st = lib.ats_device_status(ctypes.byref(code))
    if st != ATS_OK:
        detail = lib.ats_last_error_message().decode(errors="replace") or lib.ats_strerror(st).decode()
        raise AtsError(after, st, detail)


def query(name: str, *args):
    return getattr(load(), name)(*args)


@contextlib.contextmanager
def gemm_sm_limit(sms: int):
    """Launch the persistent tensor-core GEMMs of this thread on at most ``sms``
    SMs inside the block (0: all), leaving the rest to a collective that runs
    beside them on another stream."""
    prev = query("ats_gemm_sm_limit")
    call("ats_set_gemm_sm_limit", int(sms))
    try:
        yield
    finally:
        call("ats_set_gemm_sm_limit", prev)


@contextlib.contextmanager
def gemm_pairs(enabled: bool):
    """Run the tensor-core expert, dense-FFN and MLA GEMMs inside the block on
    CTA pairs (256-row tiles) or on single CTAs (128-row tiles, the default).
    The setting is process-wide; both give identical results."""
    prev = query("ats_gemm_pairs")
    call("ats_set_gemm_pairs", 1 if enabled else 0)
    try:
        yield
    finally:
        call("ats_set_gemm_pairs", prev)


def dtype_code(t: torch.dtype) -> int:
    if t == torch.float32:
        return ATS_F32
    if t == torch.bfloat16:
        return ATS_BF16
    raise TypeError(f"ats_v2_b200 kernels take float32 or bfloat16 tensors, got {t}")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def strides3(*s: int):
    return _I64x3(*s)


def on_cpu(name: str, *tensors: torch.Tensor | None) -> bool:
    """True when every given tensor is a CPU tensor, False when every one is a
    CUDA tensor on one device; mixed devices raise.

    The mirror modules use it as the reference's own modules do (for example
    ``fused_mla_kv_decompress``, mla_triton.py:144-151, runs its kernel only
    for CUDA tensors): CPU tensors take the reference's torch formulas, which
    its CPU tests pin, and CUDA tensors always take this library's kernels --
    a CUDA tensor never runs the torch formula, and a missing library raises."""
    devs = {t.device.type for t in tensors if t is not None}
    if devs == {"cpu"}:
        return True
    if "cpu" in devs:
        raise RuntimeError(f"{name}: tensors on different devices ({sorted(devs)})")
    require_cuda(name, *tensors)
    return False


def require_cuda(name: str, *tensors: torch.Tensor) -> None:
    """Every tensor must live on one CUDA device: there is no CPU path."""
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError(f"{name}: ats_v2_b200 runs on CUDA tensors only (got a {t.device} tensor)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"{name}: tensors on different devices ({dev} and {t.device})")
