"""The C-ABI library: loads, exports every symbol include/ats_b200.h declares,
and rejects bad arguments on the host (no GPU needed: nothing is launched)."""

from __future__ import annotations

import ctypes
import re

import pytest

from ats_v2_b200 import _lib
from tests.conftest import ROOT

HEADER = ROOT / "include" / "ats_b200.h"


def declared_symbols() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"ATS_API\s+[\w\s\*]+?\b(ats_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert "ats_rmsnorm_fwd" in syms and "ats_moe_route_plan" in syms and "ats_rope_apply" in syms
    assert len(syms) >= 20


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, f"declared but not exported: {missing}"


def test_python_binding_covers_every_declared_symbol():
    assert set(declared_symbols()) <= set(_lib.SIGNATURES)


def test_abi_version_and_strings():
    lib = _lib.load()
    assert lib.ats_abi_version() == 1
    assert lib.ats_strerror(0) == b"ok"
    assert lib.ats_strerror(_lib.ATS_EBADARG) == b"invalid argument"
    assert lib.ats_strerror(12345) == b"unknown status"


def test_bad_arguments_rejected_before_any_launch():
    lib = _lib.load()
    # rows < 0
    st = lib.ats_rmsnorm_fwd(None, 8, 0, None, 0, None, 8, None, -1, 8, 1e-6, None)
    assert st == _lib.ATS_EBADARG
    assert b"bad shape" in lib.ats_last_error_message()
    # unsupported dtype code
    st = lib.ats_rmsnorm_fwd(None, 8, 7, None, 0, None, 8, None, 4, 8, 1e-6, None)
    assert st == _lib.ATS_EBADARG
    # rope: odd head dim
    s3 = _lib.strides3(1, 1, 1)
    st = lib.ats_rope_apply(None, None, 1, s3, s3, None, None, 0, None, None, None, None, 8, 1, 1, 7, 1, 0, None)
    assert st == _lib.ATS_EBADARG
    # moe: k > E
    st = lib.ats_moe_topk(None, 4, 2, 3, None, None, None, None)
    assert st == _lib.ATS_EBADARG
    # workspace too small
    st = lib.ats_moe_route_plan(None, 4, 4, 2, 4, 0, 0.01, None, None, None, None, None, None, 0, None)
    assert st == _lib.ATS_EBADARG
    assert b"workspace too small" in lib.ats_last_error_message()


def test_gemm_sm_limit_is_per_thread_host_state():
    import threading
    lib = _lib.load()
    assert lib.ats_gemm_sm_limit() == 0
    with _lib.gemm_sm_limit(100):
        assert lib.ats_gemm_sm_limit() == 100
        seen = []
        t = threading.Thread(target=lambda: seen.append(lib.ats_gemm_sm_limit()))
        t.start()
        t.join()
        assert seen == [0]  # another thread's launches are not limited
    assert lib.ats_gemm_sm_limit() == 0
    assert lib.ats_set_gemm_sm_limit(-1) == _lib.ATS_EBADARG
    assert lib.ats_gemm_sm_limit() == 0


def test_peer_exchange_entry_points_check_arguments_on_the_host():
    import ctypes
    lib = _lib.load()
    assert lib.ats_ipc_handle_bytes() == 64  # sizeof(cudaIpcMemHandle_t)
    h = ctypes.create_string_buffer(64)
    off, size = ctypes.c_uint64(), ctypes.c_uint64()
    assert lib.ats_ipc_export(None, h, ctypes.byref(off), ctypes.byref(size)) == _lib.ATS_EBADARG
    assert lib.ats_ipc_open(None, None) == _lib.ATS_EBADARG
    assert lib.ats_ipc_close(None) == _lib.ATS_EBADARG
    assert lib.ats_peer_copies(-1, None, None, None, None) == _lib.ATS_EBADARG
    assert lib.ats_peer_copies(2, None, None, None, None) == _lib.ATS_EBADARG
    zero = (ctypes.c_uint64 * 1)(0)
    nul = (ctypes.c_void_p * 1)(None)
    assert lib.ats_peer_copies(1, nul, nul, zero, None) == _lib.ATS_OK  # empty copies issue nothing
    assert lib.ats_peer_copies(0, None, None, None, None) == _lib.ATS_OK


def test_workspace_queries():
    lib = _lib.load()
    assert lib.ats_rmsnorm_bwd_workspace_bytes(16384, 4096) >= 148 * 4096 * 4
    P, S = _lib.ATS_MOE_PACKED, _lib.ATS_MOE_SLOTS
    assert lib.ats_moe_workspace_bytes(8192, 8, 2, 8192, P) > 0
    assert lib.ats_moe_workspace_bytes(8192, 8, 17, 8192, P) == 0  # k > 16 is invalid
    assert lib.ats_moe_workspace_bytes(8192, 8, 2, 8192, 7) == 0  # unknown layout
    mr = lib.ats_moe_max_rows(8192, 8, 2, 8192, P)
    assert mr % 128 == 0 and 16384 <= mr <= 16384 + 8 * 128
    # packed: kept rows plus per-expert padding; slots: E x capacity rounded to 128
    assert lib.ats_moe_max_rows(32768, 64, 2, 1280, P) <= 65536 + 64 * 128
    assert lib.ats_moe_max_rows(32768, 64, 2, 1280, S) == 64 * 1280
    assert lib.ats_moe_max_rows(1000, 4, 2, 300, S) == 4 * 384
    assert lib.ats_moe_ep_segments_bytes(8, 8) > 0


def test_errors_surface_as_python_exceptions():
    with pytest.raises(_lib.AtsError) as ei:
        _lib.call("ats_moe_topk", None, 4, 2, 3, None, None, None, None)
    assert ei.value.status == _lib.ATS_EBADARG


def test_library_is_sm100a_only():
    # the fatbin carries sm_100a code: the link line and the build flags say so
    from ats_v2_b200 import _build

    assert _build.ARCH == ["-gencode", "arch=compute_100a,code=sm_100a"]
    assert "--use_fast_math" not in _build.FLAGS
    assert isinstance(_lib.load(), ctypes.CDLL)
