"""ctypes binding of libhelm_b200.so (declared in include/helm_b200.h).

This module is the only place that touches the C ABI.  Loading fails loudly:
there is no Python or CPU fallback for any kernel.  The library is looked up
in-tree (helm_b200/lib/libhelm_b200.so) unless HELM_B200_LIB names another
file.
"""
from __future__ import annotations

import ctypes
import os
import pathlib

LIB_PATH = pathlib.Path(os.environ.get(
    "HELM_B200_LIB", pathlib.Path(__file__).resolve().parent / "lib" / "libhelm_b200.so"))

ABI_VERSION = 4

# helm_dtype
F32, F16, BF16, I8 = 0, 1, 2, 3

# status codes
OK, ERR_INVALID_ARGUMENT, ERR_UNSUPPORTED, ERR_WORKSPACE, ERR_CUDA = 0, 1, 2, 3, 4

# device error flag bits
DEVERR_PAGE_ID, DEVERR_PAGE_USED, DEVERR_NUM_PAGES, DEVERR_TIMEOUT, DEVERR_APPEND_FULL = 1, 2, 4, 8, 16

_c = ctypes
_p = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64


MAX_RANKS = 8


class ShardExchange(ctypes.Structure):
    _fields_ = [
        ("rank", _i32), ("world", _i32),
        ("peer_recv", _p * MAX_RANKS), ("peer_flags", _p * MAX_RANKS),
        ("recv_local", _p), ("flags_local", _p), ("counters", _p),
        ("wait_ns", ctypes.c_uint64),
    ]


class PagedAttnParams(ctypes.Structure):
    _fields_ = [
        ("q", _p), ("k_base", _p), ("v_base", _p),
        ("page_stride", _i64), ("head_stride", _i64),
        ("num_pool_pages", _i32),
        ("page_table", _p), ("page_used", _p), ("num_pages", _p),
        ("page_table_stride", _i32), ("max_pages", _i32),
        ("B", _i32), ("Hq", _i32), ("Hkv", _i32), ("D", _i32), ("P", _i32),
        ("q_dtype", _i32), ("kv_dtype", _i32), ("out_dtype", _i32),
        ("scale", ctypes.c_float),
        ("num_splits", _i32),
        ("workspace", _p), ("workspace_bytes", _i64),
        ("out", _p), ("out_record", _p),
        ("error_flag", _p),
        ("exchange", _c.POINTER(ShardExchange)),
    ]


class KVAppendParams(ctypes.Structure):
    _fields_ = [
        ("k_new", _p), ("v_new", _p), ("src_dtype", _i32),
        ("k_base", _p), ("v_base", _p),
        ("page_stride", _i64), ("head_stride", _i64),
        ("num_pool_pages", _i32), ("kv_dtype", _i32),
        ("B", _i32), ("Hkv", _i32), ("D", _i32), ("P", _i32),
        ("dest", _p), ("dest_host", _p), ("page_table", _p), ("page_used", _p), ("num_pages", _p),
        ("page_table_stride", _i32),
        ("spare_pages", _p), ("spare_next", _p), ("spare_stride", _i32),
        ("error_flag", _p),
    ]


class DecodePrologueParams(ctypes.Structure):
    _fields_ = [
        ("append", KVAppendParams),
        ("q_in", _p), ("q_out", _p), ("Hq", _i32),
        ("q_stride", _i64), ("k_stride", _i64), ("v_stride", _i64),
        ("q_norm_w", _p), ("k_norm_w", _p), ("norm_dtype", _i32), ("eps", ctypes.c_float),
        ("cos", _p), ("sin", _p), ("cs_dtype", _i32), ("cs_stride", _i64),
        ("do_append", _i32),
    ]


class KVPrefillParams(ctypes.Structure):
    _fields_ = [
        ("k_src", _p), ("v_src", _p), ("src_dtype", _i32),
        ("src_head_stride", _i64), ("src_tok_stride", _i64),
        ("k_base", _p), ("v_base", _p),
        ("page_stride", _i64), ("head_stride", _i64),
        ("num_pool_pages", _i32), ("kv_dtype", _i32),
        ("Hkv", _i32), ("D", _i32), ("P", _i32),
        ("pages", _p), ("count", _i32),
        ("page_table", _p), ("page_used", _p), ("num_pages", _p),
        ("page_table_stride", _i32), ("first_index", _i32),
        ("error_flag", _p),
    ]


class GatherMergeParams(ctypes.Structure):
    _fields_ = [
        ("rank", _i32), ("world", _i32), ("rows", _i32), ("D", _i32),
        ("record", _p),
        ("peer_recv", _p * MAX_RANKS), ("peer_flags", _p * MAX_RANKS),
        ("recv_local", _p), ("flags_local", _p), ("counters", _p),
        ("out", _p), ("out_dtype", _i32), ("out_record", _p), ("error_flag", _p),
        ("wait_ns", ctypes.c_uint64),
        ("num_partials", _i32), ("partial_stride", _i64),
    ]


# (name, restype, argtypes) for every entry point of include/helm_b200.h
SIGNATURES = [
    ("helm_abi_version", _c.c_int, []),
    ("helm_last_error", _c.c_char_p, []),
    ("helm_paged_attn_workspace_bytes", _i64, [_c.POINTER(PagedAttnParams), _c.POINTER(_i32)]),
    ("helm_paged_attn_decode", _c.c_int, [_c.POINTER(PagedAttnParams), _p]),
    ("helm_lse_merge", _c.c_int, [_p, _i32, _i64, _i32, _i32, _p, _i32, _p, _p]),
    ("helm_int8_linear", _c.c_int, [_p, _i32, _p, _p, _i32, _p, _p, _i32, _i32, _i32, _p]),
    ("helm_int8_linear_glu", _c.c_int, [_p, _i32, _p, _p, _i32, _p, _p, _i32, _i32, _i32, _p]),
    ("helm_int8_packed_bytes", _i64, [_i32, _i32]),
    ("helm_int8_pack_weight", _c.c_int, [_p, _i32, _i32, _p, _p]),
    ("helm_int8_linear_packed", _c.c_int, [_p, _i32, _p, _p, _i32, _p, _p, _i32, _i32, _i32, _p]),
    ("helm_int8_linear_glu_packed", _c.c_int, [_p, _i32, _p, _p, _i32, _p, _p, _i32, _i32, _i32, _p]),
    ("helm_int8_gemm_packed", _c.c_int, [_p, _i32, _p, _p, _i32, _p, _p, _i32, _i32, _i32, _p]),
    ("helm_int8_linear_error", _c.c_int, [_p, _i32]),
    ("helm_kv_append", _c.c_int, [_c.POINTER(KVAppendParams), _p]),
    ("helm_decode_prologue", _c.c_int, [_c.POINTER(DecodePrologueParams), _p]),
    ("helm_kv_write_pages", _c.c_int, [_c.POINTER(KVPrefillParams), _p]),
    ("helm_rmsnorm", _c.c_int, [_p, _i32, _i64, _p, _i32, _p, _i64, _i64, _i32, ctypes.c_float, _p]),
    ("helm_copy_pages", _c.c_int, [_p, _i64, _p, _p, _i32, _i64, _c.POINTER(_i32), _p]),
    ("helm_move_pages", _c.c_int, [_p, _p, _p, _p, _i32, _i64, _i64, _i64, _c.POINTER(_i32), _p]),
    ("helm_gather_merge_state_bytes", _i64, [_i32, _i32, _i32, _c.POINTER(_i64), _c.POINTER(_i64),
                                              _c.POINTER(_i64)]),
    ("helm_gather_merge", _c.c_int, [_c.POINTER(GatherMergeParams), _p]),
    ("helm_ipc_export", _c.c_int, [_p, _p, _c.POINTER(_i64)]),
    ("helm_ipc_import", _c.c_int, [_p, _i64, _c.POINTER(_p), _c.POINTER(_p)]),
    ("helm_ipc_close", _c.c_int, [_p]),
    ("helm_shard_exchange_bytes", _i64, [_i32, _i32, _i32, _c.POINTER(_i64), _c.POINTER(_i64),
                                          _c.POINTER(_i64)]),
]

_lib = None
_load_error: str | None = None


def _load():
    global _lib, _load_error
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        _load_error = f"{LIB_PATH} not found (build it with `python -m helm_b200.build_native`)"
        raise RuntimeError("helm_b200: native library missing: " + _load_error)
    try:
        lib = ctypes.CDLL(str(LIB_PATH))
    except OSError as e:  # pragma: no cover - depends on the host
        _load_error = str(e)
        raise RuntimeError(f"helm_b200: cannot load {LIB_PATH}: {e}") from e
    for name, res, args in SIGNATURES:
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    ver = lib.helm_abi_version()
    if ver != ABI_VERSION:
        _load_error = f"ABI version {ver} != {ABI_VERSION}"
        raise RuntimeError("helm_b200: " + _load_error)
    _lib = lib
    return lib


def lib():
    """The loaded library; raises RuntimeError when it is missing."""
    return _load()


def is_available() -> bool:
    try:
        _load()
        return True
    except RuntimeError:
        return False


def load_error() -> str | None:
    try:
        _load()
    except RuntimeError:
        pass
    return _load_error


class HelmError(RuntimeError):
    """A non-zero status from the C ABI."""

    def __init__(self, fn: str, code: int, msg: str):
        super().__init__(f"{fn} failed with status {code}: {msg}")
        self.code = code


def check(fn: str, code: int) -> None:
    if code != OK:
        msg = _load().helm_last_error()
        raise HelmError(fn, code, msg.decode() if msg else "")
