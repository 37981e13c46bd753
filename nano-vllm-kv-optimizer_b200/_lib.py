"""ctypes binding of libnanokv.so (the C ABI declared in include/nanokv.h).

The library is built in-tree (``build.py``) and loaded from this directory.  A
missing library is a hard error: there is no CPU or eager fallback.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
# NKV_LIB=checked selects the bounds-checked debug build (libnanokv_checked.so);
# NKV_LIB=<path>.so loads another build of the same ABI (A/B comparisons)
_env_lib = os.environ.get("NKV_LIB", "")
LIB_PATH = (os.path.join(HERE, "libnanokv_checked.so") if _env_lib == "checked"
            else os.path.abspath(_env_lib) if _env_lib.endswith(".so")
            else os.path.join(HERE, "libnanokv.so"))

NKV_OK = 0
IPC_HANDLE_BYTES = 64
NKV_ERR_ARG = -1
NKV_ERR_UNSUPPORTED = -2
NKV_ERR_CUDA = -3
NKV_ERR_DEVICE = -4

STORE_BF16 = 0
STORE_INT8_REF = 1
STORE_INT8_TOKEN = 2

c_vp = C.c_void_p
c_i64 = C.c_int64
c_int = C.c_int


class AttendArgs(C.Structure):
    _fields_ = [
        ("q", c_vp), ("q_row_stride", c_i64), ("q_head_stride", c_i64),
        ("nq", c_int), ("hq", c_int), ("hkv", c_int), ("head_dim", c_int), ("block_size", c_int),
        ("scale", C.c_float),
        ("block_ids", c_vp), ("n_sel", c_int), ("max_blocks", c_int), ("store_kind", c_int),
        ("k_store", c_vp), ("v_store", c_vp),
        ("k_chan_scale", c_vp), ("v_block_scale", c_vp), ("k_tok_scale", c_vp), ("v_tok_scale", c_vp),
        ("allowed", c_vp), ("allowed_stride", c_int),
        ("sink_k", c_vp), ("sink_v", c_vp), ("sink_cap", c_int), ("sink_len", c_int),
        ("ring_k", c_vp), ("ring_v", c_vp), ("ring_cap", c_int), ("ring_start", c_int),
        ("ring_len", c_int),
        ("cur_k", c_vp), ("cur_v", c_vp), ("cur_row_stride", c_i64), ("cur_head_stride", c_i64),
        ("n_cur", c_int), ("ring_write_pos", c_int),
        ("out", c_vp), ("out_row_stride", c_i64), ("out_head_stride", c_i64),
        ("workspace", c_vp), ("workspace_bytes", C.c_size_t),
        ("overlap_select", c_int),
    ]


class DecodeArgs(C.Structure):
    _fields_ = [
        ("attend", AttendArgs),
        ("reps", c_vp), ("r", c_int), ("reps_blocks", c_int), ("nblocks", c_int),
        ("protected_ids", c_vp), ("n_protected", c_int), ("k", c_int),
        ("out_ids", c_vp), ("out_topk_scores", c_vp),
        ("select_workspace", c_vp), ("select_workspace_bytes", C.c_size_t),
        ("ring_head", c_vp),
    ]


class StoreArgs(C.Structure):
    _fields_ = [
        ("k", c_vp), ("v", c_vp),
        ("k_row_stride", c_i64), ("k_head_stride", c_i64),
        ("v_row_stride", c_i64), ("v_head_stride", c_i64),
        ("T", c_int), ("hkv", c_int), ("head_dim", c_int), ("block_size", c_int), ("r", c_int),
        ("start_block", c_int), ("max_blocks", c_int), ("store_blocks", c_int),
        ("store_kind", c_int),
        ("k_store", c_vp), ("v_store", c_vp),
        ("k_chan_scale", c_vp), ("v_block_scale", c_vp), ("k_tok_scale", c_vp), ("v_tok_scale", c_vp),
        ("reps", c_vp), ("rep_index", c_vp),
        ("sink_k", c_vp), ("sink_v", c_vp), ("sink_cap", c_int), ("sink_write", c_int),
        ("ring_k", c_vp), ("ring_v", c_vp), ("ring_cap", c_int), ("ring_pos0", c_int),
        ("ring_first", c_int),
    ]


# every symbol include/nanokv.h declares, with its ctypes signature
SIGNATURES = {
    "nkv_last_error": (C.c_char_p, []),
    "nkv_version": (c_int, []),
    "nkv_check": (c_int, [c_vp, c_vp]),
    "nkv_map_host": (c_int, [c_vp, C.POINTER(c_vp)]),
    "nkv_select_workspace_bytes": (C.c_size_t, [c_int, c_int]),
    "nkv_select": (c_int, [c_vp, c_vp, c_int, c_i64, c_i64, c_int, c_int, c_int, c_vp, c_int,
                           c_int, c_int, c_vp, c_int, c_int, c_vp, c_vp, c_vp, c_vp, C.c_size_t]),
    "nkv_select_per_query": (c_int, [c_vp, c_vp, c_int, c_i64, c_i64, c_int, c_int, c_int, c_vp,
                                     c_int, c_int, c_int, c_vp, c_int, c_int, c_vp, c_vp, c_vp,
                                     c_vp, c_vp, C.c_size_t]),
    "nkv_attend_workspace_bytes": (C.c_size_t, [c_int, c_int, c_int, c_int]),
    "nkv_attend": (c_int, [c_vp, C.POINTER(AttendArgs)]),
    "nkv_attend_last_config": (c_int, [C.POINTER(c_int), C.POINTER(c_int), C.POINTER(c_int)]),
    "nkv_attend_static": (c_int, [c_vp, C.POINTER(AttendArgs)]),
    "nkv_attend_static_check": (c_int, [c_vp]),
    "nkv_decode_step": (c_int, [c_vp, C.POINTER(DecodeArgs)]),
    "nkv_decode_last_form": (c_int, []),
    "nkv_reload_env": (None, []),
    "nkv_select_scores": (c_int, [c_vp, c_vp, c_i64, c_i64, c_int, c_int, c_int, c_vp, c_int, c_int, c_int,
                                  c_vp, c_int, c_vp, c_vp, C.c_size_t]),
    "nkv_attend_ranked": (c_int, [c_vp, C.POINTER(AttendArgs), c_vp, c_int, c_vp, c_vp]),
    "nkv_shard_exchange_bytes": (C.c_size_t, [c_int, c_int, c_int]),
    "nkv_peer_alloc": (c_int, [C.c_size_t, C.POINTER(c_vp), c_vp]),
    "nkv_peer_open": (c_int, [c_vp, C.POINTER(c_vp)]),
    "nkv_peer_close": (c_int, [c_vp]),
    "nkv_peer_free": (c_int, [c_vp]),
    "nkv_shard_scores": (c_int, [c_vp, c_vp, c_i64, c_i64, c_int, c_int, c_int, c_vp, c_int, c_int, c_int, c_vp, c_int,
                                 c_vp, c_int, c_int, c_vp, C.c_size_t]),
    "nkv_shard_attend": (c_int, [c_vp, C.POINTER(AttendArgs), c_vp, c_int, c_int, c_int, c_int, c_vp, c_vp, c_vp]),
    "nkv_prefill_workspace_bytes": (C.c_size_t, [c_int, c_int, c_int, c_int]),
    "nkv_prefill": (c_int, [c_vp, C.POINTER(AttendArgs)]),
    "nkv_prefill_gather": (c_int, [c_vp, C.POINTER(AttendArgs), c_vp, c_vp]),
    "nkv_store_chunk": (c_int, [c_vp, C.POINTER(StoreArgs)]),
    "nkv_ring_append": (c_int, [c_vp, c_vp, c_vp, c_int, c_i64, c_i64, c_i64, c_i64, c_int, c_int,
                                c_vp, c_vp, c_int, c_int]),
    "nkv_k_channel_scale": (c_int, [c_vp, c_vp, c_int, c_i64, c_i64, c_int, c_int, c_vp]),
    "nkv_query_summaries": (c_int, [c_vp, c_vp, c_int, c_i64, c_i64, c_int, c_int, c_int, c_vp]),
    "nkv_store_kvcache": (c_int, [c_vp, c_vp, c_i64, c_vp, c_i64, c_vp, c_vp, c_vp, c_int, c_int]),
    "nkv_selftest_div": (c_int, [c_vp, c_vp, c_vp, c_vp, c_int]),
    "nkv_qk_norm_rope": (c_int, [c_vp, c_vp, C.c_longlong, c_int, c_int, c_int, c_int, c_vp, c_vp, c_vp, c_vp,
                                 C.c_longlong, C.c_float, c_vp]),
    "nkv_add_rms_norm": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_int, C.c_float, c_int]),
    "nkv_silu_mul": (c_int, [c_vp, c_vp, c_vp, c_int, c_int]),
    "nkv_gemv_bf16": (c_int, [c_vp, c_vp, c_i64, c_int, c_vp, c_i64, c_int, c_int, c_vp, c_i64]),
}

_lib = None
_lock = threading.Lock()


class NanoKVError(RuntimeError):
    def __init__(self, fn: str, code: int, msg: str):
        super().__init__(f"{fn} failed ({code}): {msg}")
        self.code = code


class NanoKVUnsupported(NanoKVError, ValueError):
    """Geometry outside what the kernels are built for (no fallback exists)."""


def load(path: str | None = None):
    """Load (once) and return the ctypes library with signatures attached."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        p = path or LIB_PATH
        if not os.path.exists(p):
            raise ImportError(
                f"{p} is missing: build it with `python -c 'import __graft_entry__ as g; g.build()'` "
                "(the sparse path has no non-CUDA implementation)")
        lib = C.CDLL(p)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def call(name: str, *args):
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != NKV_OK:
        msg = lib.nkv_last_error().decode(errors="replace")
        cls = NanoKVUnsupported if rc == NKV_ERR_UNSUPPORTED else NanoKVError
        raise cls(name, rc, msg)
    return rc


def set_env(name: str, value) -> None:
    """Set (or, with None, remove) an NKV_* tuning variable and make the
    library read the environment again (it caches the variables)."""
    if value is None:
        os.environ.pop(name, None)
    else:
        os.environ[name] = str(value)
    if _lib is not None:
        _lib.nkv_reload_env()


def device_pointer(t) -> int:
    """Device address of a CUDA tensor, or of a pinned host tensor (mapped)."""
    if t.is_cuda:
        return t.data_ptr()
    out = c_vp()
    call("nkv_map_host", c_vp(t.data_ptr()), C.byref(out))
    return out.value


def attend_last_config():
    """(cluster, splits per head, keys per CTA) of the last nkv_attend launch."""
    a, b, c = c_int(), c_int(), c_int()
    call("nkv_attend_last_config", C.byref(a), C.byref(b), C.byref(c))
    return a.value, b.value, c.value
