"""The C ABI's hot-path entry points as torch custom operators (``torch.ops.nanokv``).

The reference's selector, gather-attend, segmented prefill and paged-cache
store (``nanovllm/sparse/m12_runtime.py:959-1055, 845-896, 809-839``,
``nanovllm/layers/attention.py:11-41``) become operators with schemas and fake
(meta) implementations, so a caller can use them from torch code that is
traced or compiled, and the dispatcher sees their inputs, outputs and
mutations.  Each operator fills the same argument struct as
``M12LayerRuntime`` and calls the same entry point of ``libnanokv.so``; there
is no CPU implementation.

Layouts are the library's own (include/nanokv.h): q ``[nq, hq, D]``; the block
store ``[cap, hkv, B, D]`` bf16 in device memory; sink ``[hkv, S, D]``; recent
ring ``[hkv, R, D]`` (physical slots ``ring_start ..`` mod R); current tokens
``[nq, hkv, D]``; representatives ``[hkv, max_blocks, r, D]``.  ``attend`` and
``prefill`` write nothing but their output (no ring slot is written), so they
are functional; ``store_kvcache`` mutates its two caches.

    ops = importlib.import_module("nano-vllm-kv-optimizer_b200").torch_ops
    ids, scores = torch.ops.nanokv.select(q, reps, nblocks, protected_ids, 32)
    o = torch.ops.nanokv.attend(q, ids, k_store, v_store, sink_k, sink_v, 64,
                                ring_k, ring_v, ring_start, 512, k_cur, v_cur, scale)
"""
from __future__ import annotations

import ctypes as C
from typing import Tuple

import torch
from torch import Tensor

from . import _lib
from ._lib import AttendArgs, call

_WS: dict = {}  # (device index, stream handle, kind) -> zeroed workspace (kernels leave it zeroed)


def _stream(t: Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _workspace(t: Tensor, kind: str, nbytes: int) -> Tensor:
    key = (t.device.index, _stream(t), kind)
    ws = _WS.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=t.device)
        _WS[key] = ws
    return ws


def _rows(t: Tensor) -> Tensor:
    """16-byte aligned rows with unit innermost stride (what the kernels read)."""
    if t.stride(-1) == 1 and t.data_ptr() % 16 == 0 and all(s % 8 == 0 for s in t.stride()[:-1]):
        return t
    return t.contiguous()


def _check(name: str, cond: bool, msg: str) -> None:
    if not cond:
        raise ValueError(f"nanokv::{name}: {msg}")


@torch.library.custom_op("nanokv::select", mutates_args=(), device_types="cuda")
def select(q: Tensor, reps: Tensor, nblocks: int, protected_ids: Tensor, k: int) -> Tuple[Tensor, Tensor]:
    """Top-k block ids (int64, score descending, equal scores by ascending id)
    and their scores (fp32) of q ``[nq, hq, D]`` against the representatives
    ``[hkv, max_blocks, r, D]``; ``protected_ids`` (int32) score -inf
    (reference ``_gpu_select`` :999-1008; the caller applies the budget rule
    ``k = min(req, max(1, unprotected blocks))``)."""
    _check("select", q.dim() == 3 and reps.dim() == 4 and q.shape[2] == reps.shape[3], "bad shapes")
    _check("select", 1 <= k and 1 <= nblocks <= reps.shape[1], "bad k or nblocks")
    q = _rows(q)
    prot = protected_ids.to(device=q.device, dtype=torch.int32).contiguous()
    hkv, max_blocks, r, d = reps.shape
    ids = torch.empty(k, dtype=torch.int64, device=q.device)
    scores = torch.empty(k, dtype=torch.float32, device=q.device)
    ws = _workspace(q, "select", _lib.load().nkv_select_workspace_bytes(max_blocks, q.shape[0]))
    call("nkv_select", _stream(q), q.data_ptr(), q.shape[0], q.stride(0), q.stride(1), q.shape[1], hkv, d,
         reps.contiguous().data_ptr(), r, max_blocks, nblocks, prot.data_ptr(), prot.numel(), k, ids.data_ptr(),
         scores.data_ptr(), 0, ws.data_ptr(), ws.numel())
    return ids, scores


@select.register_fake
def _(q, reps, nblocks, protected_ids, k):
    return q.new_empty(k, dtype=torch.int64), q.new_empty(k, dtype=torch.float32)


def _segments(name, q, block_ids, k_store, v_store, sink_k, sink_v, sink_len, ring_k, ring_v, ring_start, ring_len,
              cur_k, cur_v, scale, prefill):
    _check(name, q.dim() == 3 and k_store.dim() == 4 and k_store.shape == v_store.shape, "bad shapes")
    _check(name, cur_k.shape == cur_v.shape and cur_k.shape[0] == q.shape[0], "one current token per query")
    _check(name, k_store.dtype == torch.bfloat16, "bf16 block store only")
    nq, hq, d = q.shape
    cap, hkv, B, _ = k_store.shape
    n_sel = block_ids.numel()
    q, cur_k, cur_v = _rows(q), _rows(cur_k), _rows(cur_v)
    if cur_k.stride() != cur_v.stride():
        cur_k, cur_v = cur_k.contiguous(), cur_v.contiguous()
    ids = block_ids.to(device=q.device, dtype=torch.int64).contiguous()
    k_store, v_store = k_store.contiguous(), v_store.contiguous()
    sink_k, sink_v, ring_k, ring_v = (t.contiguous() for t in (sink_k, sink_v, ring_k, ring_v))
    out = torch.empty(nq, hq, d, dtype=q.dtype, device=q.device)
    a = AttendArgs()
    a.q, a.q_row_stride, a.q_head_stride = q.data_ptr(), q.stride(0), q.stride(1)
    a.nq, a.hq, a.hkv, a.head_dim, a.block_size = nq, hq, hkv, d, B
    a.scale = float(scale)
    a.block_ids, a.n_sel = (ids.data_ptr() if n_sel else 0), n_sel
    a.max_blocks, a.store_kind = cap, _lib.STORE_BF16
    a.k_store, a.v_store = k_store.data_ptr(), v_store.data_ptr()
    a.sink_k, a.sink_v, a.sink_cap, a.sink_len = sink_k.data_ptr(), sink_v.data_ptr(), sink_k.shape[1], sink_len
    a.ring_k, a.ring_v, a.ring_cap = ring_k.data_ptr(), ring_v.data_ptr(), ring_k.shape[1]
    a.ring_start, a.ring_len = ring_start, ring_len
    a.cur_k, a.cur_v = cur_k.data_ptr(), cur_v.data_ptr()
    a.cur_row_stride, a.cur_head_stride = cur_k.stride(0), cur_k.stride(1)
    a.n_cur, a.ring_write_pos = nq, -1
    a.out, a.out_row_stride, a.out_head_stride = out.data_ptr(), out.stride(0), out.stride(1)
    ntok = n_sel * B + sink_len + ring_len + nq
    lib = _lib.load()
    nbytes = (lib.nkv_prefill_workspace_bytes if prefill else lib.nkv_attend_workspace_bytes)(hkv, hq, nq, ntok)
    ws = _workspace(q, "prefill" if prefill else "attend", nbytes)
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    call("nkv_prefill" if prefill else "nkv_attend", _stream(q), C.byref(a))
    return out


@torch.library.custom_op("nanokv::attend", mutates_args=(), device_types="cuda")
def attend(q: Tensor, block_ids: Tensor, k_store: Tensor, v_store: Tensor, sink_k: Tensor, sink_v: Tensor,
           sink_len: int, ring_k: Tensor, ring_v: Tensor, ring_start: int, ring_len: int, cur_k: Tensor,
           cur_v: Tensor, scale: float) -> Tensor:
    """One softmax of q ``[nq, hq, D]`` (nq <= 8: a decode step or a verify
    pass) over the selected blocks, the sink, the ring slice and the current
    tokens (query i sees current tokens 0..i): the reference's decode gather,
    pack and ``_fused_attention`` (m12_runtime.py:1213-1320, 845-896) without
    the ring append."""
    return _segments("attend", q, block_ids, k_store, v_store, sink_k, sink_v, sink_len, ring_k, ring_v, ring_start,
                     ring_len, cur_k, cur_v, scale, prefill=False)


@attend.register_fake
def _(q, block_ids, k_store, v_store, sink_k, sink_v, sink_len, ring_k, ring_v, ring_start, ring_len, cur_k, cur_v,
      scale):
    return q.new_empty(q.shape)


@torch.library.custom_op("nanokv::prefill", mutates_args=(), device_types="cuda")
def prefill(q: Tensor, block_ids: Tensor, k_store: Tensor, v_store: Tensor, sink_k: Tensor, sink_v: Tensor,
            sink_len: int, ring_k: Tensor, ring_v: Tensor, ring_start: int, ring_len: int, cur_k: Tensor,
            cur_v: Tensor, scale: float) -> Tensor:
    """A prefill chunk q ``[T, hq, D]`` over the same segments with the chunk
    causal (bottom-right): the reference's later-chunk pack +
    ``_prefill_attention`` (m12_runtime.py:589-642, 809-839); with no
    selected blocks, sink or ring it is the first chunk's dense causal
    attention."""
    return _segments("prefill", q, block_ids, k_store, v_store, sink_k, sink_v, sink_len, ring_k, ring_v, ring_start,
                     ring_len, cur_k, cur_v, scale, prefill=True)


@prefill.register_fake
def _(q, block_ids, k_store, v_store, sink_k, sink_v, sink_len, ring_k, ring_v, ring_start, ring_len, cur_k, cur_v,
      scale):
    return q.new_empty(q.shape)


@torch.library.custom_op("nanokv::store_kvcache", mutates_args=("k_cache", "v_cache"), device_types="cuda")
def store_kvcache(key: Tensor, value: Tensor, k_cache: Tensor, v_cache: Tensor, slot_mapping: Tensor) -> None:
    """k_cache[slot[i]] = key[i], v_cache[slot[i]] = value[i] for slot[i] != -1
    (the reference's Triton ``store_kvcache``, nanovllm/layers/attention.py:11-41);
    caches ``[slots, heads * D]`` bf16, key/value ``[N, heads, D]``."""
    n = key.shape[0]
    row = k_cache.shape[-1]
    _check("store_kvcache", key.shape == value.shape and key[0].numel() == row and k_cache.shape == v_cache.shape,
           "bad shapes")
    _check("store_kvcache", k_cache.is_contiguous() and v_cache.is_contiguous(), "caches must be contiguous")
    key, value = _rows(key.reshape(n, row)), _rows(value.reshape(n, row))
    slots = slot_mapping.to(device=key.device, dtype=torch.int64).contiguous()
    call("nkv_store_kvcache", _stream(key), key.data_ptr(), key.stride(0), value.data_ptr(), value.stride(0),
         k_cache.data_ptr(), v_cache.data_ptr(), slots.data_ptr(), n, row)


@store_kvcache.register_fake
def _(key, value, k_cache, v_cache, slot_mapping):
    return None
