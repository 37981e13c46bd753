"""The segmented-prefill operator seam: the reference's
``SegmentedPrefillAdapter`` contract (nanovllm/sparse/segmented_prefill_adapter.py:50-158)
on this package's prefill kernel.

``prepare(q, stage_k, stage_v, sink, recent, current)`` takes the four key
segments of a later prefill chunk -- the selected history (``stage_k/v``
[S, Hkv, D], pinned host staging or device memory, S a multiple of the block
size), the sink, the recent window and the current chunk (each a (k, v) pair
[L, Hkv, D] on the device) -- and returns a ``PrefillInvocation``;
``attend(invocation)`` returns o [Tq, Hq, D]: exact attention of every query
over [selected | sink | recent] and causally over the current chunk (the
bottom-right alignment of the reference's ``flash_attn_func(causal=True)``
for Sq < Sk).  Like the reference's adapter it owns no KV state or selection
and keeps one scratch set per device and stream, overwritten by the next
``prepare``.

The segments are re-laid out head-major on the device (the selected tokens as
a [blocks][Hkv][64][D] block store read through block ids 0..n-1, the sink
and recent window as head-major windows) and attended by the tcgen05 prefill
kernel (``nkv_prefill``; ``nkv_attend`` for up to 8 queries).  The reference's
``backend="operator"`` loads an external frozen operator package that is not
part of the reference repository; here ``backend="b200"`` (and
``"flash_reuse"``, the reference's exact-attention backend, as an alias) run
this kernel.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from . import _lib
from ._lib import AttendArgs, call


@dataclass(frozen=True)
class PrefillInvocation:
    q: torch.Tensor
    segments: tuple
    mode: str
    packed: tuple | None


class SegmentedPrefillAdapter:
    """Single-stream prefill scratch shared across sequential layers, with the
    reference adapter's ``prepare`` / ``attend`` / ``precompile`` / ``stats``."""

    BLOCK = 64

    def __init__(self, backend: str = "b200", scale: float = 128 ** -0.5,
                 geometry=(32, 8, 128, torch.bfloat16), operator_root=None):
        if backend not in ("b200", "flash_reuse"):
            raise ValueError("expected backend 'b200' (or 'flash_reuse'); the reference's external "
                             "'operator' package is not available")
        hq, hkv, dim, dtype = geometry
        if dim != 128 or dtype != torch.bfloat16 or hq % hkv:
            raise _lib.NanoKVUnsupported("SegmentedPrefillAdapter", _lib.NKV_ERR_UNSUPPORTED,
                                         f"geometry {geometry}: bf16, head_dim 128, hq a multiple of hkv")
        self.backend, self.scale, self.geometry = backend, float(scale), geometry
        self.stream = torch.cuda.current_stream()
        self.device = self.stream.device
        self.calls = self.scratch_builds = 0
        self._ws = None
        self._ids = None

    def _stream_check(self, device):
        if device != self.device or torch.cuda.current_stream(device).cuda_stream != self.stream.cuda_stream:
            raise ValueError("shared prefill scratch belongs to one CUDA device/stream")

    def precompile(self, tokens, lengths):
        return "b200"

    @staticmethod
    def _head_major(x: torch.Tensor) -> torch.Tensor:
        return x.permute(1, 0, 2).contiguous()

    def prepare(self, q, stage_k, stage_v, sink, recent, current) -> PrefillInvocation:
        self._stream_check(q.device)
        lengths = (stage_k.shape[0], sink[0].shape[0], recent[0].shape[0], current[0].shape[0])
        if stage_k.shape != stage_v.shape or current[0].shape[0] != q.shape[0]:
            raise ValueError("inconsistent selected/current lengths")
        if stage_k.device.type == "cpu" and (not stage_k.is_pinned() or not stage_v.is_pinned()):
            raise ValueError("selected CPU staging must be pinned")
        S = lengths[0]
        if S % self.BLOCK:
            raise ValueError(f"selected length {S} is not a multiple of the block size {self.BLOCK}")
        hq, hkv, dim, _ = self.geometry
        nblk = S // self.BLOCK
        sel = None
        if nblk:
            sk = stage_k.to(q.device, non_blocking=True)
            sv = stage_v.to(q.device, non_blocking=True)
            # token-major [S, Hkv, D] -> block store [blocks][Hkv][64][D]
            sel = tuple(t.view(nblk, self.BLOCK, hkv, dim).permute(0, 2, 1, 3).contiguous() for t in (sk, sv))
        sk_hm = tuple(self._head_major(t) for t in sink) if lengths[1] else None
        rc_hm = tuple(self._head_major(t) for t in recent) if lengths[2] else None
        self.scratch_builds += 1
        return PrefillInvocation(q, (sel, sink, recent, current), "b200", (sel, sk_hm, rc_hm))

    def attend(self, inv: PrefillInvocation) -> torch.Tensor:
        self._stream_check(inv.q.device)
        hq, hkv, dim, _ = self.geometry
        q = inv.q if (inv.q.stride(-1) == 1 and inv.q.data_ptr() % 16 == 0) else inv.q.contiguous()
        sel, sk_hm, rc_hm = inv.packed
        cur_k, cur_v = inv.segments[3]
        if cur_k.stride() != cur_v.stride() or cur_k.stride(-1) != 1:
            cur_k, cur_v = cur_k.contiguous(), cur_v.contiguous()
        nq = q.shape[0]
        nblk = 0 if sel is None else sel[0].shape[0]
        sink_len = 0 if sk_hm is None else sk_hm[0].shape[1]
        rlen = 0 if rc_hm is None else rc_hm[0].shape[1]
        if nblk and (self._ids is None or self._ids.numel() < nblk):
            self._ids = torch.arange(max(nblk, 64), dtype=torch.int64, device=q.device)
        out = torch.empty(nq, hq, dim, dtype=q.dtype, device=q.device)
        prefill = nq > 8
        a = AttendArgs()
        a.q, a.q_row_stride, a.q_head_stride = q.data_ptr(), q.stride(0), q.stride(1)
        a.nq, a.hq, a.hkv, a.head_dim, a.block_size = nq, hq, hkv, dim, self.BLOCK
        a.scale = self.scale
        a.block_ids, a.n_sel = (self._ids.data_ptr(), nblk) if nblk else (0, 0)
        a.max_blocks = max(nblk, 1)
        a.store_kind = _lib.STORE_BF16
        a.k_store, a.v_store = (sel[0].data_ptr(), sel[1].data_ptr()) if nblk else (0, 0)
        if sink_len:
            a.sink_k, a.sink_v = sk_hm[0].data_ptr(), sk_hm[1].data_ptr()
        a.sink_cap, a.sink_len = sink_len, sink_len
        if rlen:
            a.ring_k, a.ring_v = rc_hm[0].data_ptr(), rc_hm[1].data_ptr()
        a.ring_cap, a.ring_start, a.ring_len = rlen, 0, rlen
        a.cur_k, a.cur_v = cur_k.data_ptr(), cur_v.data_ptr()
        a.cur_row_stride, a.cur_head_stride = cur_k.stride(0), cur_k.stride(1)
        a.n_cur, a.ring_write_pos = cur_k.shape[0], -1
        a.out, a.out_row_stride, a.out_head_stride = out.data_ptr(), out.stride(0), out.stride(1)
        ntok = nblk * self.BLOCK + sink_len + rlen + cur_k.shape[0]
        lib = _lib.load()
        fn = "nkv_prefill_workspace_bytes" if prefill else "nkv_attend_workspace_bytes"
        need = getattr(lib, fn)(hkv, hq, nq, ntok)
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.zeros(need, dtype=torch.uint8, device=q.device)
        a.workspace, a.workspace_bytes = self._ws.data_ptr(), self._ws.numel()
        call("nkv_prefill" if prefill else "nkv_attend", self.stream.cuda_stream, C.byref(a))
        self.calls += 1
        return out

    def attend_runtime(self, rt, q, ids, k, v) -> torch.Tensor:
        """``M12LayerRuntime.prefill_chunk`` through this seam (``M12Config.prefill_adapter``):
        the runtime's segments in the reference's layout -- its selected blocks
        ``k_cpu[ids]`` as [n * 64, Hkv, D], the sink, the sink-deduplicated
        recent slice, the chunk -- then ``prepare`` and ``attend`` (the
        reference's prefill_chunk does the same with its CPU gather,
        m12_runtime.py:589-642)."""
        from .m12_runtime import prefill_recent_slice
        cfg = rt.cfg
        n = int(ids.numel())
        shape = (n * cfg.block_size, cfg.num_kv_heads, cfg.head_dim)
        if n:
            store_k, store_v = rt.k_cpu, rt.v_cpu
            idx = ids.to(store_k.device)
            sel_k, sel_v = store_k[idx].reshape(shape), store_v[idx].reshape(shape)
            if sel_k.device.type == "cpu":
                sel_k, sel_v = sel_k.pin_memory(), sel_v.pin_memory()
        else:
            sel_k = sel_v = torch.empty(shape, dtype=q.dtype, device=q.device)
        sink_len = min(cfg.sink_tokens, rt.valid_len)
        _, off, rlen = prefill_recent_slice(rt.valid_len, cfg.sink_tokens, cfg.recent_tokens)
        recent = (rt.recent_k[off:off + rlen], rt.recent_v[off:off + rlen])
        inv = self.prepare(q, sel_k, sel_v, (rt.sink_k[:sink_len], rt.sink_v[:sink_len]), recent, (k, v))
        return self.attend(inv)

    def check(self) -> None:
        """Raise if a kernel of the last calls reported an error (bounded wait, bad index)."""
        if self._ws is not None:
            call("nkv_check", self.stream.cuda_stream, self._ws.data_ptr())

    def stats(self):
        return dict(direct_calls=self.calls, fa2_calls=0, workspace_builds=self.scratch_builds,
                    shared_scratch_bytes=0 if self._ws is None else self._ws.numel())
