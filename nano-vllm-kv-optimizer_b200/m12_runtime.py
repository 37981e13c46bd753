"""Drop-in M12 sparse layer runtime for B200, backed by the libnanokv C ABI.

Mirrors the public surface of the reference's ``nanovllm/sparse/m12_runtime.py``
(``M12Config`` :98-166, ``M12LayerRuntime`` :169-1346 and the helpers :32-95):
same method names, arguments, state attributes and error behaviour, so that
``Attention.forward`` (reference ``nanovllm/layers/attention.py:64-99``) can call
it unchanged.

What differs is where the data lives and who computes:
  * history K/V stay resident in a block store ``[blocks, Hkv, B, D]`` in HBM
    (``kv_residency="hbm"``) or in pinned host memory mapped into the device
    address space (``"host"``, the offload mode), never gathered/packed;
  * sink and recent windows are head-major; the recent window is a ring buffer
    whose logical contents equal the reference's left-aligned buffer exactly
    (including its shift-on-decode behaviour), so no per-token memmove;
  * selection ids stay on the device between the select and attend kernels;
    nothing on the decode path synchronises with the host.
Every tensor operation of the sparse path goes through ``_lib`` (hand-written
sm_100a kernels).  There is no CPU or eager fallback: a geometry the kernels do
not support raises ``NanoKVUnsupported``.
"""
from __future__ import annotations

import ctypes as C
import math
from contextlib import nullcontext
from dataclasses import dataclass
from time import perf_counter

import torch

from . import _lib
from ._lib import AttendArgs, StoreArgs, call


# ----------------------------------------------------------------------------
# Helpers with the reference's exact semantics (pure host logic)
# ----------------------------------------------------------------------------
def prefill_recent_slice(valid_len: int, sink_tokens: int, recent_tokens: int) -> tuple[int, int, int]:
    """Part of the left-aligned recent window not already covered by the sink.

    Same contract as the reference (m12_runtime.py:32-50): returns
    ``(buffer_start, buffer_offset, length)`` for the logical suffix
    ``[max(0, valid_len - recent_tokens), valid_len)`` minus the sink prefix.
    """
    assert valid_len >= 0
    assert sink_tokens >= 0
    assert recent_tokens >= 0
    sink_len = min(sink_tokens, valid_len)
    held = min(recent_tokens, valid_len)
    start = valid_len - held
    first = max(sink_len, start)
    return start, first - start, valid_len - first


def prefill_query_summaries(q: torch.Tensor, nsegments: int) -> torch.Tensor:
    """Mean query of each of ``nsegments`` consecutive parts of the chunk.

    Reference m12_runtime.py:53-67.  On a CUDA bf16 input the means are computed
    by ``nkv_query_summaries`` (fp32 accumulation, bf16 result); other inputs
    (host tensors in tests) use the same definition through torch.
    """
    assert q.ndim == 3, "q must be [T, Hq, D]"
    assert nsegments > 0
    nsegments = min(nsegments, q.shape[0])
    if q.is_cuda and q.dtype == torch.bfloat16 and q.shape[-1] == 128:
        out = torch.empty(nsegments, q.shape[1], q.shape[2], dtype=q.dtype, device=q.device)
        qq = _aligned(q)
        call("nkv_query_summaries", _stream(q.device), qq.data_ptr(), qq.shape[0], qq.stride(0),
             qq.stride(1), qq.shape[1], qq.shape[2], nsegments, out.data_ptr())
        return out
    if nsegments == 1:
        return q.mean(dim=0, keepdim=True)
    return torch.stack([part.mean(dim=0) for part in torch.tensor_split(q, nsegments)])


def dynamic_top_k_from_scores(top_scores: torch.Tensor, max_k: int, target_mass: float) -> int:
    """Decode budget among {half, three quarters, all} of ``max_k`` candidates.

    Host-side heuristic with the reference's rule (m12_runtime.py:70-95).
    """
    assert top_scores.ndim == 1 and top_scores.device.type == "cpu"
    assert 0.0 < target_mass <= 1.0 and max_k > 0
    count = top_scores.numel()
    if count < max_k or count <= 1 or not bool(torch.isfinite(top_scores).all()):
        return count
    spread = top_scores.std(unbiased=False)
    if float(spread) <= 1e-6:
        return count
    mass = torch.softmax((top_scores - top_scores[0]) / spread, dim=0).cumsum(dim=0)
    for choice in sorted({max(1, (max_k + 1) // 2), max(1, (3 * max_k + 3) // 4), max_k}):
        if float(mass[choice - 1]) >= target_mass:
            return choice
    return max_k


# ----------------------------------------------------------------------------
# Recent-window ring arithmetic.  The reference keeps the recent window as a
# left-aligned buffer of R slots that it shifts (m12_runtime.py:488-503 on store,
# :1169-1172 on decode, :788-802 on commit).  Here logical slot i lives at ring
# position (head + i) % R, so every update is an O(new tokens) write.
# ----------------------------------------------------------------------------
def ring_append_plan(head: int, valid_len: int, T: int, R: int) -> tuple[int, int, int]:
    """Append T tokens (store / commit).  Returns (pos0, first, new_head):
    token i >= first goes to position (pos0 + i) % R."""
    old_len = min(R, valid_len)
    return (head + old_len) % R, max(0, T - R), (head + max(0, old_len + T - R)) % R


def ring_decode_plan(head: int, valid_len: int, R: int) -> tuple[int, int, int, int]:
    """Decode shift-and-append.  Returns (write_pos, start, length, new_head):
    the new token is written at write_pos; the attended window is ring
    positions (start + j) % R for j < length, followed by the new token."""
    rlen = min(R, valid_len + 1)
    new_head = (head + 1) % R
    return head, (new_head + R - rlen) % R, rlen - 1, new_head


def ring_slice_start(head: int, offset: int, R: int) -> int:
    """Ring position of logical slot ``offset``."""
    return (head + offset) % R


# ----------------------------------------------------------------------------
# Config
# ----------------------------------------------------------------------------
@dataclass
class M12Config:
    """Knobs of the sparse path; field names and defaults follow the reference
    (m12_runtime.py:98-147).  B200 additions are at the end."""

    block_size: int = 64
    r: int = 4
    recent_tokens: int = 512
    sink_tokens: int = 64
    top_k_blocks: int = 32
    prefill_top_k_blocks: int | None = None
    decode_top_k_blocks: int | None = None
    dynamic_top_k: bool = False
    dynamic_top_k_mass: float = 0.90
    decode_relative_a: float | None = None
    decode_relative_max_blocks: int = 48
    decode_relative_union: bool = False
    decode_query_window: int = 1
    fused_selector: bool = False          # accepted; selection is always the fused kernel
    quant_history: bool = False           # int8 history, reference scheme
    verify_union_blocks: int = 0
    fused_dequant: bool = False           # accepted; dequant is always fused into attention
    gather_sort: bool = False
    max_model_len: int = 131072
    num_heads: int = 32
    num_kv_heads: int = 8
    head_dim: int = 128
    dtype: torch.dtype = torch.bfloat16
    scale: float = 128.0 ** -0.5
    use_index_select: bool = True         # accepted; there is no host gather
    decode_kv_pipeline: bool = False      # accepted; there is no host gather
    selector_cuda_graph: bool = False     # accepted; whole steps are graph-capturable
    selector_static_mask: bool = False    # accepted; the protected list is cached on device
    check_finite_outputs: bool = False
    prefill_query_segments: int = 1
    prefill_attention_backend: str = "torch"
    prefill_adapter: object | None = None
    # ---- B200 additions ----
    kv_residency: str = "hbm"             # "hbm" | "host" (pinned, mapped: offload mode)
    quant_scheme: str = "reference"       # with quant_history: "reference" | "token"
    device: str | torch.device = "cuda"

    def __post_init__(self):
        if self.decode_kv_pipeline and not self.use_index_select:
            raise ValueError("decode_kv_pipeline requires use_index_select")
        for name, budget in (("prefill_top_k_blocks", self.prefill_top_k_blocks),
                             ("decode_top_k_blocks", self.decode_top_k_blocks)):
            if budget is not None and not 1 <= budget <= self.top_k_blocks:
                raise ValueError(f"{name} must be in [1, top_k_blocks]")
        if self.decode_relative_a is not None:
            if not 0.0 < self.decode_relative_a < 1.0:
                raise ValueError("decode_relative_a must be in (0, 1)")
            if self.decode_relative_max_blocks < 1:
                raise ValueError("decode_relative_max_blocks must be >= 1")
        if self.decode_query_window < 1:
            raise ValueError("decode_query_window must be >= 1")
        if self.fused_dequant and not self.quant_history:
            raise ValueError("fused_dequant requires quant_history")
        if self.kv_residency not in ("hbm", "host"):
            raise ValueError("kv_residency must be 'hbm' or 'host'")
        if self.quant_scheme not in ("reference", "token"):
            raise ValueError("quant_scheme must be 'reference' or 'token'")
        if self.prefill_attention_backend not in ("torch", "flash", "nkv"):
            raise ValueError(f"unknown prefill attention backend: {self.prefill_attention_backend!r}")


# ----------------------------------------------------------------------------
# small utilities
# ----------------------------------------------------------------------------
def _stream(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream_fast(device_index: int) -> int:
    """The current stream's handle without the device-object round trip."""
    if _raw_stream is not None:
        return _raw_stream(device_index)
    return torch.cuda.current_stream(device_index).cuda_stream


def _aligned(t: torch.Tensor) -> torch.Tensor:
    """The kernels read rows with 16-byte vector loads."""
    if (t.stride(-1) == 1 and t.data_ptr() % 16 == 0
            and all(s % 8 == 0 for s in t.stride()[:-1])):
        return t
    return t.contiguous()


def _ptr(t) -> int:
    return 0 if t is None else t.data_ptr()


def _trimmed(ids_dev: torch.Tensor, count_dev) -> torch.Tensor:
    """Host copy of device ids, cut to a device-held count when there is one."""
    ids = ids_dev.cpu()
    return ids if count_dev is None else ids[:int(count_dev.cpu()[0])]


class M12LayerRuntime:
    """Per-layer block-sparse attention runtime (reference m12_runtime.py:169)."""

    def __init__(self, layer_id: int, cfg: M12Config):
        self.layer_id = layer_id
        self.cfg = cfg
        self.enabled = True
        dev = torch.device(cfg.device)
        if dev.type != "cuda":
            raise ValueError("M12LayerRuntime runs on CUDA devices only")
        if dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        if cfg.dtype != torch.bfloat16 or cfg.head_dim != 128:
            raise _lib.NanoKVUnsupported(
                "M12LayerRuntime", _lib.NKV_ERR_UNSUPPORTED,
                "kernels are built for bf16 activations with head_dim 128")
        if cfg.num_heads % cfg.num_kv_heads or cfg.num_heads // cfg.num_kv_heads not in (1, 2, 4, 8):
            raise _lib.NanoKVUnsupported("M12LayerRuntime", _lib.NKV_ERR_UNSUPPORTED,
                                         "query heads per kv head must be 1, 2, 4 or 8")
        if cfg.block_size not in (16, 32, 64, 128):
            raise _lib.NanoKVUnsupported("M12LayerRuntime", _lib.NKV_ERR_UNSUPPORTED,
                                         "block_size must be 16, 32, 64 or 128")
        if cfg.recent_tokens < 1:
            raise ValueError("recent_tokens must be >= 1 (decode appends into it)")
        _lib.load()
        B, Hkv, D = cfg.block_size, cfg.num_kv_heads, cfg.head_dim
        self.max_blocks = (cfg.max_model_len + B - 1) // B
        self.groups_per_kv = cfg.num_heads // cfg.num_kv_heads
        kw = dict(device=dev)

        # ---- block store (lazily grown, like the reference's host history) ----
        self.quant_history = cfg.quant_history
        if cfg.quant_history:
            self.store_kind = _lib.STORE_INT8_REF if cfg.quant_scheme == "reference" else _lib.STORE_INT8_TOKEN
        else:
            self.store_kind = _lib.STORE_BF16
        self._k_store = self._v_store = None
        self._k_tok_scale = self._v_tok_scale = None
        self.v_scale_cpu = None          # reference name; [cap, Hkv] fp32 (INT8_REF)
        self.cpu_blocks_cap = 0
        self.nblocks_filled = 0
        self._store_views = None
        self._store_ptrs = (0, 0)

        # ---- representatives [Hkv, max_blocks, r, D] --------------------------
        self.reps_gpu = torch.empty(Hkv, self.max_blocks, cfg.r, D, dtype=cfg.dtype, **kw)
        self.rep_index = torch.zeros(Hkv, self.max_blocks, cfg.r, dtype=torch.int16, **kw)

        # ---- sink and recent ring, head-major -----------------------------------
        self._sink_k = torch.zeros(Hkv, cfg.sink_tokens, D, dtype=cfg.dtype, **kw)
        self._sink_v = torch.zeros(Hkv, cfg.sink_tokens, D, dtype=cfg.dtype, **kw)
        self._ring_k = torch.zeros(Hkv, cfg.recent_tokens, D, dtype=cfg.dtype, **kw)
        self._ring_v = torch.zeros(Hkv, cfg.recent_tokens, D, dtype=cfg.dtype, **kw)
        self._ring_head = 0              # physical slot of logical recent[0]

        sel_budget = cfg.top_k_blocks
        if cfg.decode_relative_a is not None:
            sel_budget = max(sel_budget, cfg.decode_relative_max_blocks)
        if cfg.verify_union_blocks > 0:
            sel_budget = max(sel_budget, cfg.verify_union_blocks)
        self.max_selected_tokens = sel_budget * B
        self.packed_total = self.max_selected_tokens + cfg.sink_tokens + cfg.recent_tokens

        # ---- int8 scales --------------------------------------------------------
        self.k_scale = None              # [Hkv, D] fp32 (INT8_REF), fixed by the first chunk

        # ---- device-side selection outputs and workspaces -----------------------
        self._ids = torch.zeros(max(sel_budget, 8 * cfg.top_k_blocks), dtype=torch.int64, **kw)
        self._topk_scores = torch.zeros_like(self._ids, dtype=torch.float32)
        self._union_count = torch.zeros(1, dtype=torch.int32, **kw)
        self._allowed = torch.zeros(8, 8 * cfg.top_k_blocks, dtype=torch.uint8, **kw)
        self._prot_key = None
        self._dargs, self._dkey, self._ids_view = None, None, None
        # prefill over int8 or host-resident history: the selected blocks are
        # staged in device bf16 once per call (nkv_prefill_gather) and attended
        # on the tensor-core kernel; False attends them in place
        self.prefill_gather = True
        self._stage = None
        self._bscores = None
        self._lib_h = _lib.load()
        # nkv_decode_step taking the argument struct's address (no ctypes byref per call)
        self._step_fn = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_void_p)(
            C.cast(self._lib_h.nkv_decode_step, C.c_void_p).value)
        # the single-call decode applies when no selection variant is configured
        self._fast_ok = (cfg.decode_relative_a is None and not cfg.dynamic_top_k and not cfg.gather_sort
                         and cfg.decode_query_window <= 1)
        self._decode_requested = cfg.top_k_blocks if cfg.decode_top_k_blocks is None else cfg.decode_top_k_blocks
        self._budget_key, self._budget_val = None, 0
        self._dev_index = self.device.index
        # the timing record of the fast decode path (the same keys as the reference's)
        self._fast_timings = {
            "selector_ms": 0.0, "selector_enqueue_ms": 0.0,
            "d2h_ms": 0.0, "cpu_gather_ms": 0.0, "h2d_pack_ms": 0.0,
            "h2d_event_spans_cpu_gather": False, "recent_ms": 0.0,
            "packed_attn_ms": 0.0, "selected_tokens": 0, "total_attend_tokens": 0,
        }
        self._prot_dev = torch.zeros(1, dtype=torch.int32, **kw)
        self._n_prot_dev = 0
        self._sel_ws = None
        self._att_ws = None
        self._qwin = None
        self._qwin_count = 0
        # device address of a device-resident ring head ({head, arrivals}
        # int32), set only while a DeviceRingHeads recording captures this
        # layer's decode
        self._ring_dev_ptr = 0
        self._ring_ptr_in_args = 0
        # output tensor of the next fast decode calls instead of a new one (set
        # only while a DeviceRingHeads recording writes into stacked outputs)
        self._out_override = None

        # ---- state ---------------------------------------------------------------
        self.valid_len = 0
        self.prefill_len = 0
        self._last_ids_dev = None
        self._last_ids_host = None
        self.protected_blocks: set[int] = set()
        self.timings: dict[str, float] = {}
        self.last_prefill_query_summaries = 0
        self.last_prefill_block_ids: torch.Tensor | None = None
        self.prefill_cpu_gather_ms = 0.0
        self.profile_cuda_stages = False
        self.cuda_stage_events: dict = {}
        self.profile_torch_stages = False
        self.profile_nsys_stages = False
        self.record_ids = False
        self.ids_history: list[list[int]] = []
        self.record_q = False
        self.q_history: list[torch.Tensor] = []
        self._pending_k = None
        self._pending_v = None
        self._last_verify_dev = self._last_verify_host = self._last_verify_count = None
        self._last_ids_count = None
        self.last_verify_timings: dict = {}
        self.verify_mode = False
        self.verify_lossless = False
        self.use_index_select = cfg.use_index_select
        self._reps_version = 0
        self.selector_graph_setup_ms = 0.0
        self.selector_graph_builds = 0

    # ------------------------------------------------------------------
    # reference-layout views
    # ------------------------------------------------------------------
    @property
    def sink_k(self):
        return self._sink_k.permute(1, 0, 2)

    @property
    def sink_v(self):
        return self._sink_v.permute(1, 0, 2)

    @property
    def recent_k(self):
        """Logical left-aligned recent window [R, Hkv, D] (a gathered copy)."""
        return self._logical_ring(self._ring_k)

    @property
    def recent_v(self):
        return self._logical_ring(self._ring_v)

    def _logical_ring(self, ring):
        R = self.cfg.recent_tokens
        idx = (torch.arange(R, device=ring.device) + self._ring_head) % R
        return ring[:, idx].permute(1, 0, 2)

    @property
    def k_cpu(self):
        """History block store in the reference's block-major layout [cap, B, Hkv, D]."""
        return None if self._store_views is None else self._store_views[0]

    @property
    def v_cpu(self):
        return None if self._store_views is None else self._store_views[1]

    @property
    def last_block_ids(self):
        if self._last_ids_host is None and self._last_ids_dev is not None:
            self._last_ids_host = _trimmed(self._last_ids_dev, self._last_ids_count)
        return self._last_ids_host

    @last_block_ids.setter
    def last_block_ids(self, value):
        self._last_ids_dev = self._last_ids_count = None
        self._last_ids_host = value

    def _set_last_ids(self, ids_dev, count_dev=None):
        self._last_ids_dev, self._last_ids_count = ids_dev, count_dev
        self._last_ids_host = None

    @property
    def last_verify_block_ids(self):
        """The blocks the last verify pass attended (host int64), copied from
        the device when first read, so that a verify pass does not wait for
        the device."""
        if self._last_verify_host is None and self._last_verify_dev is not None:
            self._last_verify_host = _trimmed(self._last_verify_dev, self._last_verify_count)
        return self._last_verify_host

    @last_verify_block_ids.setter
    def last_verify_block_ids(self, value):
        self._last_verify_dev = self._last_verify_count = None
        self._last_verify_host = value

    # ------------------------------------------------------------------
    # lifecycle
    # ------------------------------------------------------------------
    def reset(self) -> None:
        """Start a new sequence, keeping every buffer (reference :322-349).

        The recent ring restarts at physical slot 0, so a reused runtime lays
        out its next sequence exactly as a fresh one (the decode kernels tile
        the ring by physical runs)."""
        self.nblocks_filled = 0
        self.valid_len = 0
        self._ring_head = 0
        self.prefill_len = 0
        self._last_ids_dev = self._last_ids_host = None
        self.protected_blocks.clear()
        self.timings.clear()
        self.last_prefill_query_summaries = 0
        self.last_prefill_block_ids = None
        self.prefill_cpu_gather_ms = 0.0
        self.cuda_stage_events.clear()
        self.ids_history.clear()
        self.q_history.clear()
        self._qwin_count = 0
        self.k_scale = None
        self._pending_k = None
        self._pending_v = None
        self.last_verify_block_ids = None
        self.selector_graph_setup_ms = 0.0
        self.selector_graph_builds = 0

    def _alloc_store(self, cap: int):
        cfg = self.cfg
        B, Hkv, D = cfg.block_size, cfg.num_kv_heads, cfg.head_dim
        int8 = self.store_kind != _lib.STORE_BF16
        dt = torch.int8 if int8 else cfg.dtype
        shape = (cap, Hkv, B, D)
        if cfg.kv_residency == "hbm":
            k = torch.empty(shape, dtype=dt, device=self.device)
            v = torch.empty(shape, dtype=dt, device=self.device)
        else:
            # pinned host memory; with unified addressing its host pointer is
            # also a valid device pointer (mapped, zero-copy)
            k = torch.empty(shape, dtype=dt, pin_memory=True)
            v = torch.empty(shape, dtype=dt, pin_memory=True)
        old = (self._k_store, self._v_store)
        n_old = self.nblocks_filled
        if old[0] is not None and n_old > 0:
            k[:n_old].copy_(old[0][:n_old])
            v[:n_old].copy_(old[1][:n_old])
        self._k_store, self._v_store = k, v
        self._store_ptrs = (_lib.device_pointer(k), _lib.device_pointer(v))
        if self.store_kind == _lib.STORE_INT8_REF:
            vs = torch.zeros(cap, Hkv, dtype=torch.float32, device=self.device)
            if self.v_scale_cpu is not None and n_old > 0:
                vs[:n_old].copy_(self.v_scale_cpu[:n_old])
            self.v_scale_cpu = vs
        elif self.store_kind == _lib.STORE_INT8_TOKEN:
            ks = torch.zeros(cap, Hkv, B, dtype=torch.bfloat16, device=self.device)
            vs = torch.zeros(cap, Hkv, B, dtype=torch.bfloat16, device=self.device)
            if self._k_tok_scale is not None and n_old > 0:
                ks[:n_old].copy_(self._k_tok_scale[:n_old])
                vs[:n_old].copy_(self._v_tok_scale[:n_old])
            self._k_tok_scale, self._v_tok_scale = ks, vs
        self.cpu_blocks_cap = cap
        self._store_views = (k.permute(0, 2, 1, 3), v.permute(0, 2, 1, 3))

    def reserve_blocks(self, nblocks: int):
        """Preallocate the block store for ``nblocks`` blocks (reference :400-415)."""
        need = min(nblocks, self.max_blocks)
        if self._k_store is None or self.cpu_blocks_cap < need:
            self._alloc_store(need)

    def _ensure_store(self, need: int):
        if need > self.max_blocks:
            raise ValueError(f"history of {need} blocks exceeds max_model_len")
        if self._k_store is None or self.cpu_blocks_cap < need:
            self._alloc_store(min(self.max_blocks, max(need, 2 * (self.cpu_blocks_cap or 1))))

    def _select_ws(self, nq: int):
        need = _lib.load().nkv_select_workspace_bytes(self.max_blocks, nq)
        if self._sel_ws is None or self._sel_ws.numel() < need:
            self._sel_ws = torch.zeros(need, dtype=torch.uint8, device=self.device)
        return self._sel_ws

    def _attend_ws(self, nq: int, ntok: int, prefill: bool = False):
        fn = "nkv_prefill_workspace_bytes" if prefill else "nkv_attend_workspace_bytes"
        cfg = self.cfg
        need = getattr(_lib.load(), fn)(cfg.num_kv_heads, cfg.num_heads, nq, ntok)
        if self._att_ws is None or self._att_ws.numel() < need:
            # counters must start at zero; kernels reset them after use
            self._att_ws = torch.zeros(need, dtype=torch.uint8, device=self.device)
        return self._att_ws

    def _protected_dev(self, nblocks: int):
        ids = tuple(sorted(p for p in self.protected_blocks if 0 <= p < nblocks))
        if ids != self._prot_key:
            self._prot_key = ids
            if ids:
                self._prot_dev = torch.tensor(ids, dtype=torch.int32).to(self.device, non_blocking=True)
            self._n_prot_dev = len(ids)
        return self._prot_dev, self._n_prot_dev

    def _profile_range(self, name: str):
        if self.profile_torch_stages:
            return torch.profiler.record_function(f"m12.{name}")
        if self.profile_nsys_stages:
            return torch.cuda.nvtx.range(f"m12.{name}.layer{self.layer_id}")
        return nullcontext()

    # ------------------------------------------------------------------
    # store (reference _store_kv :420-513 + _build_reps_gpu :354-395)
    # ------------------------------------------------------------------
    def _build_reps_gpu(self, k_blocks: torch.Tensor, start: int, nblocks: int):
        """Rebuild representatives of ``nblocks`` blocks from [N, B, Hkv, D] keys.

        Reference :354-395.  Runs the store kernel in reps-only mode (block store
        untouched)."""
        self._reps_version += 1
        cfg = self.cfg
        kb = k_blocks[:nblocks].reshape(nblocks * cfg.block_size, cfg.num_kv_heads, cfg.head_dim)
        self._launch_store(kb, kb, start, reps_only=True)

    def _launch_store(self, k, v, start_block, reps_only=False, sink_write=0,
                      ring_pos0=0, ring_first=None):
        cfg = self.cfg
        k, v = _aligned(k), _aligned(v)
        T = k.shape[0]
        a = StoreArgs()
        a.k, a.v = k.data_ptr(), v.data_ptr()
        a.k_row_stride, a.k_head_stride = k.stride(0), k.stride(1)
        a.v_row_stride, a.v_head_stride = v.stride(0), v.stride(1)
        a.T, a.hkv, a.head_dim, a.block_size, a.r = T, cfg.num_kv_heads, cfg.head_dim, cfg.block_size, cfg.r
        a.start_block = start_block
        a.max_blocks = self.max_blocks
        if reps_only:
            a.store_kind = _lib.STORE_BF16
            a.k_store = a.v_store = 0
        else:
            a.store_blocks = self.cpu_blocks_cap
            a.store_kind = self.store_kind
            a.k_store, a.v_store = self._store_ptrs
            a.k_chan_scale = _ptr(self.k_scale)
            a.v_block_scale = _ptr(self.v_scale_cpu) if self.store_kind == _lib.STORE_INT8_REF else 0
            a.k_tok_scale = _ptr(self._k_tok_scale)
            a.v_tok_scale = _ptr(self._v_tok_scale)
        a.reps = self.reps_gpu.data_ptr()
        a.rep_index = self.rep_index.data_ptr()
        a.sink_k, a.sink_v = self._sink_k.data_ptr(), self._sink_v.data_ptr()
        a.sink_cap, a.sink_write = cfg.sink_tokens, sink_write
        if reps_only:
            a.ring_cap = 0
        else:
            a.ring_k, a.ring_v = self._ring_k.data_ptr(), self._ring_v.data_ptr()
            a.ring_cap, a.ring_pos0 = cfg.recent_tokens, ring_pos0
            a.ring_first = ring_first if ring_first is not None else max(0, T - cfg.recent_tokens)
        call("nkv_store_chunk", _stream(self.device), C.byref(a))

    def _store_kv(self, k: torch.Tensor, v: torch.Tensor):
        """Append a prefill chunk (reference :420-513)."""
        cfg = self.cfg
        B, R = cfg.block_size, cfg.recent_tokens
        T = k.shape[0]
        assert T >= 2
        nb = -(-T // B)
        start = self.nblocks_filled
        need = start + nb
        self._ensure_store(need)
        if self.store_kind == _lib.STORE_INT8_REF and self.k_scale is None:
            self.k_scale = torch.empty(cfg.num_kv_heads, cfg.head_dim, dtype=torch.float32,
                                       device=self.device)
            kk = _aligned(k)
            call("nkv_k_channel_scale", _stream(self.device), kk.data_ptr(), T, kk.stride(0),
                 kk.stride(1), cfg.num_kv_heads, cfg.head_dim, self.k_scale.data_ptr())
        sink_write = min(cfg.sink_tokens, T) if self.prefill_len == 0 else 0
        self._reps_version += 1
        pos0, first, new_head = ring_append_plan(self._ring_head, self.valid_len, T, R)
        self._launch_store(k, v, start, sink_write=sink_write, ring_pos0=pos0, ring_first=first)
        self._ring_head = new_head
        self.valid_len += T
        self.prefill_len += T
        self.nblocks_filled = need
        n_recent_blocks = R // B
        self.protected_blocks = {0} | set(range(max(1, need - n_recent_blocks), need))

    # ------------------------------------------------------------------
    # selection (reference _gpu_select :959-1055, per-query :1057-1087)
    # ------------------------------------------------------------------
    def _budget(self, requested: int) -> int:
        nblocks = self.nblocks_filled
        key = (nblocks, requested, len(self.protected_blocks))
        if key == self._budget_key:
            return self._budget_val
        n_prot = len([p for p in self.protected_blocks if p < nblocks])
        kk = min(requested, max(1, nblocks - n_prot))
        self._budget_key, self._budget_val = key, kk
        return kk

    def _select_dev(self, q: torch.Tensor, k: int, block_scores=None):
        """Launch the select kernel; returns the device ids view [k]."""
        cfg = self.cfg
        if q.ndim == 2:
            q = q.unsqueeze(0)
        assert q.ndim == 3 and tuple(q.shape[1:]) == (cfg.num_heads, cfg.head_dim)
        if q.dtype != torch.bfloat16:
            q = q.to(torch.bfloat16)
        q = _aligned(q)
        nblocks = self.nblocks_filled
        prot, nprot = self._protected_dev(nblocks)
        if k > self._ids.numel():
            self._ids = torch.zeros(k, dtype=torch.int64, device=self.device)
            self._topk_scores = torch.zeros(k, dtype=torch.float32, device=self.device)
        ws = self._select_ws(1)
        call("nkv_select", _stream(self.device), q.data_ptr(), q.shape[0], q.stride(0), q.stride(1),
             cfg.num_heads, cfg.num_kv_heads, cfg.head_dim, self.reps_gpu.data_ptr(), cfg.r,
             self.max_blocks, nblocks, prot.data_ptr(), nprot, k, self._ids.data_ptr(),
             self._topk_scores.data_ptr(), _ptr(block_scores), ws.data_ptr(), ws.numel())
        ids = self._ids[:k]
        if cfg.gather_sort and k > 1:
            ids = ids.sort().values
        return ids

    def _gpu_select(self, q: torch.Tensor, *, dynamic: bool = False, budget: int | None = None,
                    use_graph: bool = False, use_static_mask: bool = False,
                    use_relative: bool = False) -> tuple[torch.Tensor, dict]:
        """Global Top-K block selection; returns (host int64 ids, info).

        Same contract as the reference (:959-1055).  ``use_graph`` and
        ``use_static_mask`` are accepted (the kernel path is already one launch
        with a cached protected list)."""
        cfg = self.cfg
        requested = cfg.top_k_blocks if budget is None else budget
        k = self._budget(requested)
        t0 = perf_counter()
        if use_relative:
            ids_dev, k = self._relative_select(q, k)
        else:
            ids_dev = self._select_dev(q, k)
        t1 = perf_counter()
        chosen = k
        if dynamic and cfg.dynamic_top_k and k == requested:
            chosen = dynamic_top_k_from_scores(self._topk_scores[:k].cpu(), requested,
                                               cfg.dynamic_top_k_mass)
        ids_cpu = ids_dev.cpu()[:chosen]
        info = {"d2h_ms": (perf_counter() - t1) * 1000.0, "enqueue_ms": (t1 - t0) * 1000.0,
                "n_selected": chosen, "n_candidates": k,
                "n_query_summaries": 1 if q.ndim == 2 else q.shape[0]}
        return ids_cpu, info

    def _relative_select(self, q, k):
        """Relative-threshold selection (reference :1015-1031): candidates are the
        best ``cap`` blocks; keep those within ln(a)/scale of the best."""
        cfg = self.cfg
        nblocks = self.nblocks_filled
        n_prot = len([p for p in self.protected_blocks if p < nblocks])
        cap = min(cfg.decode_relative_max_blocks, max(1, nblocks - n_prot))
        cand = self._select_dev(q, cap)
        scores = self._topk_scores[:cap]
        threshold = float(scores[0].item()) + math.log(cfg.decode_relative_a) / cfg.scale
        above = scores >= threshold
        if cfg.decode_relative_union:
            above = above | (torch.arange(cap, device=self.device) < k)
        keep = cand[above]
        if keep.numel() == 0:
            keep = cand[:k]
        return keep, int(keep.numel())

    def _gpu_select_per_query(self, q: torch.Tensor, k: int):
        """Per-query Top-K, sorted union and allowed mask (reference :1057-1087).

        Returns (union ids on the host, allowed [Tq, U] bool on the device)."""
        union_cpu, allowed, _ = self._select_per_query_dev(q, k)
        return union_cpu, allowed

    def _select_per_query_padded(self, q: torch.Tensor, k: int):
        """The per-query selection without a device wait: the sorted union's
        ids and allowed mask padded to Tq * k entries (past the union count,
        block 0 allowed for no query: keys that contribute nothing), and the
        device-held union count."""
        written = self._select_per_query_launch(q, k)
        E = written.shape[1]
        live = torch.arange(E, device=self.device) < self._union_count  # device-side compare
        ids = torch.where(live, self._ids[:E], 0)
        allowed = written.bool() & live
        return ids, allowed, self._union_count

    def _select_per_query_dev(self, q: torch.Tensor, k: int):
        written = self._select_per_query_launch(q, k)
        U = int(self._union_count.item())
        union = self._ids[:U].clone()
        return union.cpu(), written[:, :U].bool(), union

    def _select_per_query_launch(self, q: torch.Tensor, k: int):
        cfg = self.cfg
        if q.ndim == 2:
            q = q.unsqueeze(0)
        q = _aligned(q)
        Tq = q.shape[0]
        kk = self._budget(int(k))
        nblocks = self.nblocks_filled
        prot, nprot = self._protected_dev(nblocks)
        E = Tq * kk
        if self._ids.numel() < E:
            self._ids = torch.zeros(E, dtype=torch.int64, device=self.device)
        if self._allowed.shape[0] < Tq or self._allowed.shape[1] < E:
            self._allowed = torch.zeros(max(8, Tq), max(E, self._allowed.shape[1]),
                                        dtype=torch.uint8, device=self.device)
        allowed = self._allowed[:Tq, :E]
        allowed = allowed if allowed.is_contiguous() else allowed.contiguous()
        ws = self._select_ws(Tq)
        call("nkv_select_per_query", _stream(self.device), q.data_ptr(), Tq, q.stride(0), q.stride(1),
             cfg.num_heads, cfg.num_kv_heads, cfg.head_dim, self.reps_gpu.data_ptr(), cfg.r,
             self.max_blocks, nblocks, prot.data_ptr(), nprot, kk, self._ids.data_ptr(),
             self._union_count.data_ptr(), allowed.data_ptr(), 0, ws.data_ptr(), ws.numel())
        return allowed  # [Tq, Tq * k] dense: the tensor the kernel wrote

    # ------------------------------------------------------------------
    # attention launches
    # ------------------------------------------------------------------
    def _attend(self, q, ids_dev, n_sel, sink_len, ring_start, ring_len, cur_k, cur_v,
                ring_write_pos=-1, allowed=None, prefill=False, after_select=False):
        cfg = self.cfg
        q = _aligned(q)
        nq = q.shape[0]
        n_cur = 0 if cur_k is None else cur_k.shape[0]
        if cur_k is not None:
            cur_k, cur_v = _aligned(cur_k), _aligned(cur_v)
            if cur_k.stride() != cur_v.stride():
                cur_k, cur_v = cur_k.contiguous(), cur_v.contiguous()
        out = torch.empty(nq, cfg.num_heads, cfg.head_dim, dtype=q.dtype, device=q.device)
        ntok = n_sel * cfg.block_size + sink_len + ring_len + n_cur
        a = AttendArgs()
        a.q, a.q_row_stride, a.q_head_stride = q.data_ptr(), q.stride(0), q.stride(1)
        a.nq, a.hq, a.hkv, a.head_dim, a.block_size = nq, cfg.num_heads, cfg.num_kv_heads, cfg.head_dim, cfg.block_size
        a.scale = cfg.scale
        a.block_ids, a.n_sel = _ptr(ids_dev) if n_sel else 0, n_sel
        a.max_blocks = self.cpu_blocks_cap
        a.store_kind = self.store_kind
        a.k_store, a.v_store = self._store_ptrs if self._k_store is not None else (0, 0)
        a.k_chan_scale = _ptr(self.k_scale)
        a.v_block_scale = _ptr(self.v_scale_cpu) if self.store_kind == _lib.STORE_INT8_REF else 0
        a.k_tok_scale, a.v_tok_scale = _ptr(self._k_tok_scale), _ptr(self._v_tok_scale)
        if allowed is not None:
            allowed = allowed.to(torch.uint8).contiguous()
            a.allowed, a.allowed_stride = allowed.data_ptr(), allowed.stride(0)
        a.sink_k, a.sink_v = self._sink_k.data_ptr(), self._sink_v.data_ptr()
        a.sink_cap, a.sink_len = cfg.sink_tokens, sink_len
        a.ring_k, a.ring_v = self._ring_k.data_ptr(), self._ring_v.data_ptr()
        a.ring_cap, a.ring_start, a.ring_len = cfg.recent_tokens, ring_start, ring_len
        if cur_k is not None:
            a.cur_k, a.cur_v = cur_k.data_ptr(), cur_v.data_ptr()
            a.cur_row_stride, a.cur_head_stride = cur_k.stride(0), cur_k.stride(1)
        a.n_cur, a.ring_write_pos = n_cur, ring_write_pos
        a.out, a.out_row_stride, a.out_head_stride = out.data_ptr(), out.stride(0), out.stride(1)
        ws = self._attend_ws(nq, ntok, prefill)
        a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
        a.overlap_select = 1 if after_select else 0
        stream = _stream(self.device)
        if prefill and n_sel > 0 and allowed is None and self.prefill_gather and (
                self.store_kind != _lib.STORE_BF16 or cfg.kv_residency == "host"):
            # int8 or host-resident history: the selected blocks are copied once
            # into a device bf16 staging store (dequantised on the way) and the
            # chunk attends to that on the tensor-core kernel
            sk, sv, sids = self._prefill_staging(n_sel)
            call("nkv_prefill_gather", stream, C.byref(a), sk.data_ptr(), sv.data_ptr())
            a.k_store, a.v_store, a.store_kind = sk.data_ptr(), sv.data_ptr(), _lib.STORE_BF16
            a.block_ids, a.max_blocks = sids.data_ptr(), n_sel
            a.k_chan_scale = a.v_block_scale = a.k_tok_scale = a.v_tok_scale = 0
        call("nkv_prefill" if prefill else "nkv_attend", stream, C.byref(a))
        return out

    def _prefill_staging(self, n_sel: int):
        """Device bf16 staging store [n_sel][Hkv][B][D] for the selected blocks
        of a prefill call, and the ids 0 .. n_sel - 1 that address it."""
        cfg = self.cfg
        if self._stage is None or self._stage[0].shape[0] < n_sel:
            shape = (n_sel, cfg.num_kv_heads, cfg.block_size, cfg.head_dim)
            self._stage = (torch.empty(shape, dtype=torch.bfloat16, device=self.device),
                           torch.empty(shape, dtype=torch.bfloat16, device=self.device),
                           torch.arange(n_sel, dtype=torch.int64, device=self.device))
        return self._stage

    # ------------------------------------------------------------------
    # prefill
    # ------------------------------------------------------------------
    def first_chunk_attention(self, q, k, v):
        """Dense causal attention within the first chunk (the caller's FA2 varlen
        call in the reference, attention.py:80-85), on the prefill kernel."""
        return self._attend(q, None, 0, 0, 0, 0, k, v, prefill=True)

    def prefill_first(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> dict:
        """Store the first chunk; dense attention is done by the caller (:518-523)."""
        assert self.prefill_len == 0, "prefill_first called after history exists"
        with self._profile_range("prefill_first_store_kv"):
            self._store_kv(k, v)
        return {"nblocks": self.nblocks_filled, "valid_len": self.valid_len}

    def _history_segments(self):
        """(sink_len, ring_start, ring_len) of the sink-deduplicated recent slice."""
        cfg = self.cfg
        sink_len = min(cfg.sink_tokens, self.valid_len)
        _, off, rlen = prefill_recent_slice(self.valid_len, cfg.sink_tokens, cfg.recent_tokens)
        return sink_len, ring_slice_start(self._ring_head, off, cfg.recent_tokens), rlen

    def prefill_chunk(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                      device: torch.device) -> torch.Tensor:
        """One later chunk: one softmax over [selected | sink | recent | chunk
        (causal)], then the chunk is stored (reference :528-651)."""
        cfg = self.cfg
        assert self.prefill_len > 0, "prefill_chunk requires prior history"
        assert not (self.quant_history and cfg.prefill_adapter is not None), \
            "quant_history is incompatible with the segmented prefill adapter"
        with self._profile_range("prefill_selector"):
            q_summary = prefill_query_summaries(q, cfg.prefill_query_segments)
            self.last_prefill_query_summaries = q_summary.shape[0]
            requested = cfg.top_k_blocks if cfg.prefill_top_k_blocks is None else cfg.prefill_top_k_blocks
            kk = self._budget(requested)
            ids = self._select_dev(q_summary, kk)
        sink_len, ring_start, ring_len = self._history_segments()
        with self._profile_range("prefill_attention"):
            if cfg.prefill_adapter is not None:
                o = cfg.prefill_adapter.attend_runtime(self, q, ids, k, v)
            else:
                o = self._attend(q, ids, kk, sink_len, ring_start, ring_len, k, v,
                                 prefill=q.shape[0] > 8)
        with self._profile_range("prefill_store_kv"):
            self._store_kv(k, v)
        self._set_last_ids(ids)
        self.last_prefill_block_ids = ids.clone()
        return o

    # ------------------------------------------------------------------
    # speculative verification (reference :656-807)
    # ------------------------------------------------------------------
    def verify_tokens(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                      device: torch.device) -> torch.Tensor:
        cfg = self.cfg
        Tq = k.shape[0]
        assert Tq >= 1, "verify needs at least one token"
        assert self.prefill_len > 0, "verify requires a complete prefill"
        assert not (self.quant_history and cfg.prefill_adapter is not None), \
            "quant_history is incompatible with the segmented prefill adapter"
        t0 = perf_counter()
        allowed = None
        count = None
        if self.verify_lossless:
            ids, allowed, count = self._select_per_query_padded(q, cfg.top_k_blocks)
            n_sel = ids.numel()
        else:
            n_sel = self._budget(cfg.top_k_blocks)
            ids = self._select_dev(q, n_sel)
        t1 = perf_counter()
        sink_len, ring_start, ring_len = self._history_segments()
        o = self._attend(q, ids, n_sel, sink_len, ring_start, ring_len, k, v, allowed=allowed,
                         prefill=Tq > 8)
        t2 = perf_counter()
        self.last_verify_timings = {"selector_ms": (t1 - t0) * 1000.0, "gather_ms": 0.0,
                                    "pack_ms": 0.0, "attention_ms": (t2 - t1) * 1000.0,
                                    "tokens": int(Tq), "blocks": int(n_sel)}
        self._pending_k = k
        self._pending_v = v
        count = None if count is None else count.clone()  # the union count of this call
        self._set_last_ids(ids, count)
        self._last_verify_dev, self._last_verify_host = ids.clone(), None
        self._last_verify_count = count
        return o

    def commit_verified(self, n: int) -> None:
        """Append the first n pending tokens to the recent window (:777-803)."""
        if n <= 0:
            self._pending_k = self._pending_v = None
            return
        cfg = self.cfg
        R = cfg.recent_tokens
        k = _aligned(self._pending_k[:n])
        v = _aligned(self._pending_v[:n])
        T = int(n)
        pos0, _, new_head = ring_append_plan(self._ring_head, self.valid_len, T, R)
        call("nkv_ring_append", _stream(self.device), k.data_ptr(), v.data_ptr(), T, k.stride(0),
             k.stride(1), v.stride(0), v.stride(1), cfg.num_kv_heads, cfg.head_dim,
             self._ring_k.data_ptr(), self._ring_v.data_ptr(), R, pos0)
        self._ring_head = new_head
        self.valid_len += T
        self._pending_k = self._pending_v = None

    def rollback_verified(self) -> None:
        self._pending_k = self._pending_v = None

    # ------------------------------------------------------------------
    # packed attention (introspection twin of the reference's _fused_attention)
    # ------------------------------------------------------------------
    def _fused_attention(self, q, k, v, hist_len, sink_len, causal_from, attn_mask=None):
        """Attention of q over packed keys [S, Hkv, D]: keys before causal_from are
        visible to every query, chunk keys causally (reference :845-896).

        The packed prefix is passed to the kernel as a head-major window; a
        non-None ``attn_mask`` is not supported here (verify_tokens builds its
        mask on the device)."""
        if attn_mask is not None:
            raise NotImplementedError("attn_mask is applied inside verify_tokens")
        cfg = self.cfg
        S = k.shape[0]
        prefix = min(causal_from, S)
        hk = k[:prefix].permute(1, 0, 2).contiguous()
        hv = v[:prefix].permute(1, 0, 2).contiguous()
        saved = (self._sink_k, self._sink_v, cfg.sink_tokens)
        try:
            self._sink_k, self._sink_v = hk, hv
            cfg.sink_tokens = prefix
            cur_k = k[prefix:] if prefix < S else None
            cur_v = v[prefix:] if prefix < S else None
            if cur_k is not None and cur_k.shape[0] != q.shape[0]:
                raise NotImplementedError("chunk length must equal the number of queries")
            return self._attend(q, None, 0, prefix, 0, 0, cur_k, cur_v,
                                prefill=q.shape[0] > 8)
        finally:
            self._sink_k, self._sink_v, cfg.sink_tokens = saved

    # ------------------------------------------------------------------
    # decode (reference :1141-1346)
    # ------------------------------------------------------------------
    def _routing_query(self, q):
        W = self.cfg.decode_query_window
        if W <= 1:
            return q[0]
        if self._qwin is None:
            self._qwin = torch.zeros(W, *q.shape[1:], dtype=q.dtype, device=q.device)
        # keep the window in time order (oldest first) like the reference's list
        if self._qwin_count < W:
            self._qwin[self._qwin_count].copy_(q[0])
            self._qwin_count += 1
        else:
            self._qwin = torch.roll(self._qwin, -1, 0)
            self._qwin[W - 1].copy_(q[0])
        n = self._qwin_count
        if n == 1:
            return self._qwin[0]
        return prefill_query_summaries(self._qwin[:n], 1)[0]

    def _decode_args(self, kk: int):
        """Persistent nkv_decode_step arguments; the buffer-dependent part is
        rebuilt only when the store, the history length, the budget or a
        workspace changed since the previous step."""
        cfg = self.cfg
        key = (self.nblocks_filled, self.cpu_blocks_cap, self._store_ptrs, kk, id(self._ids),
               id(self.k_scale), id(self.v_scale_cpu), id(self._k_tok_scale), id(self._sel_ws),
               id(self._att_ws))
        if key == self._dkey:
            return self._dargs
        d = _lib.DecodeArgs()
        a = d.attend
        a.nq, a.hq, a.hkv, a.head_dim, a.block_size = 1, cfg.num_heads, cfg.num_kv_heads, cfg.head_dim, cfg.block_size
        a.scale = cfg.scale
        a.max_blocks = self.cpu_blocks_cap
        a.store_kind = self.store_kind
        a.k_store, a.v_store = self._store_ptrs
        a.k_chan_scale = _ptr(self.k_scale)
        a.v_block_scale = _ptr(self.v_scale_cpu) if self.store_kind == _lib.STORE_INT8_REF else 0
        a.k_tok_scale, a.v_tok_scale = _ptr(self._k_tok_scale), _ptr(self._v_tok_scale)
        a.sink_k, a.sink_v, a.sink_cap = self._sink_k.data_ptr(), self._sink_v.data_ptr(), cfg.sink_tokens
        a.ring_k, a.ring_v, a.ring_cap = self._ring_k.data_ptr(), self._ring_v.data_ptr(), cfg.recent_tokens
        a.n_cur = 1
        ws = self._attend_ws(1, kk * cfg.block_size + cfg.sink_tokens + cfg.recent_tokens + 1)
        a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
        prot, nprot = self._protected_dev(self.nblocks_filled)
        d.reps, d.r, d.reps_blocks, d.nblocks = self.reps_gpu.data_ptr(), cfg.r, self.max_blocks, self.nblocks_filled
        d.protected_ids, d.n_protected, d.k = prot.data_ptr(), nprot, kk
        d.out_ids, d.out_topk_scores = self._ids.data_ptr(), self._topk_scores.data_ptr()
        sws = self._select_ws(1)
        d.select_workspace, d.select_workspace_bytes = sws.data_ptr(), sws.numel()
        a.out_row_stride, a.out_head_stride = cfg.num_heads * cfg.head_dim, cfg.head_dim
        self._dstrides = None  # (q strides, cur strides) last written into the args
        self._ring_ptr_in_args = 0  # ring_head last written into the args
        self._daddr = C.addressof(d)
        key = (self.nblocks_filled, self.cpu_blocks_cap, self._store_ptrs, kk, id(self._ids),
               id(self.k_scale), id(self.v_scale_cpu), id(self._k_tok_scale), id(self._sel_ws),
               id(self._att_ws))
        self._dargs, self._dkey = d, key
        self._ids_view = self._ids[:kk]
        return d

    def _decode_fill(self, q, k, v, kk):
        """Per-call fields of the persistent decode arguments; returns
        (args, output, ring head after the step)."""
        cfg = self.cfg
        d = self._decode_args(kk)
        a = d.attend
        qs = q.stride()
        qp = q.data_ptr()
        if qs[-1] != 1 or qs[1] % 8 or qp % 16:
            q = q.contiguous()
            qs, qp = q.stride(), q.data_ptr()
        ks, vs = k.stride(), v.stride()
        kp, vp = k.data_ptr(), v.data_ptr()
        if ks != vs or ks[-1] != 1 or ks[1] % 8 or kp % 16 or vp % 16:
            k, v = k.contiguous(), v.contiguous()
            ks, kp, vp = k.stride(), k.data_ptr(), v.data_ptr()
        out = self._out_override
        if out is None:
            out = torch.empty(1, cfg.num_heads, cfg.head_dim, dtype=q.dtype, device=q.device)
        a.q, a.cur_k, a.cur_v, a.out = qp, kp, vp, out.data_ptr()
        strides = (qs[0], qs[1], ks[0], ks[1])
        if strides != self._dstrides:
            a.q_row_stride, a.q_head_stride, a.cur_row_stride, a.cur_head_stride = strides
            self._dstrides = strides
        sink_len = min(cfg.sink_tokens, self.valid_len)
        if a.sink_len != sink_len:
            a.sink_len = sink_len
        w, a.ring_start, a.ring_len, head_new = ring_decode_plan(self._ring_head, self.valid_len,
                                                                 cfg.recent_tokens)
        a.ring_write_pos = w
        return d, out, head_new

    def _decode_fast(self, q, k, v, kk):
        """The plain decode step as one native call (nkv_decode_step)."""
        d, out, head_new = self._decode_fill(q, k, v, kk)
        if self._ring_ptr_in_args != self._ring_dev_ptr:
            d.ring_head = self._ring_ptr_in_args = self._ring_dev_ptr
        rc = self._step_fn(_stream_fast(self._dev_index), self._daddr)
        if rc != _lib.NKV_OK:
            call("nkv_decode_step", _stream(q.device), C.byref(d))  # raises with the message
        self._ring_head = head_new
        return out, d.attend.sink_len, d.attend.ring_len

    # ------------------------------------------------------------------
    # decode split in two halves around a cross-device score reduction
    # ------------------------------------------------------------------
    def block_scores_dev(self, q: torch.Tensor) -> torch.Tensor:
        """Protection-masked block scores of one decode query over this layer's
        heads ([nblocks] fp32 on the device): the scoring half of the selection
        (reference _gpu_select :999-1003 before its topk).  The view is reused
        by the next call."""
        cfg = self.cfg
        if q.ndim == 2:
            q = q.unsqueeze(0)
        assert q.shape[0] == 1 and tuple(q.shape[1:]) == (cfg.num_heads, cfg.head_dim)
        q = _aligned(q)
        nb = self.nblocks_filled
        prot, nprot = self._protected_dev(nb)
        if self._bscores is None:
            self._bscores = torch.empty(self.max_blocks, dtype=torch.float32, device=self.device)
        ws = self._select_ws(1)
        call("nkv_select_scores", _stream(self.device), q.data_ptr(), q.stride(0), q.stride(1), cfg.num_heads,
             cfg.num_kv_heads, cfg.head_dim, self.reps_gpu.data_ptr(), cfg.r, self.max_blocks, nb,
             prot.data_ptr(), nprot, self._bscores.data_ptr(), ws.data_ptr(), ws.numel())
        return self._bscores[:nb]

    def shard_scores(self, q: torch.Tensor, exchanges, n_ranks: int, rank: int) -> None:
        """Scoring half of a KV-head-sharded decode step with the exchange in
        the kernels: this layer's masked block scores go, tagged with the step,
        into every rank's exchange buffer (``exchanges``: the ctypes array of
        the ranks' buffers, nkv_shard_scores)."""
        cfg = self.cfg
        if q.ndim == 2:
            q = q.unsqueeze(0)
        q = _aligned(q)
        nb = self.nblocks_filled
        prot, nprot = self._protected_dev(nb)
        ws = self._select_ws(1)
        call("nkv_shard_scores", _stream(self.device), q.data_ptr(), q.stride(0), q.stride(1), cfg.num_heads,
             cfg.num_kv_heads, cfg.head_dim, self.reps_gpu.data_ptr(), cfg.r, self.max_blocks, nb,
             prot.data_ptr(), nprot, C.cast(exchanges, C.c_void_p), n_ranks, rank, ws.data_ptr(), ws.numel())

    def decode_shard(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, exchanges, n_ranks: int, rank: int,
                     out_full: torch.Tensor) -> torch.Tensor:
        """The rest of a KV-head-sharded decode step after shard_scores on
        every rank: ranks the max over ranks of the exchanged scores, attends
        this layer's heads, writes their rows of ``out_full`` [1, Hq_all, D]
        and exchanges rows with the other ranks inside the kernel
        (nkv_shard_attend); returns ``out_full``."""
        cfg = self.cfg
        assert q.shape[0] == 1 and k.shape[0] == 1
        assert out_full.is_contiguous() and out_full.shape[-2] == cfg.num_heads * n_ranks
        kk = self._budget(self._decode_requested)
        d, _, head_new = self._decode_fill(q, k, v, kk)
        a = _lib.AttendArgs.from_buffer_copy(d.attend)
        a.out = out_full.data_ptr() + rank * cfg.num_heads * cfg.head_dim * 2
        a.out_row_stride, a.out_head_stride = cfg.num_heads * n_ranks * cfg.head_dim, cfg.head_dim
        a.block_ids, a.n_sel, a.overlap_select = self._ids.data_ptr(), kk, 1
        call("nkv_shard_attend", _stream(self.device), C.byref(a), C.cast(exchanges, C.c_void_p), n_ranks, rank,
             self.max_blocks, self.nblocks_filled, self._ids.data_ptr(), self._topk_scores.data_ptr(),
             out_full.data_ptr())
        self._ring_head = head_new
        self.valid_len += 1
        self._last_ids_dev, self._last_ids_host = self._ids_view, None
        return out_full

    def decode_ranked(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                      scores: torch.Tensor) -> torch.Tensor:
        """The rest of a decode step given the block scores of every KV head
        (for example max-reduced over the devices that hold the other heads):
        the attention kernel ranks `scores` itself, attends this layer's heads
        to the top blocks, sink, recent window and the current token, and
        appends the token to the recent window."""
        cfg = self.cfg
        assert q.shape[0] == 1 and k.shape[0] == 1
        assert scores.dtype == torch.float32 and scores.numel() == self.nblocks_filled and scores.is_contiguous()
        kk = self._budget(self._decode_requested)
        d, out, head_new = self._decode_fill(q, k, v, kk)
        a = d.attend
        a.block_ids, a.n_sel, a.overlap_select = self._ids.data_ptr(), kk, 0
        call("nkv_attend_ranked", _stream(self.device), C.byref(a), scores.data_ptr(), scores.numel(),
             self._ids.data_ptr(), self._topk_scores.data_ptr())
        self._ring_head = head_new
        self.valid_len += 1
        self._last_ids_dev, self._last_ids_host = self._ids_view, None
        return out


    def decode(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
               device: torch.device) -> torch.Tensor:
        """One decode step: ring append, select, attend; no host synchronisation."""
        cfg = self.cfg
        R = cfg.recent_tokens
        assert q.shape[0] == 1 and k.shape[0] == 1
        if (self._fast_ok and not self.record_q and q.dtype == torch.bfloat16
                and self._k_store is not None):
            t0 = perf_counter()
            kk = self._budget(self._decode_requested)
            o, sink_len, ring_len = self._decode_fast(q, k, v, kk)
            t2 = perf_counter()
            if self.record_ids:
                self.ids_history.append(self._ids_view.cpu().tolist())
            self.valid_len += 1
            self._last_ids_dev, self._last_ids_host = self._ids_view, None
            tm = self._fast_timings
            tm["packed_attn_ms"] = (t2 - t0) * 1000.0
            tm["selected_tokens"] = kk * cfg.block_size
            tm["total_attend_tokens"] = kk * cfg.block_size + sink_len + ring_len + 1
            self.timings = tm
            if cfg.check_finite_outputs and not bool(torch.isfinite(o).all()):
                raise RuntimeError("M12 sparse decode output is non-finite")
            return o
        if self.record_q:
            self.q_history.append(q[0].detach().cpu().clone())
        t0 = perf_counter()
        q_route = self._routing_query(q)
        requested = cfg.top_k_blocks if cfg.decode_top_k_blocks is None else cfg.decode_top_k_blocks
        kk = self._budget(requested)
        # the attend kernel may overlap the select kernel only when nothing is
        # launched between them (no sort / dynamic budget / threshold step)
        plain = (cfg.decode_relative_a is None and not cfg.dynamic_top_k and not cfg.gather_sort
                 and q_route.data_ptr() == q.data_ptr())
        if cfg.decode_relative_a is not None:
            ids, kk = self._relative_select(q_route, kk)
        else:
            ids = self._select_dev(q_route, kk)
            if cfg.dynamic_top_k and kk == requested:
                kk = dynamic_top_k_from_scores(self._topk_scores[:kk].cpu(), requested,
                                               cfg.dynamic_top_k_mass)
                ids = ids[:kk]
        t1 = perf_counter()
        if self.record_ids:
            self.ids_history.append(ids.cpu().tolist())
        # recent window after the shift-and-append: logical slots [R - rlen, R),
        # the last of which is the current token (written by the attend kernel
        # into the physical slot that held logical slot 0)
        sink_len = min(cfg.sink_tokens, self.valid_len)
        write_pos, ring_start, ring_len, head_new = ring_decode_plan(self._ring_head, self.valid_len, R)
        o = self._attend(q, ids, kk, sink_len, ring_start, ring_len, k, v, ring_write_pos=write_pos,
                         after_select=plain)
        self._ring_head = head_new
        rlen = ring_len + 1
        t2 = perf_counter()
        self.valid_len += 1
        self._set_last_ids(ids)
        self.timings = {
            "selector_ms": (t1 - t0) * 1000.0, "selector_enqueue_ms": (t1 - t0) * 1000.0,
            "d2h_ms": 0.0, "cpu_gather_ms": 0.0, "h2d_pack_ms": 0.0,
            "h2d_event_spans_cpu_gather": False, "recent_ms": 0.0,
            "packed_attn_ms": (t2 - t1) * 1000.0,
            "selected_tokens": kk * cfg.block_size,
            "total_attend_tokens": kk * cfg.block_size + sink_len + rlen,
        }
        if cfg.check_finite_outputs and not bool(torch.isfinite(o).all()):
            raise RuntimeError("M12 sparse decode output is non-finite")
        return o
