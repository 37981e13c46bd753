"""KV-head sharding of the sparse path over the GPUs of one node.

Each rank of a ``torch.distributed`` process group (one GPU per rank) holds
the history, representatives, sink and recent window of its share of the KV
heads (rank i owns KV heads [i*Hkv/P, (i+1)*Hkv/P) and their query heads) and
runs the per-layer kernels on them.  A decode step exchanges two things over
NVLink:

1. block selection is global in the reference: a block's score is the maximum
   over every query head (m12_runtime.py:999-1003).  Each rank scores its own
   heads; the maximum over ranks of the fp32 block scores gives every rank the
   global scores, from which its attention kernel ranks the same Top-K as a
   single GPU would;
2. the per-rank attention outputs [1, Hq/P, D] are gathered into [1, Hq, D]
   (the all-gather before o_proj).

Two forms of the scoring:

- ``scoring="sharded"`` (option B): each rank scores its own heads and the
  block scores are max-reduced over the ranks (one exchange), as above;
- ``scoring="replicated"`` (option A): every rank also keeps the
  representatives of every KV head (built from the full-width keys each rank
  receives; the store itself stays sharded) and scores all heads itself, so
  every rank computes the single-GPU scores with no exchange; the output
  gather (one NCCL all-gather) is the only collective.

Two forms of the exchange for sharded scoring:

- ``exchange="peer"`` (the default where every pair of GPUs has peer access):
  inside the kernels, through per-layer exchange buffers that every rank maps
  (CUDA IPC).  The scoring kernel writes its scores as step-tagged 8-byte words
  into every rank's buffer; the attention kernel polls them, ranks the max,
  attends, pushes its output rows to the other ranks the same way and pulls
  theirs before it ends.  No collective library call on the data path.
- ``exchange="nccl"``: a MAX all-reduce of the scores ([nblocks], 2 KB at 32K)
  and an all-gather of the outputs (NCCL), around the same two kernels.

Prefill needs no exchange for the store (each rank stores its heads' K/V);
the segmented prefill attention of a later chunk selects with query segment
means whose scores reduce the same way.
"""
from __future__ import annotations

import ctypes as C
import dataclasses

import torch
import torch.distributed as dist

from . import _lib
from .m12_runtime import M12Config, M12LayerRuntime


class KVHeadShardedLayer:
    """One layer's sparse runtime with its KV heads split over a process group.

    ``runtime_factory(layer_id, local_cfg)`` builds the per-rank runtime (the
    CUDA ``M12LayerRuntime`` by default); it must provide ``prefill_first``,
    ``_store_kv``, ``block_scores_dev`` and ``decode_ranked``.
    """

    def __init__(self, layer_id: int, cfg: M12Config, group=None, runtime_factory=None, exchange: str = "auto",
                 scoring: str = "sharded"):
        if exchange not in ("auto", "peer", "nccl"):
            raise ValueError(f"exchange must be 'auto', 'peer' or 'nccl', not {exchange!r}")
        if scoring not in ("sharded", "replicated"):
            raise ValueError(f"scoring must be 'sharded' or 'replicated', not {scoring!r}")
        if scoring == "replicated" and runtime_factory is not None:
            raise ValueError("replicated scoring needs the CUDA runtime (its representatives store)")
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if cfg.num_kv_heads % self.world:
            raise ValueError(f"{cfg.num_kv_heads} KV heads do not split over {self.world} ranks")
        self.hkv = cfg.num_kv_heads // self.world
        self.hq = cfg.num_heads // self.world
        self.kv0 = self.rank * self.hkv
        self.q0 = self.rank * self.hq
        self.cfg = cfg
        self.local_cfg = dataclasses.replace(cfg, num_heads=self.hq, num_kv_heads=self.hkv)
        self.rt = (runtime_factory or M12LayerRuntime)(layer_id, self.local_cfg)
        self.scoring = scoring
        self.exchange = "nccl" if (self.world == 1 or exchange == "nccl" or runtime_factory is not None
                                   or scoring == "replicated") else exchange
        # replicated scoring: every KV head's representatives [Hkv][max_blocks][r][D]
        self.reps_all = self._rep_index_all = self._scores = None
        if scoring == "replicated":
            dev = self.rt.device
            self.reps_all = torch.zeros(cfg.num_kv_heads, self.rt.max_blocks, cfg.r, cfg.head_dim,
                                        dtype=torch.bfloat16, device=dev)
            self._rep_index_all = torch.zeros(cfg.num_kv_heads, self.rt.max_blocks, cfg.r, dtype=torch.int16,
                                              device=dev)
            self._scores = torch.empty(self.rt.max_blocks, dtype=torch.float32, device=dev)
        self._exch = None      # ctypes array of the ranks' exchange buffers (peer form)
        self._exch_cap = 0     # block capacity they were made for
        self._own = None       # this rank's buffer
        self._opened = []      # the peers' buffers opened here

    # this rank's heads of full-width tensors [T, heads, D]
    def _kv(self, x: torch.Tensor) -> torch.Tensor:
        return x[:, self.kv0:self.kv0 + self.hkv]

    def _q(self, x: torch.Tensor) -> torch.Tensor:
        return x[:, self.q0:self.q0 + self.hq]

    @property
    def valid_len(self) -> int:
        return self.rt.valid_len

    @property
    def last_block_ids(self):
        return self.rt.last_block_ids

    def prefill_first(self, q, k, v) -> dict:
        start = self.rt.nblocks_filled if self.reps_all is not None else 0
        out = self.rt.prefill_first(None if q is None else self._q(q), self._kv(k), self._kv(v))
        self._store_reps_all(k, start)
        return out

    def store(self, k: torch.Tensor, v: torch.Tensor) -> None:
        """Append a chunk of history (the store half of prefill)."""
        start = self.rt.nblocks_filled if self.reps_all is not None else 0
        self.rt._store_kv(self._kv(k), self._kv(v))
        self._store_reps_all(k, start)

    def _store_reps_all(self, k: torch.Tensor, start_block: int) -> None:
        """Replicated scoring: the representatives of every KV head for the
        chunk's blocks (the store kernel's representatives-only form)."""
        if self.reps_all is None:
            return
        cfg = self.cfg
        k = k if (k.stride(-1) == 1 and k.data_ptr() % 16 == 0) else k.contiguous()
        a = _lib.StoreArgs()
        a.k = a.v = k.data_ptr()
        a.k_row_stride, a.k_head_stride = k.stride(0), k.stride(1)
        a.v_row_stride, a.v_head_stride = k.stride(0), k.stride(1)
        a.T, a.hkv, a.head_dim, a.block_size, a.r = k.shape[0], cfg.num_kv_heads, cfg.head_dim, cfg.block_size, cfg.r
        a.start_block, a.max_blocks = start_block, self.rt.max_blocks
        a.store_kind = _lib.STORE_BF16
        a.k_store = a.v_store = 0
        a.reps, a.rep_index = self.reps_all.data_ptr(), self._rep_index_all.data_ptr()
        a.sink_cap = a.sink_write = a.ring_cap = 0
        _lib.call("nkv_store_chunk", torch.cuda.current_stream(self.rt.device).cuda_stream, C.byref(a))

    def scores_all(self, q: torch.Tensor) -> torch.Tensor:
        """Replicated scoring: the single-GPU block scores from every query head
        and every KV head's representatives ([nblocks] fp32)."""
        cfg, rt = self.cfg, self.rt
        q = q if q.ndim == 3 else q.unsqueeze(0)
        if q.stride(-1) != 1 or q.stride(1) % 8 or q.data_ptr() % 16:
            q = q.contiguous()
        nb = rt.nblocks_filled
        prot, nprot = rt._protected_dev(nb)
        ws = rt._select_ws(1)
        _lib.call("nkv_select_scores", torch.cuda.current_stream(rt.device).cuda_stream, q.data_ptr(), q.stride(0),
                  q.stride(1), cfg.num_heads, cfg.num_kv_heads, cfg.head_dim, self.reps_all.data_ptr(), cfg.r,
                  rt.max_blocks, nb, prot.data_ptr(), nprot, self._scores.data_ptr(), ws.data_ptr(), ws.numel())
        return self._scores[:nb]

    # ---- peer exchange buffers (collective: every rank calls at the same point) ----
    def _peer_ok(self) -> bool:
        """Whether every rank's GPU can access every other's memory."""
        dev = torch.cuda.current_device() if self.rt.device.index is None else self.rt.device.index
        devs = [None] * self.world
        dist.all_gather_object(devs, dev, group=self.group)
        ok = all(a == b or torch.cuda.can_device_access_peer(dev, b) for a in [dev] for b in devs)
        oks = [None] * self.world
        dist.all_gather_object(oks, bool(ok), group=self.group)
        return all(oks)

    def _ensure_exchange(self) -> None:
        cap = self.rt.max_blocks
        if self._exch is not None and cap <= self._exch_cap:
            return
        if self.exchange == "auto":
            self.exchange = "peer" if self._peer_ok() else "nccl"
            if self.exchange == "nccl":
                return
        self.close()
        lib = _lib.load()
        nbytes = lib.nkv_shard_exchange_bytes(self.world, cap, self.cfg.num_heads)
        own = C.c_void_p()
        handle = C.create_string_buffer(_lib.IPC_HANDLE_BYTES)
        _lib.call("nkv_peer_alloc", nbytes, C.byref(own), handle)
        handles = [None] * self.world
        dist.all_gather_object(handles, handle.raw, group=self.group)
        ptrs = (C.c_void_p * self.world)()
        for r, hb in enumerate(handles):
            if r == self.rank:
                ptrs[r] = own.value
                continue
            p = C.c_void_p()
            _lib.call("nkv_peer_open", C.create_string_buffer(hb, _lib.IPC_HANDLE_BYTES), C.byref(p))
            ptrs[r] = p.value
            self._opened.append(p.value)
        self._own, self._exch, self._exch_cap = own.value, ptrs, cap
        # no rank writes into a peer's buffer before every rank has opened it
        dist.barrier(group=self.group)

    def close(self) -> None:
        """Release the peer exchange buffers (collective where they exist)."""
        if self._exch is None:
            return
        torch.cuda.synchronize()
        dist.barrier(group=self.group)  # no peer still writes into them
        lib = _lib.load()
        for p in self._opened:
            lib.nkv_peer_close(C.c_void_p(p))
        if self._own:
            lib.nkv_peer_free(C.c_void_p(self._own))
        self._exch, self._own, self._opened, self._exch_cap = None, None, [], 0

    def decode(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, device=None) -> torch.Tensor:
        """One decode step for full-width q [1, Hq, D], k/v [1, Hkv, D] (every
        rank gets the same inputs, as with a replicated model); returns the
        full-width output [1, Hq, D] on every rank."""
        if self.world > 1 and self.exchange != "nccl":
            self._ensure_exchange()
        if self.world > 1 and self.exchange == "peer":
            out = torch.empty(1, self.cfg.num_heads, self.cfg.head_dim, dtype=q.dtype, device=q.device)
            self.rt.shard_scores(self._q(q), self._exch, self.world, self.rank)
            return self.rt.decode_shard(self._q(q), self._kv(k), self._kv(v), self._exch, self.world, self.rank,
                                        out)
        if self.scoring == "replicated":
            scores = self.scores_all(q)
        else:
            scores = self.rt.block_scores_dev(self._q(q))
            if self.world > 1:
                dist.all_reduce(scores, op=dist.ReduceOp.MAX, group=self.group)
        o = self.rt.decode_ranked(self._q(q), self._kv(k), self._kv(v), scores)
        if self.world == 1:
            return o
        # rank-major rows = head-major rows: rank i holds query heads [i hq, (i + 1) hq)
        out = torch.empty(self.world * o.numel(), dtype=o.dtype, device=o.device)
        dist.all_gather_into_tensor(out, o.contiguous().view(-1), group=self.group)
        return out.view(1, self.cfg.num_heads, self.cfg.head_dim)
