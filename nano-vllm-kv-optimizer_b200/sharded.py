"""KV-head sharding of the sparse path over the GPUs of one node.

Each rank of a ``torch.distributed`` process group (one GPU per rank, NCCL)
holds the history, representatives, sink and recent window of its share of
the KV heads (rank i owns KV heads [i*Hkv/P, (i+1)*Hkv/P) and their query
heads) and runs the per-layer kernels on them.  A decode step exchanges two
things over NVLink:

1. block selection is global in the reference: a block's score is the maximum
   over every query head (m12_runtime.py:999-1003).  Each rank scores its own
   heads; one MAX all-reduce of the fp32 block scores ([nblocks], 2 KB at 32K)
   gives every rank the global scores, from which its attention kernel ranks
   the same Top-K as a single GPU would;
2. the per-rank attention outputs [1, Hq/P, D] are all-gathered into
   [1, Hq, D] (the all-gather before o_proj).

Prefill needs no exchange for the store (each rank stores its heads' K/V);
the segmented prefill attention of a later chunk selects with query segment
means whose scores reduce the same way.
"""
from __future__ import annotations

import dataclasses

import torch
import torch.distributed as dist

from .m12_runtime import M12Config, M12LayerRuntime


class KVHeadShardedLayer:
    """One layer's sparse runtime with its KV heads split over a process group.

    ``runtime_factory(layer_id, local_cfg)`` builds the per-rank runtime (the
    CUDA ``M12LayerRuntime`` by default); it must provide ``prefill_first``,
    ``_store_kv``, ``block_scores_dev`` and ``decode_ranked``.
    """

    def __init__(self, layer_id: int, cfg: M12Config, group=None, runtime_factory=None):
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
        return self.rt.prefill_first(None if q is None else self._q(q), self._kv(k), self._kv(v))

    def store(self, k: torch.Tensor, v: torch.Tensor) -> None:
        """Append a chunk of history (the store half of prefill)."""
        self.rt._store_kv(self._kv(k), self._kv(v))

    def decode(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, device=None) -> torch.Tensor:
        """One decode step for full-width q [1, Hq, D], k/v [1, Hkv, D] (every
        rank gets the same inputs, as with a replicated model); returns the
        full-width output [1, Hq, D] on every rank."""
        scores = self.rt.block_scores_dev(self._q(q))
        if self.world > 1:
            dist.all_reduce(scores, op=dist.ReduceOp.MAX, group=self.group)
        o = self.rt.decode_ranked(self._q(q), self._kv(k), self._kv(v), scores)
        if self.world == 1:
            return o
        parts = [torch.empty_like(o) for _ in range(self.world)]
        dist.all_gather(parts, o.contiguous(), group=self.group)
        return torch.cat(parts, dim=1)
