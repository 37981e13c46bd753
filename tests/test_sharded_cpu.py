"""KV-head sharding (KVHeadShardedLayer) on CPU with gloo ranks.

Each rank's per-layer runtime is replaced by the oracle restricted to its KV
heads (a test double: the product runtime is CUDA); the test checks the
sharding itself - which heads each rank owns, the MAX all-reduce of block
scores, ranking from the reduced scores and the all-gather of the outputs -
against the unsharded oracle: identical block ids and outputs within fp32
rounding, for 2 and 4 ranks.
"""
import importlib
import os
import socket
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from helpers import PKG_NAME, orc, qkv

CFG = dict(block_size=16, r=4, recent_tokens=32, sink_tokens=16, top_k_blocks=4,
           num_heads=8, num_kv_heads=4, head_dim=128)


class OracleShardRuntime:
    """Per-rank stand-in for M12LayerRuntime over the rank's heads (oracle math)."""

    def __init__(self, layer_id, cfg):
        self.layer = orc.OracleLayer(orc.OracleConfig(**{k: getattr(cfg, k) for k in CFG}))
        self.last_block_ids = None

    @property
    def valid_len(self):
        return self.layer.valid_len

    def prefill_first(self, q, k, v):
        self.layer.store(k.contiguous(), v.contiguous())
        self.layer.prefill_len = self.layer.valid_len
        return {}

    def _store_kv(self, k, v):
        self.layer.store(k.contiguous(), v.contiguous())

    def block_scores_dev(self, q):
        L = self.layer
        return orc.mask_protected(orc.block_scores(q.contiguous(), L.reps, L.nblocks), L.protected, L.nblocks)

    def decode_ranked(self, q, k, v, scores):
        L = self.layer
        kk = orc.select_k(L.nblocks, L.protected, L.cfg.top_k_blocks)
        L.force_ids = orc.rank_blocks(scores)[:kk]
        o = L.decode(q.contiguous(), k.contiguous(), v.contiguous())
        self.last_block_ids = L.last_ids
        return o


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q_out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        _run(rank, world, q_out)
    except Exception:  # report at once instead of leaving the parent waiting
        q_out.put(("error", rank, traceback.format_exc()))
        raise
    finally:
        dist.destroy_process_group()


def _run(rank, world, q_out):
    nkv = importlib.import_module(PKG_NAME)
    cfg = nkv.M12Config(device="cpu", **CFG)
    layer = nkv.KVHeadShardedLayer(0, cfg, runtime_factory=OracleShardRuntime)
    g = torch.Generator().manual_seed(11)
    full = orc.OracleLayer(orc.OracleConfig(**CFG))
    for c in range(3):
        q, k, v = qkv(g, 160)  # ragged: 10 blocks per chunk
        k, v = k[:, :4], v[:, :4]
        if c == 0:
            layer.prefill_first(None, k, v)
            full.store(k, v)
            full.prefill_len = full.valid_len
        else:
            layer.store(k, v)
            full.store(k, v)
    results = []
    for _ in range(3):
        q, k, v = qkv(g, 1)
        q, k, v = q[:, :8], k[:, :4], v[:, :4]
        got = layer.decode(q, k, v)
        want = full.decode(q, k, v)
        results.append((got.float(), want.float(), layer.last_block_ids.clone(), full.last_ids.clone()))
    if rank == 0:
        q_out.put(("ok", 0, [(a.numpy(), b.numpy(), c.numpy(), d.numpy()) for a, b, c, d in results]))


@pytest.mark.parametrize("world", [2, 4])
def test_kv_head_sharding_matches_unsharded(world):
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q_out)) for r in range(world)]
    for p in procs:
        p.start()
    status, who, res = q_out.get(timeout=240)
    for p in procs:
        p.join(timeout=60)
    assert status == "ok", f"rank {who} failed:\n{res}"
    for p in procs:
        assert p.exitcode == 0
    for got, want, ids_got, ids_want in res:
        assert (ids_got == ids_want).all()
        torch.testing.assert_close(torch.from_numpy(got), torch.from_numpy(want), atol=1e-5, rtol=1e-5)
