"""KV-head sharding over 2, 4 and 8 GPUs against the oracle and against one
GPU running all heads.

Needs as many visible GPUs as ranks (skipped otherwise).  P spawned ranks each
hold Hkv/P of the KV heads; their full-width decode outputs must match the fp32
oracle within the parity tolerance, with the selected block ids equal to the
oracle's own selection modulo 1e-3 score ties, and must match the single-GPU
runtime (ids identical: each rank's block scores are the same fp32 values the
single GPU computes for those heads and the maximum over ranks is exact).
Sharded scoring with both exchange forms: NCCL collectives, and the
peer-memory exchange inside the kernels (several steps in a row, so both
parities of the exchange buffers and the step tags are exercised; no wait may
time out).  Replicated scoring (every rank scores all heads from its copy of
every head's representatives, the output all-gather the only collective):
the outputs equal the single GPU's bit for bit (the same scores, the same
kernel per head).
"""
import importlib
import os
import socket
import traceback
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from helpers import PKG_NAME, ids_match_modulo_ties, orc

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-2, 1e-2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q_out, exchange):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        _run(rank, world, q_out, exchange)
    except Exception:  # report at once instead of leaving the parent waiting
        q_out.put(("error", rank, traceback.format_exc()))
        raise
    finally:
        dist.destroy_process_group()


def _run(rank, world, q_out, exchange):
    nkv = importlib.import_module(PKG_NAME)
    dev = torch.device("cuda", rank)
    cfg = nkv.M12Config(max_model_len=16384, device=dev)
    if exchange == "replicated":
        layer = nkv.KVHeadShardedLayer(0, cfg, exchange="nccl", scoring="replicated")
    else:
        layer = nkv.KVHeadShardedLayer(0, cfg, exchange=exchange)
    single = nkv.M12LayerRuntime(0, cfg) if rank == 0 else None
    oracle = orc.OracleLayer(orc.OracleConfig()) if rank == 0 else None
    g = torch.Generator().manual_seed(3)  # host generator: every rank draws the same inputs
    for c in range(3):
        k = torch.randn(4096, 8, 128, generator=g).bfloat16()
        v = torch.randn(4096, 8, 128, generator=g).bfloat16()
        kd, vd = k.to(dev), v.to(dev)
        if c == 0:
            layer.prefill_first(None, kd, vd)
            if single:
                single.prefill_first(None, kd, vd)
        else:
            layer.store(kd, vd)
            if single:
                single._store_kv(kd, vd)
        if oracle:
            oracle.store(k, v)
            oracle.prefill_len = oracle.valid_len
    out = []
    for _ in range(5):
        q = torch.randn(1, 32, 128, generator=g).bfloat16()
        k = torch.randn(1, 8, 128, generator=g).bfloat16()
        v = torch.randn(1, 8, 128, generator=g).bfloat16()
        got = layer.decode(q.to(dev), k.to(dev), v.to(dev))
        ids = layer.last_block_ids.cpu()
        if single:
            want = single.decode(q.to(dev), k.to(dev), v.to(dev), dev)
            oracle.force_ids = ids
            o_want = oracle.decode(q, k, v)
            out.append((got.float().cpu(), want.float().cpu(), ids, single.last_block_ids.cpu(),
                        o_want, oracle.own_ids, oracle.last_scores))
    torch.cuda.synchronize()
    err = int(layer.rt._att_ws[:4].view(torch.int32).item())
    assert err == 0, f"rank {rank}: kernel error word {err}"
    assert layer.exchange == ("nccl" if exchange == "replicated" else exchange), (layer.exchange, exchange)
    layer.close()
    if rank == 0:
        q_out.put(("ok", 0, [tuple(t.numpy() for t in r) for r in out]))


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("exchange", ["nccl", "peer", "replicated"])
def test_kv_head_sharding(world, exchange):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q_out, exchange)) for r in range(world)]
    for p in procs:
        p.start()
    status, who, res = q_out.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
    assert status == "ok", f"rank {who} failed:\n{res}"
    for p in procs:
        assert p.exitcode == 0
    for got, want, ids_got, ids_want, o_want, own, scores in res:
        assert (ids_got == ids_want).all()
        ok, why = ids_match_modulo_ties(torch.from_numpy(ids_got), torch.from_numpy(own), torch.from_numpy(scores))
        assert ok, why
        torch.testing.assert_close(torch.from_numpy(got), torch.from_numpy(o_want), atol=ATOL, rtol=RTOL)
        torch.testing.assert_close(torch.from_numpy(got), torch.from_numpy(want), atol=ATOL, rtol=RTOL)
        if exchange == "replicated":
            assert (got == want).all(), "replicated scoring must reproduce the single GPU bit for bit"
