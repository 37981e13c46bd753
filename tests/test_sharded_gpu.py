"""KV-head sharding over 2 GPUs against one GPU running all heads.

Needs two visible GPUs (skipped otherwise).  Two spawned ranks each hold half
of the KV heads; their full-width decode outputs must match the single-GPU
runtime's within the parity tolerance, and the selected block ids must be
identical (each rank's block scores are the same fp32 values the single GPU
computes for those heads; the maximum over ranks is exact).  Both exchange
forms: NCCL collectives, and the peer-memory exchange inside the kernels
(several steps in a row, so both parities of the exchange buffers and the
step tags are exercised; no wait may time out).
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

from helpers import PKG_NAME

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
    layer = nkv.KVHeadShardedLayer(0, cfg, exchange=exchange)
    single = nkv.M12LayerRuntime(0, cfg) if rank == 0 else None
    g = torch.Generator(device=dev).manual_seed(3)
    for c in range(3):
        k = torch.randn(4096, 8, 128, generator=g, device=dev).bfloat16()
        v = torch.randn(4096, 8, 128, generator=g, device=dev).bfloat16()
        if c == 0:
            layer.prefill_first(None, k, v)
            if single:
                single.prefill_first(None, k, v)
        else:
            layer.store(k, v)
            if single:
                single._store_kv(k, v)
    out = []
    for _ in range(5):
        q = torch.randn(1, 32, 128, generator=g, device=dev).bfloat16()
        k = torch.randn(1, 8, 128, generator=g, device=dev).bfloat16()
        v = torch.randn(1, 8, 128, generator=g, device=dev).bfloat16()
        got = layer.decode(q, k, v)
        ids = layer.last_block_ids.cpu()
        if single:
            want = single.decode(q, k, v, dev)
            out.append((got.float().cpu(), want.float().cpu(), ids, single.last_block_ids.cpu()))
    torch.cuda.synchronize()
    err = int(layer.rt._att_ws[:4].view(torch.int32).item())
    assert err == 0, f"rank {rank}: kernel error word {err}"
    assert layer.exchange == exchange, (layer.exchange, exchange)
    layer.close()
    if rank == 0:
        q_out.put(("ok", 0, [tuple(t.numpy() for t in r) for r in out]))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("exchange", ["nccl", "peer"])
def test_kv_head_sharding_two_gpus(exchange):
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q_out, exchange)) for r in range(2)]
    for p in procs:
        p.start()
    status, who, res = q_out.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
    assert status == "ok", f"rank {who} failed:\n{res}"
    for p in procs:
        assert p.exitcode == 0
    for got, want, ids_got, ids_want in res:
        assert (ids_got == ids_want).all()
        torch.testing.assert_close(torch.from_numpy(got), torch.from_numpy(want), atol=ATOL, rtol=RTOL)
