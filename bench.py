"""Benchmark of the sparse decode hot path (select + attend per layer) at 32K.

Contract: ``python bench.py --gpus N --steps K --warmup W`` prints ONE JSON line
on rank 0.  A step is one decode token through L=36 independent layer states
(Qwen3-4B attention geometry: 32 query / 8 KV heads, head_dim 128, bf16), each
holding a 32768-token history (64-token blocks, r=4 reps, Top-32, sink 64,
recent 512) resident in HBM.  Per layer the step runs kernel (1) (score +
Top-K) and kernel (2) (fused gather-attend).  The 36 layer states together
hold ~2.7 GB and a step touches ~540 MB, more than L2 (126 MB), so no L2 flush
is needed between steps.  Inputs are synthetic (seeded N(0,1)).

Metric: device time per layer decode, whole job: step_time / (L * n_gpus) in
microseconds (lower is better); the step is replayed through DecodeGraph (the
36 layers' decode recorded once, the recent windows advancing on the device
with every replay, as in a decode loop).  With N GPUs each rank decodes its own
independent sequence (replicas; weak scaling, no collective on the data path).

``--impl reference`` times the reference's own CPU implementation on the host
cores instead: its ``M12LayerRuntime.decode`` (torch, from the reference package
installed under ``baseline/_ref``, run through the CPU device shim in
``oracle/ref_shim.py``), with the oracle port's time beside it (the port is the
reference arm when the package is absent).
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
PKG = "nano-vllm-kv-optimizer_b200"

HQ, HKV, D, B, R_REPS = 32, 8, 128, 64, 4
TOPK, SINK, RECENT = 32, 64, 512
CTX = 32768
LAYERS = 36
NSETS = 8  # distinct decode inputs in rotation (the selection changes every step)
METRIC = "sparse decode attn us/layer @32K ctx"
UNIT = "us/layer"

# algorithmic bytes per layer decode (unit of the roofline)
ATTEND_TOKENS = TOPK * B + SINK + RECENT                 # 2624 keys per kv head
ATTEND_BYTES = ATTEND_TOKENS * HKV * D * 2 * 2 + (HQ * D * 2) * 2 + HKV * D * 2 * 2
SELECT_BYTES = (CTX // B) * HKV * R_REPS * D * 2 + HQ * D * 2
STEP_BYTES = ATTEND_BYTES + SELECT_BYTES
# DRAM bytes of one launch of the step's attention kernel (decode_split_kernel),
# recorded from a separate ncu capture of this kernel
ATTEND_TRAFFIC = 10816000
# segmented prefill operator: a 4096-token chunk after a
# 28672-token history; visible (query, key) pairs per head x 32 heads x 4 D
PF_CHUNK, PF_HIST = 4096, 28672
PF_PAIRS = PF_CHUNK * (TOPK * B + SINK + RECENT) + PF_CHUNK * (PF_CHUNK + 1) // 2
PF_FLOP = PF_PAIRS * HQ * 4 * D


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def tensor_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        return float(json.load(open(p))["bf16_tflops"]), "measured (burst)"
    return 1590.0, "fallback"


# int8 history (per-token per-KV-head bf16 scale) in pinned
# host memory; per layer-token the selected blocks cross the host link
OFF_LAYERS = 8
OFF_BYTES = TOPK * B * HKV * D * 2 + TOPK * B * HKV * 2 * 2  # int8 K+V + bf16 K,V scales


def host_link_gbs(dev, mib=256):
    """Pinned host -> device copy bandwidth of this box (the offload roofline)."""
    h = torch.empty(mib << 20, dtype=torch.uint8).pin_memory()
    d = torch.empty(mib << 20, dtype=torch.uint8, device=dev)
    for _ in range(2):
        d.copy_(h, non_blocking=True)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(5):
        d.copy_(h, non_blocking=True)
    e1.record()
    e1.synchronize()
    gbs = 5 * (mib << 20) / (e0.elapsed_time(e1) * 1e-3) / 1e9
    del h, d
    return gbs


def offload_measure(nkv, dev, steps=20):
    """Decode step (select + attend) with the history int8 in mapped pinned host
    memory; the attention kernel reads the selected blocks over the host link
    and dequantises them in registers."""
    g = torch.Generator(device=dev).manual_seed(77)
    layers = []
    for li in range(OFF_LAYERS):
        rt = nkv.M12LayerRuntime(li, nkv.M12Config(max_model_len=CTX + 4096, device=dev, quant_history=True,
                                                   quant_scheme="token", kv_residency="host"))
        rt.reserve_blocks(CTX // B)
        for c in range(CTX // 4096):
            k = torch.randn(4096, HKV, D, generator=g, device=dev).bfloat16()
            v = torch.randn(4096, HKV, D, generator=g, device=dev).bfloat16()
            if c == 0:
                rt.prefill_first(None, k, v)
            else:
                rt._store_kv(k, v)
        layers.append(rt)
    torch.cuda.synchronize()
    qs = torch.randn(OFF_LAYERS, 1, HQ, D, generator=g, device=dev).bfloat16()
    ks = torch.randn(OFF_LAYERS, 1, HKV, D, generator=g, device=dev).bfloat16()
    vs = torch.randn(OFF_LAYERS, 1, HKV, D, generator=g, device=dev).bfloat16()
    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        for li, rt in enumerate(layers):
            rt.decode(qs[li], ks[li], vs[li], dev)
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for li, rt in enumerate(layers):
            rt.decode(qs[li], ks[li], vs[li], dev)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(steps):
            graph.replay()
        e1.record(stream)
    e1.synchronize()
    us = e0.elapsed_time(e1) * 1000.0 / (steps * OFF_LAYERS)
    link = host_link_gbs(dev)
    achieved = OFF_BYTES / (us * 1e-6) / 1e9
    del graph, layers
    return {"workload": "decode step @32K, int8 history (per-token bf16 scales) in pinned host memory, "
                        "8 layer states, Top-32 selected blocks read over the host link",
            "us_per_layer": round(us, 2), "host_bytes_per_layer": OFF_BYTES,
            "roofline": {"bound": "host link", "achieved": round(achieved, 1), "peak": round(link, 1),
                         "unit": "GB/s", "frac": round(achieved / link, 4),
                         "peak_kind": "measured pinned H2D copy (256 MiB) on this box"}}


# BASELINE config 5 (operator part): KV heads sharded over the N ranks, 128K
# history; 8 layer states (27.5 MB of representatives and selected KV per
# layer: 220 MB per step, above the 126 MB L2), inputs rotating over NSETS sets
SH_CTX, SH_LAYERS = 131072, 8


def _sharded_build(nkv, dev, make):
    """SH_LAYERS layers of 128K history (the same seeded K/V on every rank)."""
    g = torch.Generator(device=dev).manual_seed(5150)
    layers = []
    for li in range(SH_LAYERS):
        lay = make(li)
        rt = getattr(lay, "rt", lay)
        rt.reserve_blocks(SH_CTX // B)
        for c in range(SH_CTX // 4096):
            k = torch.randn(4096, HKV, D, generator=g, device=dev).bfloat16()
            v = torch.randn(4096, HKV, D, generator=g, device=dev).bfloat16()
            if c == 0:
                lay.prefill_first(None, k, v)
            elif lay is rt:
                rt._store_kv(k, v)
            else:
                lay.store(k, v)
        layers.append(lay)
    return layers


def _sharded_inputs(dev):
    """NSETS input sets of every layer's q/k/v and the staging buffer the step reads."""
    QKV = (HQ + 2 * HKV) * D
    xs = torch.randn(NSETS, SH_LAYERS, QKV, generator=torch.Generator(device=dev).manual_seed(77),
                     device=dev).bfloat16()
    x = xs[0].clone()
    views = [(x[li, :HQ * D].view(1, HQ, D), x[li, HQ * D:(HQ + HKV) * D].view(1, HKV, D),
              x[li, (HQ + HKV) * D:].view(1, HKV, D)) for li in range(SH_LAYERS)]
    return xs, x, views


def _graph_time(fn, xs, x, stream, steps, collective):
    """us per layer of fn() replayed from a CUDA graph (eager when every rank
    cannot capture), the staging buffer refilled from the next input set
    before each replay; max over ranks when collective."""
    import torch.distributed as dist
    with torch.cuda.stream(stream):
        for i in range(3):
            x.copy_(xs[i % NSETS])
            fn()
    torch.cuda.synchronize()
    graph, mode = None, "eager"
    try:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            fn()
        mode = "cuda graph"
    except Exception:  # noqa: BLE001 - measured eagerly instead
        graph = None
        torch.cuda.synchronize()
    if collective:
        ok = torch.tensor([0 if graph is None else 1], device=x.device)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        if int(ok.item()) == 0:
            graph, mode = None, "eager"
        dist.barrier()
    run = graph.replay if graph is not None else fn
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        for i in range(3):
            x.copy_(xs[i % NSETS])
            run()
        e0.record(stream)
        for i in range(steps):
            x.copy_(xs[i % NSETS])
            run()
        e1.record(stream)
    e1.synchronize()
    us = e0.elapsed_time(e1) * 1000.0 / (steps * SH_LAYERS)
    if collective:
        t = torch.tensor([us], device=x.device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        us = float(t.item())
    del graph
    torch.cuda.synchronize()
    return us, mode


def sharded_measure(nkv, dev, world, steps=20):
    """Decode step with the KV heads split over the ranks (KVHeadShardedLayer)
    at 128K, per layer, three forms: sharded scoring with the exchange inside
    the kernels ("peer") or as NCCL collectives ("nccl": MAX all-reduce of the
    scores, all-gather of the outputs), and replicated scoring ("replicated":
    every rank scores all heads, the output all-gather is the only collective).
    Each is replayed from a CUDA graph with the inputs changing every step
    (device time between events, max over ranks); the input copies (the same
    in every form) are inside the timed region.  For the NCCL forms the step
    is also timed cut after the scoring (with its exchange) and after the
    attention, which gives the marginal cost of each phase.  Rank 0 also times
    the same layers unsharded on its GPU."""
    import torch.distributed as dist
    res = {"workload": f"decode step @128K (Top-32 of 2048 blocks), KV heads sharded {world} ways, "
                       f"{SH_LAYERS} layer states, inputs rotating over {NSETS} sets",
           "kv_heads_per_gpu": HKV // world}
    stream = torch.cuda.Stream(dev)
    for name, exchange, scoring in (("peer", "peer", "sharded"), ("nccl", "nccl", "sharded"),
                                    ("replicated", "nccl", "replicated")):
        cfg = nkv.M12Config(max_model_len=SH_CTX + 4096, device=dev)
        layers = _sharded_build(nkv, dev, lambda li: nkv.KVHeadShardedLayer(li, cfg, exchange=exchange,
                                                                             scoring=scoring))
        xs, x, views = _sharded_inputs(dev)

        def step():
            for lay, (q, k, v) in zip(layers, views):
                lay.decode(q, k, v)
        us, mode = _graph_time(step, xs, x, stream, steps, True)
        entry = {"us_per_layer": round(us, 2), "mode": mode, "exchange": layers[0].exchange,
                 "scoring": scoring}
        if exchange == "nccl":
            def scores_only():
                for lay, (q, k, v) in zip(layers, views):
                    if scoring == "replicated":
                        lay.scores_all(q)
                    else:
                        sc = lay.rt.block_scores_dev(lay._q(q))
                        dist.all_reduce(sc, op=dist.ReduceOp.MAX, group=lay.group)

            def no_gather():
                for lay, (q, k, v) in zip(layers, views):
                    if scoring == "replicated":
                        sc = lay.scores_all(q)
                    else:
                        sc = lay.rt.block_scores_dev(lay._q(q))
                        dist.all_reduce(sc, op=dist.ReduceOp.MAX, group=lay.group)
                    lay.rt.decode_ranked(lay._q(q), lay._kv(k), lay._kv(v), sc)
            t_sc, _ = _graph_time(scores_only, xs, x, stream, steps, True)
            t_at, _ = _graph_time(no_gather, xs, x, stream, steps, True)
            entry["marginal_us_per_layer"] = {
                "scoring" + ("" if scoring == "replicated" else " + MAX all-reduce"): round(t_sc, 2),
                "attention": round(t_at - t_sc, 2), "output all-gather": round(us - t_at, 2)}
        errs = sum(int(lay.rt._att_ws[:4].view(torch.int32).item()) != 0 for lay in layers)
        t = torch.tensor([float(errs)], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        entry["kernel_errors"] = int(t.item())
        for lay in layers:
            lay.close()
        res[name] = entry
        del layers, xs, x, views
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
    if dist.get_rank() == 0:
        # the same layers on one GPU, every head (the unsharded reference point)
        rts = _sharded_build(nkv, dev, lambda li: nkv.M12LayerRuntime(
            li, nkv.M12Config(max_model_len=SH_CTX + 4096, device=dev)))
        xs, x, views = _sharded_inputs(dev)

        def step1():
            for rt, (q, k, v) in zip(rts, views):
                rt.decode(q, k, v, dev)
        us, _ = _graph_time(step1, xs, x, stream, steps, False)
        res["unsharded_1gpu_us_per_layer"] = round(us, 2)
        del rts, xs, x, views
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
    dist.barrier()
    return res


def prefill_measure(nkv, dev, iters=5):
    """Kernel (4) at BASELINE config 4: one 4096-token chunk at positions
    28672-32767 over its Top-32 blocks, sink, recent window and causal chunk."""
    g = torch.Generator(device=dev).manual_seed(4242)
    rt = nkv.M12LayerRuntime(0, nkv.M12Config(max_model_len=PF_HIST + PF_CHUNK + 4096, device=dev))
    for c in range(PF_HIST // PF_CHUNK):
        k = torch.randn(PF_CHUNK, HKV, D, generator=g, device=dev).bfloat16()
        v = torch.randn(PF_CHUNK, HKV, D, generator=g, device=dev).bfloat16()
        if c == 0:
            rt.prefill_first(None, k, v)
        else:
            rt._store_kv(k, v)
    q = torch.randn(PF_CHUNK, HQ, D, generator=g, device=dev).bfloat16()
    k = torch.randn(PF_CHUNK, HKV, D, generator=g, device=dev).bfloat16()
    v = torch.randn(PF_CHUNK, HKV, D, generator=g, device=dev).bfloat16()
    ids = rt._select_dev(nkv.m12_runtime.prefill_query_summaries(q, 1), TOPK)
    sink_len, ring_start, ring_len = rt._history_segments()

    def run():
        return rt._attend(q, ids, TOPK, sink_len, ring_start, ring_len, k, v, prefill=True)
    for _ in range(2):
        run()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        run()
    e1.record()
    e1.synchronize()
    us = e0.elapsed_time(e1) * 1000.0 / iters
    peak, kind = tensor_peak()
    tf = PF_FLOP / (us * 1e-6) / 1e12
    del rt
    return {"workload": "4096-token chunk at 28672 (Top-32, sink 64, recent 512, causal chunk), 32q/8kv d128",
            "us_per_chunk": round(us, 2), "flop_per_chunk": PF_FLOP,
            "roofline": {"bound": "tensor", "achieved": round(tf, 1), "peak": peak, "unit": "TFLOP/s",
                         "frac": round(tf / peak, 4), "peak_kind": kind}}


# kernel (5), store + representatives, per 4096-token chunk: read the chunk's
# K and V, write them into the block store, write the blocks' r
# representatives (+ int16 indices) and the last RECENT tokens into the ring
ST_T = 4096
ST_BYTES = (2 * ST_T * HKV * D * 2 + 2 * ST_T * HKV * D * 2 + (ST_T // B) * HKV * R_REPS * (D * 2 + 2)
            + 2 * min(ST_T, RECENT) * HKV * D * 2)
ST_ROT = 8  # distinct input chunks and store regions: 8 x 32 MiB > L2


def store_measure(nkv, dev, iters=16):
    """Kernel (5) on 4096-token chunks, rotating over ST_ROT inputs and store
    regions (their bytes exceed L2, so every launch reads and writes HBM)."""
    g = torch.Generator(device=dev).manual_seed(5151)
    rt = nkv.M12LayerRuntime(0, nkv.M12Config(max_model_len=ST_ROT * ST_T + 4096, device=dev))
    rt.reserve_blocks(ST_ROT * ST_T // B)
    ks = [torch.randn(ST_T, HKV, D, generator=g, device=dev).bfloat16() for _ in range(ST_ROT)]
    vs = [torch.randn(ST_T, HKV, D, generator=g, device=dev).bfloat16() for _ in range(ST_ROT)]
    rt._store_kv(ks[0], vs[0])  # first chunk: store, sink and ring set up

    def run_all():
        for j in range(ST_ROT):
            rt._launch_store(ks[j], vs[j], j * (ST_T // B), ring_pos0=0)
    run_all()  # eager once (kernel attributes), then the ST_ROT launches from a graph:
    torch.cuda.synchronize()  # the kernel's time, not the host's issue time
    st = torch.cuda.Stream(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=st):
        run_all()
    reps = max(1, iters // ST_ROT)
    with torch.cuda.stream(st):
        graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(reps):
            graph.replay()
        e1.record(st)
        e1.synchronize()
    us = e0.elapsed_time(e1) * 1000.0 / (reps * ST_ROT)
    del graph
    peak, kind = peaks()
    gbs = ST_BYTES / (us * 1e-6) / 1e9
    del rt
    return {"workload": "store + reps of a 4096-token chunk (bf16 block store, r=4), 8 rotating chunks > L2",
            "us_per_chunk": round(us, 2), "bytes_per_chunk": ST_BYTES,
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(gbs / peak, 4), "peak_kind": kind}}


def verify6_measure(nkv, dev, iters=50):
    """BASELINE config 4's multi-token variant as an operator: one layer state
    of 28672 tokens (7 stored 4096-token chunks), then verify_tokens over 6
    queries (the current token and 5 drafts) followed by rollback_verified, per
    call (eager, inputs rotating over 8 sets); per-query (lossless: union of
    the queries' Top-32 and a per-query mask) and shared selection."""
    g = torch.Generator(device=dev).manual_seed(606)
    rt = nkv.M12LayerRuntime(0, nkv.M12Config(max_model_len=PF_HIST + 4096, device=dev,
                                              verify_union_blocks=6 * TOPK))
    for c in range(PF_HIST // 4096):
        k = torch.randn(4096, HKV, D, generator=g, device=dev).bfloat16()
        v = torch.randn(4096, HKV, D, generator=g, device=dev).bfloat16()
        (rt.prefill_first(None, k, v) if c == 0 else rt._store_kv(k, v))
    sets = [tuple(torch.randn(6, h, D, generator=g, device=dev).bfloat16() for h in (HQ, HKV, HKV))
            for _ in range(NSETS)]
    rec = {"workload": "verify_tokens over 6 queries (current + 5 drafts) after a 28672-token history "
                       "(Top-32 per query, sink 64, recent 512), then rollback; eager calls"}
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for lossless in (True, False):
        rt.verify_lossless = lossless
        for i in range(5):
            rt.verify_tokens(*sets[i % NSETS], dev)
            rt.rollback_verified()
        torch.cuda.synchronize()
        e0.record()
        for i in range(iters):
            rt.verify_tokens(*sets[i % NSETS], dev)
            rt.rollback_verified()
        e1.record()
        e1.synchronize()
        rec["per_query_us" if lossless else "shared_us"] = round(e0.elapsed_time(e1) * 1000.0 / iters, 2)
        if lossless:
            rec["union_blocks_last_call"] = int(rt.last_verify_block_ids.numel())
    del rt
    return rec


# the full model decoding after a 32K prompt
MODEL_PROMPT, MODEL_CHUNK = 32768, 4096
C5_PROMPT, C5_STEPS = 131072, 256  # BASELINE config 5 (long context)
C3_STEPS = 128  # int8 history (per-token bf16 scales) in pinned host memory
C3_M12 = {"quant_history": True, "quant_scheme": "token", "kv_residency": "host"}
C3_LABEL = ("history int8 with per-token per-KV-head bf16 scales in pinned host memory; each decode step "
            "reads the selected blocks over the host link")


def model_measure(nkv, dev, steps=64, warmup=8, layer_us=None, prompt_len=None, speculative=True, seed=2,
                  m12=None, label=None, profile_replay=False):
    """Random-init Qwen3-4B-architecture model (36 layers) with the sparse
    runtime in every layer: a 32768-token prompt prefilled in 4096-token chunks
    (time to first token), then greedy decode replayed from one CUDA graph per
    token (DecodeLoop: embedding, 36 x [norm, qkv GEMM, q/k norm + RoPE, sparse
    decode step, o_proj GEMM, norm, gate/up GEMM, SwiGLU, down GEMM], final
    norm, LM head, argmax, token fed back on the device)."""
    H = nkv.qwen3_harness
    arch = H.Qwen3Arch()
    n_prompt = prompt_len or MODEL_PROMPT
    prompt = torch.randint(0, arch.vocab_size, (n_prompt,), generator=torch.Generator().manual_seed(seed))
    model = H.Qwen3SparseModel(arch, lambda i: nkv.M12LayerRuntime(
        i, nkv.M12Config(max_model_len=n_prompt + 4096, device=dev, **(m12 or {}))), device=dev, seed=0)
    # the history store reserved for the prompt before the timed prefill (the
    # reference's one-shot reserve_blocks), as a server does at setup: for the
    # host-resident history this is the pinned allocation, which would
    # otherwise grow by doubling inside the prefill
    for rt in model.runtimes:
        rt.reserve_blocks(-(-n_prompt // B))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    tok = model.prefill(prompt, MODEL_CHUNK)
    e1.record()
    e1.synchronize()
    ttft_ms = e0.elapsed_time(e1)
    tok = model.decode_step(tok)
    loop = H.DecodeLoop(model, tok, max_steps=warmup + steps + 8)
    loop.run(warmup)
    torch.cuda.synchronize()
    st = loop.stream
    with torch.cuda.stream(st):
        e0.record(st)
        for _ in range(steps):
            loop.replay()
        e1.record(st)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / steps
    if profile_replay:  # one more replay inside cudaProfilerStart/Stop (ncu --profile-from-start off)
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        with torch.cuda.stream(st):
            loop.replay()
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
    toks = loop.hist[:warmup + steps].tolist()
    model.check_errors()
    loop.close()
    # speculative verification through the model (eager): rounds of one verify
    # pass over [current token, 4 drafts] and a commit of all 5 (full
    # acceptance: the upper bound of a drafter), shared and per-query selection
    spec = {}
    cur = int(toks[-1])
    for lossless in ((False, True) if speculative else ()):
        for rt in model.runtimes:
            rt.verify_lossless = lossless
        times = []
        for r in range(2 + 8):
            drafts = [int(t) for t in toks[(r * 4) % 60:(r * 4) % 60 + 4]]
            torch.cuda.synchronize()
            e0.record()
            logits = model.verify([cur] + drafts)
            model.commit_verified(5)
            e1.record()
            e1.synchronize()
            if r >= 2:
                times.append(e0.elapsed_time(e1))
            cur = int(logits[-1].argmax())
        ms_v = statistics.median(times)
        spec["per_query" if lossless else "shared"] = {
            "verify_round_ms": round(ms_v, 3), "tok_s_at_full_acceptance": round(5000.0 / ms_v, 1)}
    for rt in model.runtimes:
        rt.verify_lossless = False
    model.check_errors()
    del loop, model
    torch.cuda.empty_cache()
    rec = {"workload": f"Qwen3-4B architecture (36 layers, random init bf16), {n_prompt}-token prompt in "
                       f"{MODEL_CHUNK}-token chunks, greedy decode from one CUDA graph per token"
                       + (f"; {label}" if label else ""),
           "decode_tok_s": round(1000.0 / ms, 1), "decode_ms_per_token": round(ms, 4),
           "prefill_ttft_ms": round(ttft_ms, 1), "decode_steps_timed": steps,
           "first_tokens": toks[:8]}
    if speculative:
        rec["speculative_verify"] = dict(spec, note="eager verify pass over [current, 4 drafts] through the 36 "
                                                    "layers + commit of all 5 tokens, median of 8 rounds; tok/s "
                                                    "at 100 % acceptance is the ceiling a drafter could reach")
    if layer_us is not None:
        rec["sparse_attention_share"] = round(layer_us * arch.num_layers / (ms * 1000.0), 3)
    return rec


class Clocks:
    """nvidia-smi sampling during the timed region."""

    def __init__(self, index):
        self.proc = None
        self.index = index
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={index}",
                 "--query-gpu=clocks.sm,clocks.max.sm,clocks_event_reasons.active,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 7:
                continue
            try:
                sm.append(float(f[0]))
                mx = float(f[1])
            except ValueError:
                continue
            for n, val in zip(names, f[3:7]):
                if val.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def build_layers(nkv, dev, n_layers, seed):
    """L layer runtimes, each with a 32K-token random history stored by kernel (5)."""
    g = torch.Generator(device=dev).manual_seed(seed)
    layers = []
    for li in range(n_layers):
        rt = nkv.M12LayerRuntime(li, nkv.M12Config(max_model_len=CTX + 4096, device=dev))
        rt.reserve_blocks(CTX // B)
        for c in range(CTX // 4096):
            k = torch.randn(4096, HKV, D, generator=g, device=dev).bfloat16()
            v = torch.randn(4096, HKV, D, generator=g, device=dev).bfloat16()
            if c == 0:
                rt.prefill_first(None, k, v)
            else:
                rt._store_kv(k, v)
        layers.append(rt)
    torch.cuda.synchronize()
    return layers


def cpu_reference(steps, warmup, threads):
    """The reference algorithm's CPU path restated (oracle port) on one 32K
    layer state: median decode call time in microseconds."""
    from oracle import m12_oracle as orc

    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(7)
    layer = orc.OracleLayer(orc.OracleConfig())
    for _ in range(CTX // 4096):
        k = torch.randn(4096, HKV, D, generator=g).bfloat16()
        v = torch.randn(4096, HKV, D, generator=g).bfloat16()
        layer.store(k, v)
    times = []
    for i in range(warmup + steps):
        q = torch.randn(1, HQ, D, generator=g).bfloat16()
        k = torch.randn(1, HKV, D, generator=g).bfloat16()
        v = torch.randn(1, HKV, D, generator=g).bfloat16()
        t = time.perf_counter()
        layer.decode(q, k, v)
        dt = time.perf_counter() - t
        if i >= warmup:
            times.append(dt)
    return statistics.median(times) * 1e6, len(times)


def reference_own(steps, warmup, threads, verify_iters=5):
    """The reference's own torch code on the host cores: its M12LayerRuntime
    (installed under baseline/_ref, run through the CPU device shim) decoding
    one 32K layer state (median of `steps` calls after `warmup`), and its
    6-query lossless verify at 28672 history (median of `verify_iters` calls,
    each followed by rollback_verified so the state is unchanged).  Returns
    None when the reference package is not installed."""
    from oracle import ref_shim

    if not ref_shim.reference_available():
        return None
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(7)
    rt = ref_shim.RefRuntime(max_model_len=CTX + 4096)
    for c in range(CTX // 4096):
        k = torch.randn(4096, HKV, D, generator=g).bfloat16()
        v = torch.randn(4096, HKV, D, generator=g).bfloat16()
        if c == 0:
            rt.prefill_first(None, k, v)
        else:
            rt._store_kv(k, v)
    times = []
    cpu = torch.device("cpu")
    for i in range(warmup + steps):
        q = torch.randn(1, HQ, D, generator=g).bfloat16()
        k = torch.randn(1, HKV, D, generator=g).bfloat16()
        v = torch.randn(1, HKV, D, generator=g).bfloat16()
        t = time.perf_counter()
        rt.decode(q, k, v, cpu)
        dt = time.perf_counter() - t
        if i >= warmup:
            times.append(dt)
    decode_us = statistics.median(times) * 1e6
    del rt
    # BASELINE config 4, multi-token variant: 5 draft tokens + 1 at 28672
    rv = ref_shim.RefRuntime(max_model_len=PF_HIST + 4096, verify_union_blocks=6 * TOPK)
    for c in range(PF_HIST // 4096):
        k = torch.randn(4096, HKV, D, generator=g).bfloat16()
        v = torch.randn(4096, HKV, D, generator=g).bfloat16()
        if c == 0:
            rv.prefill_first(None, k, v)
        else:
            rv._store_kv(k, v)
    rv.rt.verify_mode = True
    rv.rt.verify_lossless = True
    vt = []
    for i in range(1 + verify_iters):
        q = torch.randn(6, HQ, D, generator=g).bfloat16()
        k = torch.randn(6, HKV, D, generator=g).bfloat16()
        v = torch.randn(6, HKV, D, generator=g).bfloat16()
        t = time.perf_counter()
        rv.verify_tokens(q, k, v, cpu)
        dt = time.perf_counter() - t
        rv.rollback_verified()
        if i >= 1:
            vt.append(dt)
    return {"decode_us": decode_us, "decode_calls": len(times),
            "verify6_us": statistics.median(vt) * 1e6, "verify_calls": len(vt)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="nkv", choices=["nkv", "reference"])
    ap.add_argument("--layers", type=int, default=LAYERS)
    ap.add_argument("--cpu-steps", type=int, default=20)
    ap.add_argument("--no-prefill", action="store_true", help="skip the kernel (4) measurement")
    ap.add_argument("--no-offload", action="store_true", help="skip the host-offload decode measurement")
    ap.add_argument("--no-sharded", action="store_true", help="skip the KV-head-sharded measurement (N > 1)")
    ap.add_argument("--store-only", action="store_true",
                    help="run only the kernel (5) store measurement and print its record (profiling)")
    ap.add_argument("--offload-only", action="store_true",
                    help="run only the host-offload decode measurement and print its record (profiling)")
    ap.add_argument("--model-only", action="store_true",
                    help="run only the full-model decode measurement and print its record (profiling)")
    ap.add_argument("--no-model", action="store_true", help="skip the full-model decode tok/s measurement")
    ap.add_argument("--no-c5", action="store_true", help="skip the 131072-token full-model measurement (N = 1)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline (cpu_baseline is then null)")
    ap.add_argument("--profile-replay", action="store_true",
                    help="with --model-only: one extra config-2 decode replay between cudaProfilerStart/Stop")
    ap.add_argument("--no-c3", action="store_true", help="with --model-only: skip the config-3 record")
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    try:  # the cores this process may run on (cgroup / affinity), not the machine's
        threads = len(os.sched_getaffinity(0)) or 1
    except AttributeError:
        threads = os.cpu_count() or 1

    config = {"workload": "single-layer sparse decode (select+attend) @32K history, 36 layer states",
              "model": "Qwen3-4B attention geometry (32q/8kv, d128)", "context": CTX,
              "block": B, "reps": R_REPS, "top_k": TOPK, "sink": SINK, "recent": RECENT,
              "layers_per_step": args.layers, "global_batch": world, "seq_len": CTX,
              "parallelism": f"replicas{world}",
              "l2": "step touches ~540 MB of distinct KV/reps (> 126 MB L2); no flush"}

    if args.impl == "reference":
        if rank != 0:
            return
        n_steps = max(3, min(args.steps, 20) if args.steps < 20 else 20)
        own = reference_own(max(20, n_steps), max(3, args.warmup), threads)
        port_us, n_port = cpu_reference(n_steps, max(3, args.warmup), threads)
        if own is not None:
            us, kind = own["decode_us"], "reference"
            sample = (f"{own['decode_calls']} decode calls of one 32K layer state through the reference's "
                      f"own M12LayerRuntime (torch, CPU device shim), median")
        else:
            us, kind = port_us, "port"
            sample = f"{n_port} decode calls of one 32K layer state (oracle port), median"
        line = {"impl": "reference", "metric": METRIC, "value": round(us, 1), "unit": UNIT,
                "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": round(us * args.layers / 1000.0, 3),
                "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic", "config": config,
                "cpu_baseline": {"value": round(us, 1), "unit": UNIT, "cores": threads, "kind": kind,
                                 "sample": sample, "port_value": round(port_us, 1),
                                 "verify6_us_at_28672": None if own is None else round(own["verify6_us"], 1)},
                "e2e": {"value": round(us, 1), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line))
        return

    nkv = __import__("importlib").import_module(PKG)
    if args.store_only:
        print(json.dumps({"store": store_measure(nkv, torch.device("cuda", 0))}))
        return
    if args.offload_only:
        print(json.dumps({"offload": offload_measure(nkv, torch.device("cuda", 0))}))
        return
    if args.model_only:
        dev0 = torch.device("cuda", 0)
        rec = {"model": model_measure(nkv, dev0, profile_replay=args.profile_replay)}
        if not args.no_c3:
            rec["model_c3"] = model_measure(nkv, dev0, steps=C3_STEPS, warmup=8, speculative=False, m12=C3_M12,
                                            label=C3_LABEL)
        if not args.no_c5:
            rec["model_c5"] = model_measure(nkv, dev0, steps=C5_STEPS, warmup=8, prompt_len=C5_PROMPT,
                                            speculative=False)
        print(json.dumps(rec))
        return
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120))
    dev = torch.device("cuda", local if world > 1 else 0)
    torch.cuda.set_device(dev)
    L = args.layers
    layers = build_layers(nkv, dev, L, seed=1234 + rank)

    # NSETS distinct q/k/v sets per layer; step s decodes set s % NSETS, copied
    # into a persistent staging buffer whose per-layer views are the decode
    # inputs (as a model's qkv projection output would be), so the selection
    # changes from step to step
    QKV = (HQ + 2 * HKV) * D
    gq = torch.Generator(device=dev).manual_seed(99 + rank)
    xsets = torch.randn(NSETS, L, QKV, generator=gq, device=dev).bfloat16()
    xdev = torch.empty(L, QKV, dtype=torch.bfloat16, device=dev)
    xdev.copy_(xsets[0])
    views = [(xdev[li, :HQ * D].view(1, HQ, D), xdev[li, HQ * D:(HQ + HKV) * D].view(1, HKV, D),
              xdev[li, (HQ + HKV) * D:].view(1, HKV, D)) for li in range(L)]
    qs = [vw[0] for vw in views]
    ks = [vw[1] for vw in views]
    vs = [vw[2] for vw in views]

    stream = torch.cuda.Stream(dev)
    # warm the kernels once eagerly (workspace allocation happens here)
    with torch.cuda.stream(stream):
        for li, rt in enumerate(layers):
            rt.decode(qs[li], ks[li], vs[li], dev)
    stream.synchronize()
    attend_cfg = nkv._lib.attend_last_config()

    # whole step (select + attend for every layer) recorded once and replayed
    # per token with the recent windows advancing on the device (DecodeGraph)
    graph = nkv.DecodeGraph(layers, views, stream=stream)
    # kernel (2) alone, for the roofline of the dominant kernel: the step's
    # attention kernel (tile-split, it ranks the block scores itself) on each
    # layer's block scores saved from one scoring pass, back to back
    with torch.cuda.stream(stream):
        scores_saved = [rt.block_scores_dev(qs[li]).clone() for li, rt in enumerate(layers)]
    stream.synchronize()
    g_att = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_att, stream=stream):
        for li, rt in enumerate(layers):
            d, _, _ = rt._decode_fill(qs[li], ks[li], vs[li], TOPK)
            a = nkv._lib.AttendArgs.from_buffer_copy(d.attend)
            a.block_ids, a.n_sel, a.overlap_select = rt._ids.data_ptr(), TOPK, 0
            nkv._lib.call("nkv_attend_ranked", stream.cuda_stream, ctypes.byref(a), scores_saved[li].data_ptr(),
                          scores_saved[li].numel(), rt._ids.data_ptr(), rt._topk_scores.data_ptr())
    att_kernel = "decode_split_kernel" if nkv._lib.attend_last_config()[0] == 2 else "decode_kernel"

    def timed(g, iters, rotate=True):
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            ev0.record(stream)
            for i in range(iters):
                if rotate:
                    xdev.copy_(xsets[i % NSETS], non_blocking=True)
                g.replay()
            ev1.record(stream)
        ev1.synchronize()
        return ev0.elapsed_time(ev1)

    def timed_copies(iters):
        """The per-step input copies alone (reported beside the step time)."""
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            ev0.record(stream)
            for i in range(iters):
                xdev.copy_(xsets[i % NSETS], non_blocking=True)
            ev1.record(stream)
        ev1.synchronize()
        return ev0.elapsed_time(ev1)

    with torch.cuda.stream(stream):
        for i in range(max(3, args.warmup)):
            xdev.copy_(xsets[i % NSETS], non_blocking=True)
            graph.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clk = Clocks(local) if rank == 0 else None
    ms = timed(graph, args.steps)
    ms_copy = timed_copies(args.steps)
    torch.cuda.synchronize()
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    clocks = clk.stop() if clk else None
    ms_per_step = ms / args.steps
    value = ms_per_step * 1000.0 / (L * world)

    # dominant kernel (attend) timed alone
    for _ in range(3):
        g_att.replay()
    att_ms = timed(g_att, args.steps, rotate=False) / args.steps
    att_us = att_ms * 1000.0 / L
    peak, peak_kind = peaks()
    achieved = ATTEND_BYTES / (att_us * 1e-6) / 1e9
    step_gbs = STEP_BYTES / (ms_per_step * 1000.0 / L * 1e-6) / 1e9

    # end to end through the public API: the step's q/k/v for every layer
    # copied from pinned host memory in one transfer (NSETS distinct sets in
    # rotation), eager rt.decode per layer, the step's outputs gathered and
    # copied back in one transfer
    hsets = torch.randn(NSETS, L, QKV, generator=torch.Generator().manual_seed(199 + rank)).bfloat16().pin_memory()
    ho = torch.empty(L, 1, HQ, D, dtype=torch.bfloat16).pin_memory()
    e2e_steps = max(3, min(args.steps, 20))
    e2e_i = [0]

    def next_host_set():
        e2e_i[0] += 1
        return hsets[e2e_i[0] % NSETS]
    with torch.cuda.stream(stream):
        def e2e_step():
            xdev.copy_(next_host_set(), non_blocking=True)
            outs = [rt.decode(q, k, v, dev) for rt, (q, k, v) in zip(layers, views)]
            ho.copy_(torch.stack(outs), non_blocking=True)
        for _ in range(2):
            e2e_step()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        h0 = time.perf_counter()
        for _ in range(e2e_steps):
            e2e_step()
        host_us = (time.perf_counter() - h0) * 1e6 / (e2e_steps * L)  # host issue time per layer
        e1.record(stream)
        e1.synchronize()
    e2e_eager_ms = e0.elapsed_time(e1) / e2e_steps
    # the same end-to-end step through DecodeGraph: the per-step copies as
    # above, the layers' decode replayed from one CUDA graph whose recent
    # windows advance on the device with every replay
    dg = graph
    with torch.cuda.stream(stream):
        def e2e_graph_step():
            xdev.copy_(next_host_set(), non_blocking=True)
            ho.copy_(dg.replay(), non_blocking=True)
        for _ in range(2):
            e2e_graph_step()
        torch.cuda.synchronize()
        e0.record(stream)
        h0 = time.perf_counter()
        for _ in range(e2e_steps):
            e2e_graph_step()
        graph_host_us = (time.perf_counter() - h0) * 1e6 / (e2e_steps * L)
        e1.record(stream)
        e1.synchronize()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    if world > 1:
        t = torch.tensor([e2e_ms, e2e_eager_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms, e2e_eager_ms = float(t[0].item()), float(t[1].item())
    e2e_value = e2e_ms * 1000.0 / (L * world)
    e2e_eager_value = e2e_eager_ms * 1000.0 / (L * world)

    line = None
    prefill = offload = sharded = None
    if world > 1 and not args.no_sharded:
        sharded = sharded_measure(nkv, dev, world)
    if rank == 0 and not args.no_prefill:
        with torch.cuda.stream(stream):
            prefill = prefill_measure(nkv, dev)
    if rank == 0 and not args.no_offload:
        offload = offload_measure(nkv, dev)
    store = store_measure(nkv, dev) if rank == 0 else None
    verify6 = verify6_measure(nkv, dev) if rank == 0 else None
    model = model_c3 = model_c5 = None
    if not args.no_model:
        del graph, g_att, dg
        graph = g_att = dg = None
        for rt in layers:
            rt.reset()
        torch.cuda.empty_cache()
        if world == 1:
            model = model_measure(nkv, dev, layer_us=value * world)
            # the same model with the int8 history offloaded
            model_c3 = model_measure(nkv, dev, steps=C3_STEPS, warmup=8, speculative=False, m12=C3_M12,
                                     label=C3_LABEL)
            if not args.no_c5:
                # BASELINE config 5 on one GPU: a 131072-token prompt, 256 greedy steps
                model_c5 = model_measure(nkv, dev, steps=C5_STEPS, warmup=8, prompt_len=C5_PROMPT,
                                         speculative=False)
        else:
            # config 5's throughput variant: one independent 32K sequence per GPU
            # (a different prompt on every rank), whole-job tok/s over the
            # slowest rank's time per token
            rec = model_measure(nkv, dev, speculative=False, seed=2 + rank)
            t = torch.tensor([rec["decode_ms_per_token"], rec["prefill_ttft_ms"]], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            if rank == 0:
                ms_tok, ttft = float(t[0].item()), float(t[1].item())
                model = dict(rec, workload=f"{world} independent sequences, one per GPU: " + rec["workload"],
                             decode_ms_per_token=round(ms_tok, 4), prefill_ttft_ms=round(ttft, 1),
                             decode_tok_s=round(world * 1000.0 / ms_tok, 1),
                             decode_tok_s_per_gpu=round(1000.0 / ms_tok, 1), replicas=world,
                             timing="max over ranks")
    if rank == 0:
        # the CPU baseline is timed at N = 1 only (with N > 1 other ranks share the host)
        own = port = None
        if world == 1 and not args.no_cpu:
            own = reference_own(args.cpu_steps, 3, threads)
            port = cpu_reference(args.cpu_steps, 3, threads)
        line = {
            "metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5),
            "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) K/V/Q)", "config": config,
            "step_hbm_gbs": round(step_gbs, 1),
            "roofline": {"bound": "hbm", "kernel": f"{att_kernel} (kernel 2), ranked on saved block scores",
                         "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                         "us_per_launch": round(att_us, 3), "bytes_per_launch": ATTEND_BYTES,
                         "traffic": ATTEND_TRAFFIC,
                         "traffic_source": "recorded constant: ncu dram__bytes_read+write of one launch "
                                           "of this kernel, from a separate capture (not measured in this run)"},
            "cpu_baseline": None if port is None else {
                "value": round(own["decode_us"] if own else port[0], 1), "unit": UNIT, "cores": threads,
                "kind": "reference" if own else "port",
                "sample": (f"{own['decode_calls']} decode calls of one 32K layer state through the reference's own "
                           "M12LayerRuntime (torch, CPU device shim), median") if own else
                          f"{port[1]} decode calls of one 32K layer state (oracle port), median",
                "port_value": round(port[0], 1),
                "verify6_us_at_28672": round(own["verify6_us"], 1) if own else None},
            "e2e": {"value": round(e2e_value, 4), "unit": UNIT, "api": "DecodeGraph.replay (all layers)",
                    "host_us_per_layer": round(graph_host_us, 2),
                    "h2d_bytes_per_step": L * (HQ + 2 * HKV) * D * 2,
                    "d2h_bytes_per_step": L * HQ * D * 2},
            "e2e_eager": {"value": round(e2e_eager_value, 4), "unit": UNIT,
                          "api": "M12LayerRuntime.decode per layer", "host_us_per_layer": round(host_us, 2),
                          "h2d_bytes_per_step": L * (HQ + 2 * HKV) * D * 2,
                          "d2h_bytes_per_step": L * HQ * D * 2},
            "gpu_launches": 2 * L * args.steps,
            "attend_launch": {"cluster": attend_cfg[0], "splits_per_head": attend_cfg[1],
                              "keys_per_cta": attend_cfg[2]},
            "clocks": clocks,
            "prefill": prefill,
            "offload": offload,
            "store": store,
            "verify6": verify6,
            "kv_head_sharded": sharded,
            "model": model,
            "model_c3": model_c3,
            "model_c5": model_c5,
        }
        print(json.dumps(line))
    del graph, g_att, dg
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
