"""Seeded input streams shared by the golden generator and the parity tests.

Every case regenerates its tensors from a CPU ``torch.Generator`` so the committed
fixtures hold only outputs (selected ids, representative token indices, sampled
output rows), never the inputs.
"""
from __future__ import annotations

import torch

HQ, HKV, D = 32, 8, 128


def qkv(gen: torch.Generator, t: int, dtype=torch.bfloat16):
    q = torch.randn(t, HQ, D, generator=gen).to(dtype)
    k = torch.randn(t, HKV, D, generator=gen).to(dtype)
    v = torch.randn(t, HKV, D, generator=gen).to(dtype)
    return q, k, v


def sample_rows(t: int, n: int = 24) -> torch.Tensor:
    """Deterministic subset of query rows stored for long prefill outputs."""
    if t <= n:
        return torch.arange(t)
    g = torch.Generator().manual_seed(1234 + t)
    mid = torch.randperm(t - 6, generator=g)[: n - 6] + 3
    return torch.cat([torch.arange(3), mid.sort().values, torch.arange(t - 3, t)])


# Each case: config overrides for M12Config and a script of operations.
# ("first", T) prefill_first, ("chunk", T) prefill_chunk, ("store", T) a chunk
# stored without attention (the runtime's _store_kv), ("decode",) one step,
# ("verify", Tq, lossless) verify_tokens, ("commit", n) commit_verified.
CASES = {
    "decode_c1": dict(
        seed=1,
        cfg=dict(top_k_blocks=32, sink_tokens=64, recent_tokens=512),
        script=[("first", 8192), ("decode",), ("decode",)],
    ),
    "chunks": dict(
        seed=2,
        cfg=dict(top_k_blocks=8, sink_tokens=64, recent_tokens=512,
                 verify_union_blocks=48),
        script=[("first", 1024), ("chunk", 1024), ("chunk", 1024), ("chunk", 333),
                ("decode",), ("decode",), ("verify", 6, True), ("verify", 6, False),
                ("commit", 3), ("decode",)],
    ),
    "quant": dict(
        seed=3,
        cfg=dict(top_k_blocks=16, sink_tokens=64, recent_tokens=512, quant_history=True),
        script=[("first", 4096), ("chunk", 1024), ("decode",), ("decode",)],
    ),
    "short": dict(
        seed=4,
        cfg=dict(top_k_blocks=32, sink_tokens=64, recent_tokens=512),
        script=[("first", 200), ("decode",), ("decode",), ("decode",)],
    ),
    "segments": dict(
        seed=5,
        cfg=dict(top_k_blocks=12, sink_tokens=64, recent_tokens=256,
                 prefill_query_segments=4),
        script=[("first", 2048), ("chunk", 512), ("decode",)],
    ),
    # decode selection variants (reference m12_runtime.py:1015-1046, 1181-1190)
    "relative": dict(
        seed=6,
        cfg=dict(top_k_blocks=16, sink_tokens=64, recent_tokens=512,
                 decode_relative_a=0.9, decode_relative_max_blocks=24),
        script=[("first", 8192), ("decode",), ("decode",), ("decode",), ("decode",)],
    ),
    "relative_union": dict(
        seed=7,
        cfg=dict(top_k_blocks=4, sink_tokens=64, recent_tokens=512,
                 decode_relative_a=0.5, decode_relative_max_blocks=24, decode_relative_union=True),
        script=[("first", 8192), ("decode",), ("decode",), ("decode",)],
    ),
    "dynamic": dict(
        seed=8,
        cfg=dict(top_k_blocks=32, sink_tokens=64, recent_tokens=512,
                 dynamic_top_k=True, dynamic_top_k_mass=0.9),
        script=[("first", 8192), ("decode",), ("decode",), ("decode",), ("decode",)],
    ),
    "qwindow": dict(
        seed=9,
        cfg=dict(top_k_blocks=16, sink_tokens=64, recent_tokens=512, decode_query_window=4),
        script=[("first", 8192)] + [("decode",)] * 6,
    ),
    # BASELINE config 4's multi-token variant: 6 queries (5 draft + 1) over a
    # 28672-token history, lossless per-query selection (union <= 192 blocks)
    "verify28k": dict(
        seed=10,
        max_model_len=32768,
        cfg=dict(top_k_blocks=32, sink_tokens=64, recent_tokens=512, verify_union_blocks=192),
        script=[("first", 4096)] + [("store", 4096)] * 6 + [
            ("verify", 6, True), ("verify", 6, False), ("commit", 2), ("decode",)],
    ),
}
