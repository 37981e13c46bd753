"""The oracle layer behind the attention-runtime interface of the full-model
harness (``Qwen3SparseModel``), for the greedy token-ID parity runs.

TEST INFRASTRUCTURE ONLY: the harness normally runs this package's CUDA
``M12LayerRuntime``; the tests swap every layer's runtime for this adapter and
run the same model again, so the two token streams differ only in the sparse
attention path.  The adapter calls ``oracle.m12_oracle`` (fp32 torch, on the
model's CUDA device with TF32 off) and returns bf16 outputs, as the reference's
``_fused_attention`` does (``nanovllm/sparse/m12_runtime.py:845-896``).
"""
from __future__ import annotations

import dataclasses

import torch

from . import m12_oracle as orc


class OracleAttentionRuntime:
    """``first_chunk_attention`` / ``prefill_first`` / ``prefill_chunk`` /
    ``decode`` / ``verify_tokens`` / ``commit_verified`` / ``rollback_verified``
    over an ``OracleLayer`` (reference ``M12LayerRuntime`` semantics)."""

    def __init__(self, cfg: orc.OracleConfig, device):
        self.cfg = dataclasses.replace(cfg, device=str(device))
        self.layer = orc.OracleLayer(self.cfg)
        self.verify_mode = False
        self.verify_lossless = False
        self.enabled = True

    @property
    def prefill_len(self):
        return self.layer.prefill_len

    @property
    def valid_len(self):
        return self.layer.valid_len

    @property
    def last_block_ids(self):
        return self.layer.last_ids

    def first_chunk_attention(self, q, k, v):
        """Dense causal attention inside the first chunk (the reference
        caller's FA2 varlen call, ``nanovllm/layers/attention.py:80-85``)."""
        return orc.attention(q, k, v, self.cfg.scale, causal_from=0).to(q.dtype)

    def prefill_first(self, q, k, v):
        self.layer.store(k, v)
        return {"nblocks": self.layer.nblocks, "valid_len": self.layer.valid_len}

    def prefill_chunk(self, q, k, v, device):
        return self.layer.prefill_chunk(q, k, v).to(q.dtype)

    def decode(self, q, k, v, device):
        return self.layer.decode(q, k, v).to(q.dtype)

    def verify_tokens(self, q, k, v, device):
        return self.layer.verify(q, k, v, lossless=self.verify_lossless).to(q.dtype)

    def commit_verified(self, n):
        self.layer.commit(n)

    def rollback_verified(self):
        self.layer.pending = None
