"""Generate tests/golden/rope.pt: rows of the reference's YaRN cos/sin cache.

Run where the reference package is importable (``baseline/_ref``, or the
checkout named by ``$NKV_REFERENCE_ROOT``):

    python tests/golden/make_rope_golden.py

Builds the reference's ``YaRNRotaryEmbedding`` (``nanovllm/layers/rotary_embedding.py``)
with the Qwen3-4B settings of BASELINE config 2 (head_dim 128, rope_theta 1e6,
YaRN factor 4 over 32768 original positions, the cache extended as
``Qwen3Attention`` does, ``nanovllm/models/qwen3.py:56-66``) and stores the cache
rows of a fixed set of positions.
"""
from __future__ import annotations

import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
from oracle.ref_shim import REFERENCE_ROOT  # noqa: E402

POSITIONS = [0, 1, 2, 100, 4095, 4096, 32767, 32768, 65536, 131071, 133119]


def main():
    sys.path.insert(0, REFERENCE_ROOT)
    from nanovllm.layers.rotary_embedding import YaRNRotaryEmbedding

    max_position = max(40960, int(32768 * 4.0)) + 2048
    emb = YaRNRotaryEmbedding(128, 128, max_position, 1e6, factor=4.0, original_max_position_embeddings=32768)
    cache = emb.cos_sin_cache[:, 0]
    torch.save({"positions": POSITIONS, "rows": cache[POSITIONS].clone(), "max_position": max_position,
                "attention_scaling": emb.attention_scaling}, os.path.join(HERE, "rope.pt"))
    print("rope.pt", cache.shape)


if __name__ == "__main__":
    main()
