"""CPU tests of the full-model harness's host-side pieces."""
import os
from importlib import import_module

import torch

from helpers import GOLDEN, pkg


def test_rope_table_matches_reference_yarn_cache():
    """The harness's YaRN cos/sin table equals the reference's own cache
    (fixture from tests/golden/make_rope_golden.py) bit for bit on the CPU."""
    H = import_module(pkg().__name__ + ".qwen3_harness")
    fx = torch.load(os.path.join(GOLDEN, "rope.pt"))
    arch = H.Qwen3Arch()
    assert arch.max_position == fx["max_position"]
    table = H.rope_cos_sin(arch, "cpu")
    assert table.shape == (fx["max_position"], 128)
    assert torch.equal(table[fx["positions"]], fx["rows"])


def test_harness_declares_the_c2_architecture():
    H = import_module(pkg().__name__ + ".qwen3_harness")
    a = H.Qwen3Arch()
    assert (a.num_layers, a.hidden_size, a.num_heads, a.num_kv_heads, a.head_dim) == (36, 2560, 32, 8, 128)
    assert (a.intermediate_size, a.vocab_size, a.rope_theta) == (9728, 151936, 1e6)
    assert a.rope_scaling["factor"] == 4.0 and a.rope_scaling["original_max_position_embeddings"] == 32768
