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


def test_ngram_proposer_matches_reference_vectors():
    """NgramProposer reproduces the reference's n-gram proposer on scripted
    rounds (fixture from tests/golden/make_ngram_golden.py)."""
    import json
    import sys
    sys.path.insert(0, GOLDEN)
    from make_ngram_golden import prompt
    P = import_module(pkg().__name__ + ".proposers")
    with open(os.path.join(GOLDEN, "ngram.json")) as f:
        cases = json.load(f)
    assert any(r["proposals"] for c in cases for r in c["rounds"])
    for c in cases:
        p = P.NgramProposer(n=c["n"], max_k=c["max_k"])
        p.prefill(prompt(c["seed"], c["prompt_len"], c["vocab"]))
        for i, r in enumerate(c["rounds"]):
            got = p.propose(r["last_token"], r["k"], c["prompt_len"] + i)
            assert got == r["proposals"], (c["seed"], i, got, r["proposals"])
            p.note_accepted(r["accepted"])
