"""Pin the CPU oracle to fixtures produced by the reference runtime itself.

The fixtures (tests/golden/*.pt) come from ``make_golden.py``, which runs the
reference ``M12LayerRuntime`` on the host.  These tests replay the same seeded
scripts through ``oracle.m12_oracle`` and require: representative token indices
equal (except fp32 near-ties), selected ids equal modulo score ties within 1e-3,
outputs within one bf16 rounding of the reference's bf16 outputs, and identical
bookkeeping (valid_len, nblocks, protected set).
"""
import pytest
import torch

from helpers import CASES, OracleReplay, ids_match_modulo_ties, load_golden, orc


@pytest.mark.parametrize("name", sorted(CASES))
def test_oracle_matches_reference_fixture(name):
    golden = load_golden(name)
    replay = OracleReplay(name, golden=golden)
    for step, (g, o) in enumerate(zip(golden["steps"], replay.steps())):
        assert g["op"] == o["op"]
        assert g["valid_len"] == o["valid_len"], step
        assert g["nblocks"] == o["nblocks"], step
        assert g["protected"] == o["protected"], step
        if "rep_idx" in g:
            same = g["rep_idx"].long() == o["rep_idx"]
            # a flip is only acceptable where the oracle's decision margin is tiny
            assert bool((same | (o["rep_margin"] < 1e-5)).all()), step
        if "ids" in g:
            ok, why = ids_match_modulo_ties(o["ids"], g["ids"], o["scores"]) \
                if g["op"][0] != "verify" or not g["op"][2] else \
                (torch.equal(o["ids"], g["ids"]), "union")
            assert ok, f"step {step} {g['op']}: {why}"
        if "o" in g:
            want = g["o"].float()
            got = o["o"]
            if "rows" in g:
                got = got[g["rows"]]
            # reference output is bf16 of the same fp32 math: allow 1-2 bf16 ulps
            torch.testing.assert_close(got, want, atol=2e-2, rtol=1e-2)


def test_recent_slice_known_answers():
    # reference tests/test_m14_prefill_layout.py:34-44
    assert orc.recent_slice(4096, 64, 512) == (3584, 0, 512)
    assert orc.recent_slice(128, 64, 512) == (0, 64, 64)
    assert orc.recent_slice(64, 64, 512) == (0, 64, 0)


def test_dynamic_budget_known_answers():
    # reference tests/test_m16_dynamic_topk.py:13-22
    assert orc.dynamic_budget(torch.ones(32), 32, 0.90) == 32
    assert orc.dynamic_budget(torch.arange(10, 0, -1).float(), 32, 0.90) == 10
    assert orc.dynamic_budget(torch.tensor([float("inf")] + [0.0] * 31), 32, 0.90) == 32
    assert orc.dynamic_budget(torch.tensor([10.0] + [0.0] * 31), 32, 0.90) == 16


def test_query_summaries_are_segment_means():
    q = torch.arange(8 * 2 * 3, dtype=torch.float32).view(8, 2, 3)
    torch.testing.assert_close(orc.query_summaries(q, 1)[0], q.mean(0))
    want = torch.stack([q[0:2].mean(0), q[2:4].mean(0), q[4:6].mean(0), q[6:8].mean(0)])
    torch.testing.assert_close(orc.query_summaries(q, 4), want)
