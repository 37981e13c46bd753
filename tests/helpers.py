"""Shared test helpers: golden loading, oracle replay, tie-aware id comparison."""
from __future__ import annotations

import importlib
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
for p in (ROOT, GOLDEN):
    if p not in sys.path:
        sys.path.insert(0, p)

from cases import CASES, qkv  # noqa: E402
from oracle import m12_oracle as orc  # noqa: E402

PKG_NAME = "nano-vllm-kv-optimizer_b200"


def pkg():
    """The product package (its directory name is not a Python identifier)."""
    return importlib.import_module(PKG_NAME)


def load_golden(name):
    return torch.load(os.path.join(GOLDEN, f"{name}.pt"), weights_only=False)


def ids_match_modulo_ties(got, want, scores, tol=1e-3):
    """True when ``got`` equals ``want`` except where their fp32 scores tie within tol.

    ``scores`` are the masked block scores both selections were ranked by.  The
    lists must have equal length; a position may differ only if the two blocks'
    scores are within ``tol``; a block present in one list only must score
    within ``tol`` of the last selected score.
    """
    got = [int(x) for x in got]
    want = [int(x) for x in want]
    if len(got) != len(want):
        return False, f"length {len(got)} != {len(want)}"
    s = scores.double()
    for i, (a, b) in enumerate(zip(got, want)):
        if a != b and abs(float(s[a]) - float(s[b])) > tol:
            return False, f"pos {i}: {a} ({float(s[a])}) vs {b} ({float(s[b])})"
    if want:
        cutoff = float(s[want[-1]])
        for x in set(got) ^ set(want):
            if abs(float(s[x]) - cutoff) > tol:
                return False, f"block {x} differs beyond tie tolerance"
    return True, ""


class OracleReplay:
    """Drive the oracle through a golden case's script, yielding per-step results."""

    def __init__(self, name, golden=None, **overrides):
        self.golden = golden
        spec = CASES[name]
        self.spec = spec
        cfg = dict(spec["cfg"])
        cfg.pop("verify_union_blocks", None)
        cfg.update(overrides)
        self.layer = orc.OracleLayer(orc.OracleConfig(**cfg))
        self.gen = torch.Generator().manual_seed(spec["seed"])

    def steps(self):
        L = self.layer
        for i, op in enumerate(self.spec["script"]):
            out = {"op": op}
            if self.golden is not None and "ids" in self.golden["steps"][i]:
                # follow the reference's choice among tied blocks so that the
                # outputs stay comparable; own_ids keeps the oracle's own pick
                if op[0] != "verify" or not op[2]:
                    L.force_ids = self.golden["steps"][i]["ids"]
            if op[0] in ("first", "chunk", "store"):
                q, k, v = qkv(self.gen, op[1])
                out["inputs"] = (q, k, v)
                start = L.nblocks
                if op[0] == "first":
                    out["o"] = L.prefill_first(q, k, v)
                elif op[0] == "store":
                    L.store(k, v)
                else:
                    out["o"] = L.prefill_chunk(q, k, v)
                    out["ids"], out["scores"] = L.last_ids, L.last_scores
                out["rep_idx"] = L.rep_idx[:, start:]
                out["rep_margin"] = L.rep_margin[:, start:]
            elif op[0] == "decode":
                q, k, v = qkv(self.gen, 1)
                out["inputs"] = (q, k, v)
                out["o"] = L.decode(q, k, v)
                out["ids"], out["scores"] = L.own_ids, L.last_scores
            elif op[0] == "verify":
                q, k, v = qkv(self.gen, op[1])
                out["inputs"] = (q, k, v)
                out["o"] = L.verify(q, k, v, lossless=op[2])
                out["ids"], out["scores"] = L.own_ids, L.last_scores
            elif op[0] == "commit":
                L.commit(op[1])
            out["valid_len"] = L.valid_len
            out["nblocks"] = L.nblocks
            out["protected"] = sorted(L.protected)
            yield out
