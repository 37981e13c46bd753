"""Golden vectors of the reference's n-gram proposer (nanovllm/sparse/proposers.py:
NgramProposer), for tests/test_harness_host.py.

Run where the reference package is importable (``baseline/_ref``, or the
checkout named by ``$NKV_REFERENCE_ROOT``):

    python tests/golden/make_ngram_golden.py

Each case: a seeded prompt over a small vocabulary (so that n-grams repeat),
then a scripted sequence of rounds: propose(last_token, k, pos), and
note_accepted(the first `accept` proposals); the proposals are recorded.
"""
from __future__ import annotations

import json
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from oracle.ref_shim import REFERENCE_ROOT  # noqa: E402

CASES = [  # (seed, prompt length, vocabulary, n, max_k, rounds); vocabulary < 0: a repeated
    (1, 200, 4, 3, 6, 12),     # pattern of |vocabulary| tokens with a few substitutions
    (2, 64, 3, 2, 8, 10),
    (3, 400, 6, 4, 4, 16),
    (4, 300, -17, 4, 8, 12),
    (5, 3, 10, 4, 8, 3),       # prompt shorter than n
]


def script(seed, rounds):
    g = torch.Generator().manual_seed(seed + 100)
    return [(int(torch.randint(0, 10, (1,), generator=g)), int(torch.randint(1, 9, (1,), generator=g)),
             int(torch.randint(0, 4, (1,), generator=g))) for _ in range(rounds)]


def prompt(seed, n, vocab):
    g = torch.Generator().manual_seed(seed)
    if vocab > 0:
        return [int(t) for t in torch.randint(0, vocab, (n,), generator=g)]
    pat = [int(t) for t in torch.randint(0, 50, (-vocab,), generator=g)]
    ids = [pat[i % len(pat)] for i in range(n)]
    for i in torch.randint(0, n, (n // 25,), generator=g).tolist():
        ids[i] = 50 + i % 7
    return ids


def main():
    sys.path.insert(0, REFERENCE_ROOT)
    from nanovllm.sparse.proposers import NgramProposer
    out = []
    for seed, n_prompt, vocab, n, max_k, rounds in CASES:
        p = NgramProposer(n=n, max_k=max_k)
        ids = prompt(seed, n_prompt, vocab)
        p.prefill(ids)
        last = ids[-1] if ids else 0
        rec = []
        for i, (tok_off, k, accept) in enumerate(script(seed, rounds)):
            last_token = (last + tok_off) % abs(vocab) if i % 3 == 2 else last
            props = p.propose(last_token, k, n_prompt + i)
            acc = props[:accept]
            p.note_accepted(acc)
            rec.append({"last_token": last_token, "k": k, "proposals": props, "accepted": acc})
            last = acc[-1] if acc else (props[0] if props else last_token)
        out.append({"seed": seed, "prompt_len": n_prompt, "vocab": vocab, "n": n, "max_k": max_k, "rounds": rec})
    with open(os.path.join(HERE, "ngram.json"), "w") as f:
        json.dump(out, f, indent=0)
    print("wrote", os.path.join(HERE, "ngram.json"))


if __name__ == "__main__":
    main()
