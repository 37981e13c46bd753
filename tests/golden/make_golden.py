"""Generate the committed golden fixtures by running the REFERENCE runtime on CPU.

Run where the reference package is importable (``baseline/_ref``, or the
checkout named by ``$NKV_REFERENCE_ROOT``):

    python tests/golden/make_golden.py [--check-oracle]

For each case in ``cases.py`` the reference ``M12LayerRuntime`` (via ``oracle/ref_shim.py``)
is driven through the case's script on seeded inputs.  The fixture stores, per
step: the selected block ids (reference ``last_block_ids``), the representative
token indices recovered from the reference's ``reps_gpu``, and the attention
output (all rows for decode/verify, ``sample_rows`` for prefill chunks).  Inputs
are regenerated from the seed by the tests, so nothing large is committed.
"""
from __future__ import annotations

import argparse
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from cases import CASES, HKV, HQ, D, qkv, sample_rows  # noqa: E402
from oracle.ref_shim import RefRuntime  # noqa: E402


def rep_indices(reps: torch.Tensor, k_blocks: torch.Tensor) -> torch.Tensor:
    """Recover which token of each block every representative copies.

    reps [Hkv, N, r, D]; k_blocks [N, B, Hkv, D].  Returns int16 [Hkv, N, r].
    """
    kb = k_blocks.permute(2, 0, 1, 3)                   # [H, N, B, D]
    eq = (reps.unsqueeze(3) == kb.unsqueeze(2)).all(-1)  # [H, N, r, B]
    idx = eq.float().argmax(-1)
    assert bool(eq.any(-1).all()), "representative is not a stored key"
    return idx.to(torch.int16)


def run_case(name: str, spec: dict) -> dict:
    gen = torch.Generator().manual_seed(spec["seed"])
    rt = RefRuntime(max_model_len=max(16384, spec.get("max_model_len", 0)), **spec["cfg"])
    B = rt.cfg.block_size
    steps = []
    all_k = []
    for op in spec["script"]:
        rec = {"op": op}
        if op[0] in ("first", "chunk", "store"):
            t = op[1]
            q, k, v = qkv(gen, t)
            start = rt.rt.nblocks_filled
            if op[0] == "first":
                rt.prefill_first(q, k, v)
                o = None
            elif op[0] == "store":
                rt._store_kv(k, v)
                o = None
            else:
                o = rt.prefill_chunk(q, k, v, torch.device("cpu"))
                rec["ids"] = rt.rt.last_prefill_block_ids.clone()
            nb = -(-t // B)
            kpad = torch.cat([k, k.new_zeros(nb * B - t, HKV, D)]).view(nb, B, HKV, D)
            rec["rep_idx"] = rep_indices(rt.rt.reps_gpu[:, start:start + nb], kpad)
            if o is not None:
                rows = sample_rows(t)
                rec["rows"] = rows
                rec["o"] = o[rows].clone()
            all_k.append(k)
        elif op[0] == "decode":
            q, k, v = qkv(gen, 1)
            o = rt.decode(q, k, v, torch.device("cpu"))
            rec["ids"] = rt.rt.last_block_ids.clone()
            rec["o"] = o.clone()
        elif op[0] == "verify":
            tq, lossless = op[1], op[2]
            q, k, v = qkv(gen, tq)
            rt.rt.verify_lossless = lossless
            o = rt.verify_tokens(q, k, v, torch.device("cpu"))
            rec["ids"] = rt.rt.last_verify_block_ids.clone()
            rec["o"] = o.clone()
        elif op[0] == "commit":
            rt.commit_verified(op[1])
        rec["valid_len"] = rt.rt.valid_len
        rec["nblocks"] = rt.rt.nblocks_filled
        rec["protected"] = sorted(rt.rt.protected_blocks)
        steps.append(rec)
    return {"name": name, "seed": spec["seed"], "cfg": spec["cfg"], "steps": steps}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", nargs="*")
    args = ap.parse_args()
    torch.set_num_threads(os.cpu_count() or 1)
    for name, spec in CASES.items():
        if args.only and name not in args.only:
            continue
        fx = run_case(name, spec)
        path = os.path.join(HERE, f"{name}.pt")
        torch.save(fx, path)
        print(name, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()
