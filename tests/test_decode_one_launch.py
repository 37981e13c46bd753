"""The one-launch decode step (scoring + selection + attention in one
cooperative cluster launch) against the oracle's selection and against the
two-launch form (scoring grid + ranked attention), which the oracle tests pin
(needs a B200).

The one-launch step scores on the tensor cores (fp32 sums of exact bf16
products in the tensor core's order), so its ids equal the oracle's except
where block scores tie within 1e-3, and its top-k scores match the oracle's
within 1e-4.  Where both forms pick the same ids, their outputs agree to bf16
rounding (max-abs 1e-2).  Several steps in a row exercise the per-launch
epoch tags; a lossless verify between steps shares the select workspace.
"""
import pytest
import torch

from helpers import ids_match_modulo_ties, orc, pkg

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _tokens(g, t, hq, hkv):
    q = torch.randn(t, hq, 128, generator=g).bfloat16()
    k = torch.randn(t, hkv, 128, generator=g).bfloat16()
    v = torch.randn(t, hkv, 128, generator=g).bfloat16()
    return q, k, v


def _runtime(hist, hq, hkv, seed):
    nkv = pkg()
    cfg = nkv.M12Config(max_model_len=hist + 4096, num_heads=hq, num_kv_heads=hkv, device=DEV)
    rt = nkv.M12LayerRuntime(0, cfg)
    g = torch.Generator().manual_seed(seed)
    left = hist
    while left > 0:
        t = min(4096, left)
        _, k, v = _tokens(g, t, hq, hkv)
        rt._store_kv(k.to(DEV), v.to(DEV))
        left -= t
    return rt


# `one`: whether the step fits one launch (with 4 KV heads the attention does
# not use thread-block clusters, so the step runs as two launches)
@pytest.mark.parametrize("hist,hq,hkv,steps,verify,one", [
    (100, 32, 8, 2, False, True),      # 2 blocks, both protected: k = 1
    (700, 32, 8, 3, False, True),      # 11 blocks: k < 32
    (8192, 32, 4, 3, False, False),    # G = 8
    (8192, 16, 8, 2, False, True),     # G = 2
    (8192, 8, 8, 2, False, True),      # G = 1
    (32768, 32, 8, 4, True, True),     # headline geometry, verify in between
    (131072, 32, 8, 2, False, True),   # 2048 blocks: 32 blocks scored per CTA
])
def test_one_launch_matches_oracle(hist, hq, hkv, steps, verify, one, monkeypatch):
    lib = pkg()._lib.load()
    seed = hist * 31 + hq
    rt1 = _runtime(hist, hq, hkv, seed)
    rt2 = _runtime(hist, hq, hkv, seed)
    g = torch.Generator().manual_seed(seed + 1)
    for step in range(steps):
        qc, kc, vc = _tokens(g, 1, hq, hkv)
        q, k, v = qc.to(DEV), kc.to(DEV), vc.to(DEV)
        nb = rt1.nblocks_filled
        want, scores = orc.select_blocks(qc, rt1.reps_gpu[:, :nb].cpu(), nb, rt1.protected_blocks,
                                         rt1.cfg.decode_top_k_blocks or rt1.cfg.top_k_blocks)
        monkeypatch.setenv("NKV_DECODE_ONE", "1")
        lib.nkv_reload_env()
        o1 = rt1.decode(q, k, v, DEV)
        form1 = lib.nkv_decode_last_form()
        ids1, sc1 = rt1.last_block_ids.cpu(), rt1._topk_scores[:len(rt1.last_block_ids)].cpu()
        monkeypatch.setenv("NKV_DECODE_ONE", "0")
        lib.nkv_reload_env()
        o2 = rt2.decode(q, k, v, DEV)
        form2 = lib.nkv_decode_last_form()
        ids2, sc2 = rt2.last_block_ids.cpu(), rt2._topk_scores[:len(rt2.last_block_ids)].cpu()
        assert form1 == (1 if one else 2) and form2 == 2, (form1, form2)
        ok, why = ids_match_modulo_ties(ids1, want, scores)
        assert ok, (step, why)
        torch.testing.assert_close(sc1, scores[ids1], atol=1e-4, rtol=1e-5)
        ok, why = ids_match_modulo_ties(ids2, want, scores)
        assert ok, (step, why)
        if torch.equal(ids1, ids2):
            torch.testing.assert_close(o1.float().cpu(), o2.float().cpu(), atol=1e-2, rtol=1e-2)
        if verify and step == 1:
            qv, kv, vv = (x.to(DEV) for x in _tokens(g, 6, hq, hkv))
            for rt in (rt1, rt2):
                rt.verify_lossless = True
                rt.verify_tokens(qv, kv, vv, DEV)
                rt.rollback_verified()
    monkeypatch.delenv("NKV_DECODE_ONE", raising=False)
    lib.nkv_reload_env()
    torch.cuda.synchronize()
    for rt in (rt1, rt2):  # no bounded wait timed out, no bad block id
        assert rt._att_ws[:4].view(torch.int32).item() == 0
