"""The segmented-prefill operator seam (needs a B200): the reference's
SegmentedPrefillAdapter contract (prepare(q, stage_k, stage_v, sink, recent,
current) -> attend) on this package's prefill kernel, against the fp32
oracle's attention over the packed segments [selected | sink | recent |
current] with the current chunk causal (reference
segmented_prefill_adapter.py:95-147, flash_attn_func causal=True for Sq < Sk).
"""
import pytest
import torch

from helpers import orc, pkg

pytestmark = pytest.mark.gpu
DEV = "cuda"
ATOL, RTOL = 2e-2, 1e-2


def _seg(g, n, hkv=8):
    return (torch.randn(n, hkv, 128, generator=g).bfloat16().to(DEV),
            torch.randn(n, hkv, 128, generator=g).bfloat16().to(DEV))


@pytest.mark.parametrize("tq,nsel_blocks,sink,recent,pinned", [
    (512, 32, 64, 512, True), (6, 32, 64, 512, True), (256, 0, 64, 100, False), (96, 4, 0, 0, False)])
def test_segmented_adapter_matches_oracle(tq, nsel_blocks, sink, recent, pinned):
    nkv = pkg()
    from importlib import import_module
    S = import_module(nkv.__name__ + ".segmented_prefill")
    g = torch.Generator().manual_seed(tq + nsel_blocks)
    ad = S.SegmentedPrefillAdapter("b200")
    q = torch.randn(tq, 32, 128, generator=g).bfloat16().to(DEV)
    sk = torch.randn(nsel_blocks * 64, 8, 128, generator=g).bfloat16()
    sv = torch.randn(nsel_blocks * 64, 8, 128, generator=g).bfloat16()
    if pinned:
        sk, sv = sk.pin_memory(), sv.pin_memory()
    else:
        sk, sv = sk.to(DEV), sv.to(DEV)
    snk, rec, cur = _seg(g, sink), _seg(g, recent), _seg(g, tq)
    inv = ad.prepare(q, sk, sv, snk, rec, cur)
    o = ad.attend(inv)
    torch.cuda.synchronize()
    ad.check()
    kp = torch.cat([sk.to(DEV), snk[0], rec[0], cur[0]]).float().cpu()
    vp = torch.cat([sv.to(DEV), snk[1], rec[1], cur[1]]).float().cpu()
    want = orc.attention(q.float().cpu(), kp, vp, 128 ** -0.5, causal_from=kp.shape[0] - tq)
    torch.testing.assert_close(o.float().cpu(), want.float(), atol=ATOL, rtol=RTOL)
    assert ad.stats()["direct_calls"] == 1


def test_segmented_adapter_rejects_bad_inputs():
    nkv = pkg()
    from importlib import import_module
    S = import_module(nkv.__name__ + ".segmented_prefill")
    ad = S.SegmentedPrefillAdapter("b200")
    q = torch.zeros(8, 32, 128, dtype=torch.bfloat16, device=DEV)
    seg = (torch.zeros(8, 8, 128, dtype=torch.bfloat16, device=DEV),) * 2
    with pytest.raises(ValueError):  # unpinned host staging
        ad.prepare(q, torch.zeros(64, 8, 128, dtype=torch.bfloat16), torch.zeros(64, 8, 128, dtype=torch.bfloat16),
                   seg, seg, seg)
    with pytest.raises(ValueError):  # current chunk length != queries
        ad.prepare(q, seg[0][:0], seg[1][:0], seg, seg, (seg[0][:4], seg[1][:4]))
    with pytest.raises(ValueError):
        S.SegmentedPrefillAdapter("operator")


def test_runtime_prefill_chunks_through_the_adapter():
    """M12Config.prefill_adapter routes prefill_chunk's attention through the
    seam; outputs match the runtime's own path within the parity tolerance and
    the stored history is the same."""
    nkv = pkg()
    from importlib import import_module
    S = import_module(nkv.__name__ + ".segmented_prefill")
    g = torch.Generator().manual_seed(77)
    ad = S.SegmentedPrefillAdapter("b200")
    plain = nkv.M12LayerRuntime(0, nkv.M12Config(max_model_len=16384, device=DEV))
    seam = nkv.M12LayerRuntime(0, nkv.M12Config(max_model_len=16384, device=DEV, prefill_adapter=ad))
    for c in range(3):
        q = torch.randn(1024, 32, 128, generator=g).bfloat16().to(DEV)
        k, v = _seg(g, 1024)
        if c == 0:
            for rt in (plain, seam):
                rt.prefill_first(q, k, v)
            continue
        o1 = plain.prefill_chunk(q, k, v, DEV)
        o2 = seam.prefill_chunk(q, k, v, DEV)
        assert torch.equal(plain.last_block_ids, seam.last_block_ids)
        torch.testing.assert_close(o2.float(), o1.float(), atol=ATOL, rtol=RTOL)
    torch.cuda.synchronize()
    assert ad.stats()["direct_calls"] == 2
    assert torch.equal(plain.recent_k, seam.recent_k)
