"""DecodeGraph: decode steps replayed from a CUDA graph against the eager
decode of an identical stack (needs a B200).

The graph runs the same kernels on the same inputs, with the recent window's
head read from the device instead of the arguments, so its outputs, selected
ids, recent windows and host state must equal the eager path's exactly.
Eager calls between replays move the window on the host; the next replay
must follow it.  A history change after the recording makes replay raise.
"""
import pytest
import torch

from helpers import pkg

pytestmark = pytest.mark.gpu
DEV = "cuda"
HQ, HKV, D = 32, 8, 128


def _stack(n_layers, hist, seed, **cfg):
    nkv = pkg()
    g = torch.Generator().manual_seed(seed)
    layers = []
    for li in range(n_layers):
        rt = nkv.M12LayerRuntime(li, nkv.M12Config(max_model_len=hist + 1024, device=DEV, **cfg))
        k = torch.randn(hist, HKV, D, generator=g).bfloat16().to(DEV)
        v = torch.randn(hist, HKV, D, generator=g).bfloat16().to(DEV)
        rt.prefill_first(None, k, v)
        layers.append(rt)
    return layers


def _token(g, n_layers):
    return [(torch.randn(1, HQ, D, generator=g).bfloat16(), torch.randn(1, HKV, D, generator=g).bfloat16(),
             torch.randn(1, HKV, D, generator=g).bfloat16()) for _ in range(n_layers)]


def _same_state(a, b):
    assert a.valid_len == b.valid_len and a._ring_head == b._ring_head
    assert torch.equal(a.recent_k, b.recent_k) and torch.equal(a.recent_v, b.recent_v)
    assert a.last_block_ids.tolist() == b.last_block_ids.tolist()


@pytest.mark.parametrize("hist,top_k,recent,extra", [
    (2048, 8, 512, {}),
    (8192, 32, 512, {}),
    (3000, 16, 64, {}),
    # int8 history (per-token scales) in mapped pinned host memory: the offload decode
    (4096, 32, 512, {"quant_history": True, "quant_scheme": "token", "kv_residency": "host"}),
])
def test_graph_replay_matches_eager(hist, top_k, recent, extra):
    nkv = pkg()
    L = 3
    ga = _stack(L, hist, seed=hist + top_k, top_k_blocks=top_k, recent_tokens=recent, **extra)
    eb = _stack(L, hist, seed=hist + top_k, top_k_blocks=top_k, recent_tokens=recent, **extra)
    g = torch.Generator().manual_seed(7)
    # one eager token on both stacks (sets up workspaces outside the capture)
    for (q, k, v), a, b in zip(_token(g, L), ga, eb):
        oa = a.decode(q.to(DEV), k.to(DEV), v.to(DEV), DEV)
        ob = b.decode(q.to(DEV), k.to(DEV), v.to(DEV), DEV)
        assert torch.equal(oa, ob)
    bufs = [(torch.empty(1, HQ, D, dtype=torch.bfloat16, device=DEV),
             torch.empty(1, HKV, D, dtype=torch.bfloat16, device=DEV),
             torch.empty(1, HKV, D, dtype=torch.bfloat16, device=DEV)) for _ in range(L)]
    dg = nkv.DecodeGraph(ga, bufs)
    for rt in ga:  # recording leaves the host state as it was
        assert rt.valid_len == hist + 1
    for step in range(6):
        toks = _token(g, L)
        if step == 3:
            # an eager token between replays moves the window on the host
            for (q, k, v), a, b in zip(toks, ga, eb):
                oa = a.decode(q.to(DEV), k.to(DEV), v.to(DEV), DEV)
                ob = b.decode(q.to(DEV), k.to(DEV), v.to(DEV), DEV)
                assert torch.equal(oa, ob)
            continue
        for (q, k, v), (bq, bk, bv) in zip(toks, bufs):
            bq.copy_(q)
            bk.copy_(k)
            bv.copy_(v)
        out = dg.replay()
        want = [b.decode(q.to(DEV), k.to(DEV), v.to(DEV), DEV) for (q, k, v), b in zip(toks, eb)]
        torch.cuda.synchronize()
        for li in range(L):
            assert torch.equal(out[li], want[li]), f"step {step} layer {li}"
            assert torch.equal(dg.outputs[li], want[li])
            assert dg.outputs[li].data_ptr() == dg.out[li].data_ptr()  # written in place, no stack copy
            _same_state(ga[li], eb[li])


def test_graph_rejects_partial_window_and_changed_history():
    nkv = pkg()
    short = _stack(1, 256, seed=3, top_k_blocks=2)  # valid_len 257 < recent_tokens - 1
    g = torch.Generator().manual_seed(1)
    q, k, v = _token(g, 1)[0]
    short[0].decode(q.to(DEV), k.to(DEV), v.to(DEV), DEV)
    bufs = [(q.to(DEV), k.to(DEV), v.to(DEV))]
    with pytest.raises(AssertionError):
        nkv.DecodeGraph(short, bufs)
    full = _stack(1, 2048, seed=4, top_k_blocks=8)
    full[0].decode(q.to(DEV), k.to(DEV), v.to(DEV), DEV)
    dg = nkv.DecodeGraph(full, bufs)
    dg.replay()
    full[0].reset()  # the history is gone: the recording no longer applies
    with pytest.raises(RuntimeError):
        dg.replay()
    torch.cuda.synchronize()
