"""torch.ops.nanokv: the C ABI's hot-path entry points as torch custom operators.

CPU: the operators are registered with their schemas, and their fake
implementations give the output shapes and dtypes under FakeTensorMode (no GPU
needed).  GPU: each operator returns what the runtime's own call returns on the
same state (the same kernel through the same argument struct: bit for bit),
store_kvcache scatters exactly like the reference's rule, and opcheck finds the
schema and the fake kernels consistent with the real ones.
"""
import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

from helpers import pkg, qkv

DEV = "cuda"


def _ops():
    pkg()
    return torch.ops.nanokv


def test_ops_registered_with_fake_shapes():
    ops = _ops()
    for name in ("select", "attend", "prefill", "store_kvcache"):
        assert hasattr(ops, name)
    with FakeTensorMode():
        q = torch.empty(3, 32, 128, dtype=torch.bfloat16, device="cuda")
        reps = torch.empty(8, 512, 4, 128, dtype=torch.bfloat16, device="cuda")
        ids, scores = ops.select(q, reps, 512, torch.empty(9, dtype=torch.int32, device="cuda"), 32)
        assert ids.shape == (32,) and ids.dtype == torch.int64 and scores.dtype == torch.float32
        store = torch.empty(600, 8, 64, 128, dtype=torch.bfloat16, device="cuda")
        sink = torch.empty(8, 64, 128, dtype=torch.bfloat16, device="cuda")
        ring = torch.empty(8, 512, 128, dtype=torch.bfloat16, device="cuda")
        cur = torch.empty(3, 8, 128, dtype=torch.bfloat16, device="cuda")
        for op in (ops.attend, ops.prefill):
            o = op(q, ids, store, store, sink, sink, 64, ring, ring, 0, 512, cur, cur, 0.088)
            assert o.shape == q.shape and o.dtype == torch.bfloat16
    schema = ops.store_kvcache.default._schema  # the two caches are declared mutated
    assert [a.name for a in schema.arguments if a.alias_info and a.alias_info.is_write] == ["k_cache", "v_cache"]


def _runtime(nkv, T=8192, seed=3):
    rt = nkv.M12LayerRuntime(0, nkv.M12Config(max_model_len=16384, device=DEV))
    g = torch.Generator().manual_seed(seed)
    for c in range(T // 4096):
        _, k, v = qkv(g, 4096)
        (rt.prefill_first(None, k.to(DEV), v.to(DEV)) if c == 0 else rt._store_kv(k.to(DEV), v.to(DEV)))
    torch.cuda.synchronize()
    return rt, g


@pytest.mark.gpu
@pytest.mark.parametrize("nq", [1, 4])
def test_select_and_attend_ops_match_runtime(nq):
    ops = _ops()
    nkv = pkg()
    rt, g = _runtime(nkv)
    q, kc, vc = (t.to(DEV) for t in qkv(g, nq))
    kk = rt._budget(32)
    want_ids = rt._select_dev(q, kk).clone()
    want_scores = rt._topk_scores[:kk].clone()
    prot, nprot = rt._protected_dev(rt.nblocks_filled)
    ids, scores = ops.select(q, rt.reps_gpu, rt.nblocks_filled, prot[:nprot], kk)
    torch.cuda.synchronize()
    assert torch.equal(ids, want_ids) and torch.equal(scores, want_scores)
    sink_len, ring_start, ring_len = rt._history_segments()
    want = rt._attend(q, ids, kk, sink_len, ring_start, ring_len, kc, vc)
    got = ops.attend(q, ids, rt._k_store, rt._v_store, rt._sink_k, rt._sink_v, sink_len, rt._ring_k, rt._ring_v,
                     ring_start, ring_len, kc, vc, rt.cfg.scale)
    torch.cuda.synchronize()
    assert torch.equal(got, want)


@pytest.mark.gpu
def test_prefill_op_matches_runtime():
    ops = _ops()
    nkv = pkg()
    rt, g = _runtime(nkv)
    q, kc, vc = (t.to(DEV) for t in qkv(g, 1024))
    ids = rt._select_dev(q[:1], 16).clone()
    sink_len, ring_start, ring_len = rt._history_segments()
    want = rt._attend(q, ids, 16, sink_len, ring_start, ring_len, kc, vc, prefill=True)
    got = ops.prefill(q, ids, rt._k_store, rt._v_store, rt._sink_k, rt._sink_v, sink_len, rt._ring_k, rt._ring_v,
                      ring_start, ring_len, kc, vc, rt.cfg.scale)
    torch.cuda.synchronize()
    assert torch.equal(got, want)


@pytest.mark.gpu
def test_store_kvcache_op():
    ops = _ops()
    g = torch.Generator().manual_seed(4)
    key = torch.randn(37, 8, 128, generator=g).bfloat16().to(DEV)
    val = torch.randn(37, 8, 128, generator=g).bfloat16().to(DEV)
    kc = torch.zeros(100, 1024, dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros_like(kc)
    slots = torch.randperm(100, generator=g)[:37]
    slots[::5] = -1
    ops.store_kvcache(key, val, kc, vc, slots.to(DEV))
    torch.cuda.synchronize()
    want_k, want_v = torch.zeros(100, 1024, dtype=torch.bfloat16), torch.zeros(100, 1024, dtype=torch.bfloat16)
    for i, s in enumerate(slots.tolist()):
        if s != -1:
            want_k[s], want_v[s] = key[i].flatten().cpu(), val[i].flatten().cpu()
    assert torch.equal(kc.cpu(), want_k) and torch.equal(vc.cpu(), want_v)


@pytest.mark.gpu
def test_opcheck():
    ops = _ops()
    nkv = pkg()
    rt, g = _runtime(nkv)
    q, kc, vc = (t.to(DEV) for t in qkv(g, 1))
    prot, nprot = rt._protected_dev(rt.nblocks_filled)
    utils = ("test_schema", "test_faketensor")
    torch.library.opcheck(ops.select, (q, rt.reps_gpu, rt.nblocks_filled, prot[:nprot], 32), test_utils=utils)
    ids, _ = ops.select(q, rt.reps_gpu, rt.nblocks_filled, prot[:nprot], 32)
    sink_len, ring_start, ring_len = rt._history_segments()
    torch.library.opcheck(ops.attend, (q, ids, rt._k_store, rt._v_store, rt._sink_k, rt._sink_v, sink_len, rt._ring_k,
                                       rt._ring_v, ring_start, ring_len, kc, vc, rt.cfg.scale), test_utils=utils)
