"""CUDA path vs the oracle and the reference fixtures (needs a B200).

Tolerances (from the path's contract): selected ids equal except where block
scores tie within 1e-3; attention outputs within max-abs 2e-2 / rel 1e-2 of the
fp32 oracle; representative token indices equal except fp32 near-ties (oracle
decision margin < 1e-5); stored K/V bytes bit-exact.
"""
import math

import pytest
import torch

from helpers import (CASES, OracleReplay, ids_match_modulo_ties, load_golden, orc, pkg, qkv)

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-2, 1e-2
DEV = "cuda"


def _cfg(**kw):
    nkv = pkg()
    base = dict(max_model_len=16384, device=DEV)
    base.update(kw)
    return nkv.M12Config(**base)


def _close(got, want):
    torch.testing.assert_close(got.float().cpu(), want.float().cpu(), atol=ATOL, rtol=RTOL)


# ----------------------------------------------------------------------------
# kernel (1): selection
# ----------------------------------------------------------------------------
@pytest.mark.parametrize("nblocks,k,nq", [(128, 32, 1), (512, 32, 1), (512, 32, 4), (2048, 32, 1),
                                          (3, 2, 1), (40, 1, 1), (512, 48, 1), (300, 64, 2),
                                          (2048, 128, 1)])
def test_select_matches_oracle(nblocks, k, nq):
    nkv = pkg()
    g = torch.Generator().manual_seed(nblocks * 7 + k)
    rt = nkv.M12LayerRuntime(0, _cfg(max_model_len=nblocks * 64))
    reps = torch.randn(8, nblocks, 4, 128, generator=g).bfloat16()
    rt.reps_gpu[:, :nblocks].copy_(reps.to(DEV))
    rt.nblocks_filled = nblocks
    rt.protected_blocks = {0} | set(range(max(1, nblocks - 8), nblocks)) | {nblocks + 5}
    q = torch.randn(nq, 32, 128, generator=g).bfloat16()
    kk = rt._budget(k)
    ids = rt._select_dev(q.to(DEV), kk).cpu()
    want, scores = orc.select_blocks(q, reps, nblocks, rt.protected_blocks, k)
    ok, why = ids_match_modulo_ties(ids, want, scores)
    assert ok, why
    got_scores = rt._topk_scores[:kk].cpu()
    torch.testing.assert_close(got_scores, scores[want], atol=1e-4, rtol=1e-5)


def test_select_ties_all_protected_and_zero_scores():
    nkv = pkg()
    rt = nkv.M12LayerRuntime(0, _cfg())
    # zero representatives: every unprotected block scores 0 -> ascending ids
    rt.nblocks_filled = 8
    rt.reps_gpu[:, :8].zero_()
    q = torch.randn(1, 32, 128).bfloat16().to(DEV)
    rt.protected_blocks = {0, 3}
    ids, info = rt._gpu_select(q[0], budget=4)
    assert ids.tolist() == [1, 2, 4, 5] and info["n_selected"] == 4
    # budget capped by the unprotected count (reference test_m19 :66-74)
    rt.nblocks_filled = 3
    rt.protected_blocks = {0, 20}
    ids, _ = rt._gpu_select(q[0], budget=6)
    assert ids.numel() == 2 and 0 not in ids.tolist()
    # all in-range blocks protected: one id from the protected set (:77-85)
    rt.protected_blocks = {0, 1, 2, 20}
    ids, _ = rt._gpu_select(q[0], budget=6)
    assert ids.numel() == 1 and ids.item() in {0, 1, 2}


def test_select_per_query_matches_oracle():
    nkv = pkg()
    g = torch.Generator().manual_seed(77)
    nblocks = 448
    rt = nkv.M12LayerRuntime(0, _cfg(max_model_len=nblocks * 64))
    reps = torch.randn(8, nblocks, 4, 128, generator=g).bfloat16()
    rt.reps_gpu[:, :nblocks].copy_(reps.to(DEV))
    rt.nblocks_filled = nblocks
    rt.protected_blocks = {0} | set(range(440, 448))
    q = torch.randn(6, 32, 128, generator=g).bfloat16()
    union, allowed = rt._gpu_select_per_query(q.to(DEV), 32)
    want_u, want_a, s = orc.select_per_query(q, reps, nblocks, rt.protected_blocks, 32)
    # per-query rankings are exact here (no near-ties at this seed)
    assert torch.equal(union, want_u)
    assert torch.equal(allowed.cpu(), want_a)


# ----------------------------------------------------------------------------
# kernel (5): store + representatives
# ----------------------------------------------------------------------------
def test_store_division_is_correctly_rounded():
    """The store kernel divides each key by its norm with a reciprocal and one
    fma correction; it must equal the IEEE division bit for bit (the division
    operator on the device), signs of zero included, over positive normal
    divisors and finite quotients (key elements over norms lie in [-1, 1])."""
    nkv = pkg()
    g = torch.Generator().manual_seed(11)
    n = 1 << 20
    a = torch.cat([torch.randn(n, generator=g).bfloat16().float(),                    # key elements
                   torch.randn(n, generator=g) * 2.0 ** torch.randint(-30, 30, (n,), generator=g).float(),
                   torch.tensor([0.0, -0.0, 1e-38, -3e-39, 65504.0, 1.0, -1.0])])
    b = torch.cat([torch.rand(n, generator=g) * 30 + 1e-3,                              # norms
                   torch.rand(n, generator=g).clamp_min(1e-6) * 2.0 ** torch.randint(-30, 30, (n,), generator=g).float(),
                   torch.tensor([1e-12, 1e-12, 1.0, 3.0, 7.0, 1e-12, 1e-12])])
    ad, bd = a.to(DEV), b.to(DEV)
    out = torch.empty_like(ad)
    nkv._lib.call("nkv_selftest_div", torch.cuda.current_stream().cuda_stream, ad.data_ptr(), bd.data_ptr(),
                  out.data_ptr(), ad.numel())
    want = ad / bd
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int32), want.view(torch.int32))


@pytest.mark.parametrize("T,start", [(4096, 0), (333, 5), (64, 0), (2, 1)])
def test_store_and_reps_match_oracle(T, start):
    nkv = pkg()
    g = torch.Generator().manual_seed(T + start)
    rt = nkv.M12LayerRuntime(0, _cfg())
    rt.nblocks_filled = start
    rt.reserve_blocks(start + 80)
    _, k, v = qkv(g, T)
    kd, vd = k.to(DEV), v.to(DEV)
    rt._launch_store(kd, vd, start, sink_write=min(64, T), ring_pos0=0)
    torch.cuda.synchronize()
    nb = -(-T // 64)
    kpad = torch.cat([k, k.new_zeros(nb * 64 - T, 8, 128)]).view(nb, 64, 8, 128)
    vpad = torch.cat([v, v.new_zeros(nb * 64 - T, 8, 128)]).view(nb, 64, 8, 128)
    # block store bit-exact (reference layout view)
    assert torch.equal(rt.k_cpu[start:start + nb].cpu(), kpad)
    assert torch.equal(rt.v_cpu[start:start + nb].cpu(), vpad)
    reps, idx, margin = orc.build_reps(kpad, 4)
    got_idx = rt.rep_index[:, start:start + nb].long().cpu()
    # each pick equals the oracle's while the two follow the same picks; the
    # first difference must be an fp32 near-tie (later picks depend on it)
    differs = got_idx != idx
    first = torch.where(differs.any(-1), differs.float().argmax(-1), torch.full(differs.shape[:-1], -1))
    has = first >= 0
    assert bool((torch.gather(margin, 2, first.clamp_min(0).unsqueeze(-1)).squeeze(-1)[has] < 1e-5).all())
    same = (got_idx == idx).all(-1)
    assert torch.equal(rt.reps_gpu[:, start:start + nb].cpu()[same], reps[same])
    n = min(64, T)
    assert torch.equal(rt.sink_k[:n].cpu(), k[:n])


def test_store_kvcache_twin():
    nkv = pkg()
    lib = nkv._lib
    N, H = 37, 8
    key = torch.randn(N, H, 128).bfloat16().to(DEV)
    val = torch.randn(N, H, 128).bfloat16().to(DEV)
    kc = torch.zeros(100, H * 128, dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros_like(kc)
    slots = torch.randperm(100)[:N]
    slots[::5] = -1
    sd = slots.to(DEV)
    lib.call("nkv_store_kvcache", torch.cuda.current_stream().cuda_stream, key.data_ptr(),
             key.stride(0), val.data_ptr(), val.stride(0), kc.data_ptr(), vc.data_ptr(),
             sd.data_ptr(), N, H * 128)
    want_k = torch.zeros(100, H * 128, dtype=torch.bfloat16)
    want_v = torch.zeros_like(want_k)
    for i, s in enumerate(slots.tolist()):
        if s != -1:
            want_k[s] = key[i].flatten().cpu()
            want_v[s] = val[i].flatten().cpu()
    assert torch.equal(kc.cpu(), want_k) and torch.equal(vc.cpu(), want_v)


# ----------------------------------------------------------------------------
# kernels (1)+(2)+(5) through the runtime, against the oracle and the fixtures
# ----------------------------------------------------------------------------
def _runtime_for(name, **extra):
    nkv = pkg()
    cfg = dict(CASES[name]["cfg"])
    cfg.setdefault("max_model_len", max(16384, CASES[name].get("max_model_len", 0)))
    cfg.update(extra)
    return nkv.M12LayerRuntime(0, _cfg(**cfg))


def _replay(name, rt, skip_chunks=False):
    """Drive the CUDA runtime and the oracle in lock step.

    The runtime selects first; its ids must equal the oracle's own selection
    modulo score ties (1e-3), and the oracle then attends the runtime's blocks
    so that outputs compare like for like.  Outputs are also compared with the
    reference fixture whenever the runtime picked exactly the reference's ids."""
    spec = CASES[name]
    golden = load_golden(name)
    cfg = dict(spec["cfg"])
    cfg.pop("verify_union_blocks", None)
    layer = orc.OracleLayer(orc.OracleConfig(**cfg))
    gen = torch.Generator().manual_seed(spec["seed"])
    for step, op in enumerate(spec["script"]):
        g = golden["steps"][step]
        out = {"op": op, "golden": g}
        if op[0] in ("first", "chunk", "store", "decode", "verify"):
            q, k, v = qkv(gen, 1 if op[0] == "decode" else op[1])
            qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
        if op[0] == "first":
            rt.prefill_first(qd, kd, vd)
            layer.store(k, v)
            layer.prefill_len = rt.prefill_len
        elif op[0] == "store":
            rt._store_kv(kd, vd)
            layer.store(k, v)
        elif op[0] == "chunk":
            if skip_chunks:
                rt._store_kv(kd, vd)
                layer.store(k, v)
            else:
                out["o"] = rt.prefill_chunk(qd, kd, vd, DEV)
                out["ids"] = rt.last_prefill_block_ids.cpu()
                layer.force_ids = out["ids"]
                out["want"] = layer.prefill_chunk(q, k, v)
        elif op[0] == "decode":
            out["o"] = rt.decode(qd, kd, vd, DEV)
            out["ids"] = rt.last_block_ids.cpu()
            layer.force_ids = out["ids"]
            out["want"] = layer.decode(q, k, v)
        elif op[0] == "verify":
            rt.verify_lossless = op[2]
            out["o"] = rt.verify_tokens(qd, kd, vd, DEV)
            out["ids"] = rt.last_verify_block_ids.cpu()
            if not op[2]:
                layer.force_ids = out["ids"]
            out["want"] = layer.verify(q, k, v, lossless=op[2])
        elif op[0] == "commit":
            rt.commit_verified(op[1])
            layer.commit(op[1])
        out["own_ids"], out["scores"] = layer.own_ids, layer.last_scores
        assert rt.valid_len == layer.valid_len == g["valid_len"], (step, op)
        assert rt.nblocks_filled == layer.nblocks == g["nblocks"], (step, op)
        assert sorted(rt.protected_blocks) == sorted(layer.protected) == g["protected"], (step, op)
        yield out


def _check_step(s):
    g = s["golden"]
    op = s["op"]
    if "ids" in s:
        if op[0] == "verify" and op[2]:
            assert torch.equal(s["ids"], s["own_ids"]), op
        else:
            ok, why = ids_match_modulo_ties(s["ids"], s["own_ids"], s["scores"])
            assert ok, f"{op}: {why}"
    if "o" in s:
        _close(s["o"], s["want"])
        if "ids" in g and torch.equal(s["ids"], g["ids"]):
            got = s["o"][g["rows"]] if "rows" in g else s["o"]
            _close(got, g["o"])


@pytest.mark.parametrize("name", ["decode_c1", "short", "relative", "relative_union", "dynamic", "qwindow",
                                  "verify28k"])
def test_runtime_decode_matches_oracle_and_reference(name):
    rt = _runtime_for(name)
    for s in _replay(name, rt):
        _check_step(s)


@pytest.mark.parametrize("name", ["chunks", "segments", "quant"])
def test_runtime_decode_after_chunks(name):
    """Later prefill chunks are stored through the store kernel; decode and
    verify steps are checked (prefill attention has its own test)."""
    rt = _runtime_for(name)
    for s in _replay(name, rt, skip_chunks=True):
        if s["op"][0] in ("decode", "verify"):
            _check_step(s)


@pytest.mark.parametrize("name", ["chunks", "segments", "quant"])
def test_runtime_prefill_chunks(name):
    """Later-chunk segmented prefill attention (kernel 4) + everything after it."""
    rt = _runtime_for(name)
    for s in _replay(name, rt):
        _check_step(s)


def test_decode_32k_matches_oracle():
    """Headline geometry: 32K history, Top-32, sink 64, recent 512."""
    nkv = pkg()
    g = torch.Generator().manual_seed(32768)
    layer = orc.OracleLayer(orc.OracleConfig())
    rt = nkv.M12LayerRuntime(0, _cfg(max_model_len=40960))
    for _ in range(8):
        q, k, v = qkv(g, 4096)
        layer.store(k, v)
        layer.prefill_len = max(layer.prefill_len, 1)
        rt._store_kv(k.to(DEV), v.to(DEV))
    layer.valid_len = rt.valid_len
    assert rt.nblocks_filled == 512 and sorted(rt.protected_blocks) == sorted(layer.protected)
    for _ in range(3):
        q, k, v = qkv(g, 1)
        got = rt.decode(q.to(DEV), k.to(DEV), v.to(DEV), DEV)
        layer.force_ids = rt.last_block_ids
        want = layer.decode(q, k, v)
        ok, why = ids_match_modulo_ties(rt.last_block_ids, layer.own_ids, layer.last_scores)
        assert ok, why
        _close(got, want)


def test_decode_128k_matches_oracle():
    """Long-context geometry (BASELINE config 5's operator): 131072-token
    history (2048 blocks, Top-32 of 2039 unprotected), sink 64, recent 512."""
    nkv = pkg()
    g = torch.Generator().manual_seed(131072)
    layer = orc.OracleLayer(orc.OracleConfig())
    rt = nkv.M12LayerRuntime(0, _cfg(max_model_len=131072 + 4096))
    for _ in range(32):
        q, k, v = qkv(g, 4096)
        layer.store(k, v)
        layer.prefill_len = max(layer.prefill_len, 1)
        rt._store_kv(k.to(DEV), v.to(DEV))
    layer.valid_len = rt.valid_len
    assert rt.nblocks_filled == 2048 and sorted(rt.protected_blocks) == sorted(layer.protected)
    for _ in range(3):
        q, k, v = qkv(g, 1)
        got = rt.decode(q.to(DEV), k.to(DEV), v.to(DEV), DEV)
        layer.force_ids = rt.last_block_ids
        want = layer.decode(q, k, v)
        ok, why = ids_match_modulo_ties(rt.last_block_ids, layer.own_ids, layer.last_scores)
        assert ok, why
        _close(got, want)


def _rows_attention(q, kp, vp, cf, rows, scale):
    """fp32 oracle attention of the query rows `rows` of a chunk over the packed keys:
    row t sees history keys [0, cf) and chunk keys [cf, cf + t]."""
    out = []
    for t in rows:
        n = cf + t + 1
        out.append(orc.attention(q[t:t + 1], kp[:n], vp[:n], scale)[0])
    return torch.stack(out)


def test_prefill_c4_full_size():
    """Segmented prefill operator at its benchmark geometry: a 4096-token chunk
    at positions 28672-32767 after 7 stored chunks (Top-32 of 448 blocks, sink
    64, recent 512, causal chunk), 32 Q / 8 KV heads.  Selection vs the oracle
    (modulo 1e-3 ties); kernel (4)'s output on 96 rows (first, last, block
    edges, random) vs the fp32 oracle over the same packed keys."""
    nkv = pkg()
    g = torch.Generator().manual_seed(28672)
    layer = orc.OracleLayer(orc.OracleConfig())
    rt = nkv.M12LayerRuntime(0, _cfg(max_model_len=36864))
    for c in range(7):
        _, k, v = qkv(g, 4096)
        if c == 0:
            rt.prefill_first(None, k.to(DEV), v.to(DEV))
        else:
            rt._store_kv(k.to(DEV), v.to(DEV))
        layer.store(k, v)
        layer.prefill_len = rt.prefill_len
    layer.valid_len = rt.valid_len
    assert rt.nblocks_filled == layer.nblocks == 448
    q, k, v = qkv(g, 4096)
    got = rt.prefill_chunk(q.to(DEV), k.to(DEV), v.to(DEV), DEV).cpu()
    ids = rt.last_prefill_block_ids.cpu()
    cfg = layer.cfg
    own = layer._select(orc.query_summaries(q, cfg.prefill_query_segments), cfg.prefill_top_k_blocks)
    ok, why = ids_match_modulo_ties(ids, own, layer.last_scores)
    assert ok, why
    kp, vp, cf = layer._history_pack(ids, k, v)
    assert cf == 32 * 64 + 64 + 512  # selected + sink + recent (no overlap at 28672)
    gen = torch.Generator().manual_seed(1)
    rows = sorted(set([0, 1, 63, 64, 127, 128, 4031, 4094, 4095] +
                      torch.randint(0, 4096, (87,), generator=gen).tolist()))
    want = _rows_attention(q, kp, vp, cf, rows, cfg.scale)
    _close(got[rows], want)


def test_first_chunk_causal_matches_oracle():
    """First-chunk dense causal attention through kernel (4) (no history)."""
    nkv = pkg()
    g = torch.Generator().manual_seed(7)
    rt = nkv.M12LayerRuntime(0, _cfg())
    q, k, v = qkv(g, 1000)
    got = rt.first_chunk_attention(q.to(DEV), k.to(DEV), v.to(DEV)).cpu()
    want = orc.attention(q, k, v, rt.cfg.scale, causal_from=0)
    _close(got, want)


@pytest.mark.parametrize("scheme", ["reference", "token"])
@pytest.mark.parametrize("residency", ["hbm", "host"])
def test_int8_history_decode(scheme, residency):
    """int8 history (reference scheme / per-token scheme), in HBM or offloaded
    to mapped pinned host memory, against the oracle's dequantised attention."""
    nkv = pkg()
    g = torch.Generator().manual_seed(99)
    rt = nkv.M12LayerRuntime(0, _cfg(quant_history=True, quant_scheme=scheme,
                                     kv_residency=residency, top_k_blocks=16))
    _, k, v = qkv(g, 4096)
    rt.prefill_first(k.new_zeros(1), k.to(DEV), v.to(DEV))
    torch.cuda.synchronize()
    # oracle with the same scheme
    layer = orc.OracleLayer(orc.OracleConfig(top_k_blocks=16, quant_history=True))
    kb, vb = k.view(64, 64, 8, 128), v.view(64, 64, 8, 128)
    if scheme == "reference":
        layer.store(k, v)
        assert torch.equal(rt.k_scale.cpu(), layer.k_scale)
        kq = orc.quant_k(kb, layer.k_scale)
        assert torch.equal(rt.k_cpu[:64].cpu(), kq)
    else:
        layer.cfg.quant_history = False
        layer.store(k, v)
        # per-token dequantised history replaces the bf16 blocks in the oracle
        kq, ks = orc.quant_token_head(k)
        vq, vs = orc.quant_token_head(v)
        kdq = (kq.float() * ks.float()[..., None]).bfloat16().view(64, 64, 8, 128)
        vdq = (vq.float() * vs.float()[..., None]).bfloat16().view(64, 64, 8, 128)
        layer.k_hist, layer.v_hist = list(kdq), list(vdq)
        assert torch.equal(rt.k_cpu[:64].cpu(), kq.view(64, 64, 8, 128))
    for _ in range(2):
        q, kk, vv = qkv(g, 1)
        got = rt.decode(q.to(DEV), kk.to(DEV), vv.to(DEV), DEV)
        layer.force_ids = rt.last_block_ids
        want = layer.decode(q, kk, vv)
        ok, why = ids_match_modulo_ties(rt.last_block_ids, layer.own_ids, layer.last_scores)
        assert ok, why
        _close(got, want)


@pytest.mark.parametrize("quant,scheme,residency", [(True, "reference", "hbm"), (True, "token", "host"),
                                                   (False, "reference", "host")])
def test_prefill_chunk_over_staged_history(quant, scheme, residency):
    """A later prefill chunk over int8 or host-resident history: the selected
    blocks staged in device bf16 (nkv_prefill_gather) and attended on the
    tensor-core kernel, against the oracle's dequantised attention and against
    the in-place form (the selected blocks read where they lie)."""
    nkv = pkg()
    outs = []
    for staged in (True, False):
        g = torch.Generator().manual_seed(77)
        rt = nkv.M12LayerRuntime(0, _cfg(quant_history=quant, quant_scheme=scheme, kv_residency=residency,
                                         top_k_blocks=16))
        rt.prefill_gather = staged
        _, k, v = qkv(g, 4096)
        rt.prefill_first(k.new_zeros(1), k.to(DEV), v.to(DEV))
        layer = orc.OracleLayer(orc.OracleConfig(top_k_blocks=16, quant_history=quant and scheme == "reference"))
        layer.store(k, v)
        if quant and scheme == "token":  # the per-token dequantised history replaces the oracle's blocks
            kq, ks = orc.quant_token_head(k)
            vq, vs = orc.quant_token_head(v)
            layer.k_hist = list((kq.float() * ks.float()[..., None]).bfloat16().view(64, 64, 8, 128))
            layer.v_hist = list((vq.float() * vs.float()[..., None]).bfloat16().view(64, 64, 8, 128))
        layer.prefill_len = rt.prefill_len
        q, kc, vc = qkv(g, 1024)
        got = rt.prefill_chunk(q.to(DEV), kc.to(DEV), vc.to(DEV), DEV)
        layer.force_ids = rt.last_prefill_block_ids.cpu()
        want = layer.prefill_chunk(q, kc, vc)
        assert rt.last_prefill_block_ids.numel() == 16
        _close(got, want)
        outs.append((rt.last_prefill_block_ids.cpu(), got.float().cpu()))
    assert torch.equal(outs[0][0], outs[1][0])
    torch.testing.assert_close(outs[0][1], outs[1][1], atol=ATOL, rtol=RTOL)


def test_offload_bf16_host_history():
    nkv = pkg()
    g = torch.Generator().manual_seed(5)
    rt = nkv.M12LayerRuntime(0, _cfg(kv_residency="host"))
    layer = orc.OracleLayer(orc.OracleConfig())
    _, k, v = qkv(g, 8192)
    rt.prefill_first(k.new_zeros(1), k.to(DEV), v.to(DEV))
    layer.store(k, v)
    layer.prefill_len = rt.prefill_len
    assert not rt.k_cpu.is_cuda
    for _ in range(2):
        q, kk, vv = qkv(g, 1)
        got = rt.decode(q.to(DEV), kk.to(DEV), vv.to(DEV), DEV)
        layer.force_ids = rt.last_block_ids
        want = layer.decode(q, kk, vv)
        ok, why = ids_match_modulo_ties(rt.last_block_ids, layer.own_ids, layer.last_scores)
        assert ok, why
        _close(got, want)


def test_reset_reuses_buffers():
    """reference tests/test_m16_dynamic_topk.py:65-85 at the production geometry."""
    nkv = pkg()
    rt = nkv.M12LayerRuntime(0, _cfg(top_k_blocks=2, max_model_len=4096))
    kv = torch.randn(256, 8, 128).bfloat16().to(DEV)
    rt.prefill_first(kv, kv, kv)
    buf = rt.k_cpu
    assert rt.valid_len == rt.prefill_len == 256 and rt.nblocks_filled == 4
    rt.reset()
    assert rt.k_cpu is buf
    assert rt.valid_len == rt.prefill_len == rt.nblocks_filled == 0 and not rt.protected_blocks
    rt.prefill_first(kv, kv, kv)
    assert rt.valid_len == 256 and rt.nblocks_filled == 4


def test_reset_then_reuse_matches_fresh_runtime():
    """A runtime that served one sequence, was reset and then serves another
    gives the same ids and bitwise the same outputs as a fresh runtime
    (the reference's reset between requests, m12_runtime.py:322-349)."""
    nkv = pkg()
    g = torch.Generator().manual_seed(321)
    _, ka, va = qkv(g, 4096)
    _, kb, vb = qkv(g, 8192 + 77)
    steps = [qkv(g, 1) for _ in range(3)]
    used = nkv.M12LayerRuntime(0, _cfg())
    used.prefill_first(None, ka.to(DEV), va.to(DEV))
    for q, k, v in steps:
        used.decode(q.to(DEV), k.to(DEV), v.to(DEV), DEV)
    used.reset()
    fresh = nkv.M12LayerRuntime(0, _cfg())
    for rt in (used, fresh):
        rt.prefill_first(None, kb[:4096].to(DEV), vb[:4096].to(DEV))
        rt._store_kv(kb[4096:].to(DEV), vb[4096:].to(DEV))
    for q, k, v in steps:
        a = used.decode(q.to(DEV), k.to(DEV), v.to(DEV), DEV)
        b = fresh.decode(q.to(DEV), k.to(DEV), v.to(DEV), DEV)
        assert torch.equal(used.last_block_ids, fresh.last_block_ids)
        assert torch.equal(a, b)
    assert torch.equal(used.recent_k, fresh.recent_k)


def test_unsupported_geometry_fails_loudly():
    nkv = pkg()
    with pytest.raises(ValueError):
        nkv.M12LayerRuntime(0, _cfg(head_dim=64, scale=0.125))
    with pytest.raises(ValueError):
        nkv.M12LayerRuntime(0, _cfg(dtype=torch.float32))
