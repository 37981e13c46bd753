"""Full-model configs (needs a B200): parity of the sparse path inside the
model, greedy tokens, and the CUDA-graph decode loop.

BASELINE configs 2 and 3: a random-init Qwen3-4B-architecture model (36 layers,
hidden 2560, 32/8 heads, head_dim 128, SwiGLU 9728, YaRN factor 4, vocab
151936), a 32768-token prompt of seeded uniform random token ids prefilled in
4096-token chunks through the sparse path (64-token blocks, r=4, Top-32, sink
64, recent 512), then 128 greedy decode steps; config 3 keeps the history int8
(the reference's scheme) in pinned host memory.

Arm A is this package (``Qwen3SparseModel`` with the CUDA ``M12LayerRuntime``).
Every attention call of arm A -- 36 layers x (first chunk, 7 later chunks, 128
decode steps) -- is repeated by a shadow oracle layer (``oracle.m12_oracle`` in
fp32 on the GPU) fed the same q/k/v: arm A's selected blocks must equal the
oracle's selection from arm A's routing query and representatives except where
block scores tie within 1e-3, and arm A's output must be within the contract's
max-abs 2e-2 / rel 1e-2 of the oracle's attention over those blocks, with a
relative error norm below 5e-3 (bf16 resolution).

Arm B is the same model (same weights and dense kernels) with the oracle as
every layer's runtime, fed arm A's tokens and blocks.  A random-init model of
this depth is chaotic: bf16-level differences in the attention outputs (arm A
vs the oracle differ by ~1.7e-3 relative per call, the rounding of bf16) grow
to ~0.04 mean / <0.3 max absolute logit differences at the LM head, and the
random model's top-2 logits are often closer than that.  So the token check is:
wherever arm A's and arm B's greedy tokens differ, arm B's logits for the two
tokens must lie within TIE_BAND (a near-tie); everywhere else they are equal.

The decode loop replayed from one CUDA graph (``DecodeLoop``) must produce the
same tokens, bit for bit, as eager decode steps of an identical model.
"""
import gc

import pytest
import torch

from helpers import ids_match_modulo_ties, orc, pkg

pytestmark = pytest.mark.gpu
DEV = "cuda"
PROMPT, STEPS, CHUNK = 32768, 128, 4096
ATOL, RTOL, REL_NORM = 2e-2, 1e-2, 5e-3
TIE_BAND = 0.3  # logit units; the measured inter-arm logit difference stays below 0.27


class ForcedOracle:
    """Oracle runtime that attends arm A's recorded blocks."""

    def __init__(self, base, prefill_ids, decode_ids):
        self.base = base
        self.prefill_ids = list(prefill_ids)
        self.decode_ids = list(decode_ids)

    @property
    def prefill_len(self):
        return self.base.prefill_len

    @property
    def last_block_ids(self):
        return self.base.last_block_ids

    def first_chunk_attention(self, q, k, v):
        return self.base.first_chunk_attention(q, k, v)

    def prefill_first(self, q, k, v):
        return self.base.prefill_first(q, k, v)

    def prefill_chunk(self, q, k, v, device):
        self.base.layer.force_ids = self.prefill_ids.pop(0)
        return self.base.prefill_chunk(q, k, v, device)

    def decode(self, q, k, v, device):
        self.base.layer.force_ids = self.decode_ids.pop(0)
        return self.base.decode(q, k, v, device)


def _shadowed_runtime(nkv):
    """M12LayerRuntime whose every call is repeated by an oracle layer on the
    same inputs; selection and output discrepancies are collected."""

    class Shadowed(nkv.M12LayerRuntime):
        def setup(self, oracle_cfg, failures, ids_log):
            self.shadow = orc.OracleLayer(oracle_cfg)
            self.failures, self.ids_log = failures, ids_log

        def _compare(self, what, o, want):
            got, want = o.float(), want.float()
            rel = float((got - want).norm() / want.norm().clamp_min(1e-30))
            bad = ((got - want).abs() > ATOL + RTOL * want.abs()).any()
            if bool(bad) or rel > REL_NORM:
                self.failures.append((self.layer_id, what, "output", rel))

        def _check_ids(self, what, ids):
            sh = self.shadow
            ok, why = ids_match_modulo_ties(ids.cpu(), sh.own_ids.cpu(), sh.last_scores.cpu())
            if not ok:
                self.failures.append((self.layer_id, what, "selection", why))
            self.ids_log.append((what, ids.cpu()))

        def first_chunk_attention(self, q, k, v):
            o = super().first_chunk_attention(q, k, v)
            self._compare("first", o, orc.attention(q, k, v, self.cfg.scale, causal_from=0))
            return o

        def prefill_first(self, q, k, v):
            self.shadow.store(k, v)
            return super().prefill_first(q, k, v)

        def prefill_chunk(self, q, k, v, device):
            o = super().prefill_chunk(q, k, v, device)
            ids = self.last_prefill_block_ids
            self.shadow.force_ids = ids
            self._compare("chunk", o, self.shadow.prefill_chunk(q, k, v))
            self._check_ids("prefill", ids)
            return o

        def decode(self, q, k, v, device):
            o = super().decode(q, k, v, device)
            ids = self._ids_view.clone()
            self.shadow.force_ids = ids
            self._compare("decode", o, self.shadow.decode(q, k, v))
            self._check_ids("decode", ids)
            return o

        def verify_tokens(self, q, k, v, device):
            o = super().verify_tokens(q, k, v, device)
            ids = self.last_verify_block_ids.clone()
            if self.verify_lossless:
                # per-query selection: the union and the output must be the oracle's own
                want = self.shadow.verify(q, k, v, lossless=True)
                if not torch.equal(ids.cpu(), self.shadow.own_ids.cpu()):
                    self.failures.append((self.layer_id, "verify", "union", ids.tolist()[:8]))
                else:
                    self._compare("verify", o, want)
                self.ids_log.append(("verify", ids.cpu()))
            else:
                # shared selection: the oracle attends arm A's blocks
                self.shadow.force_ids = ids
                self._compare("verify", o, self.shadow.verify(q, k, v, lossless=False))
                self._check_ids("verify", ids)
            return o

        def commit_verified(self, n):
            super().commit_verified(n)
            self.shadow.commit(n)
    return Shadowed


def _run_parity(cfg_kw, oracle_kw):
    nkv = pkg()
    from importlib import import_module
    H = import_module(nkv.__name__ + ".qwen3_harness")
    from oracle.harness_runtime import OracleAttentionRuntime

    assert not torch.backends.cuda.matmul.allow_tf32
    arch = H.Qwen3Arch()
    prompt = torch.randint(0, arch.vocab_size, (PROMPT,), generator=torch.Generator().manual_seed(2))
    m12 = dict(max_model_len=PROMPT + 1024, device=DEV, **cfg_kw)
    ocfg = orc.OracleConfig(device=DEV, **oracle_kw)
    Shadowed = _shadowed_runtime(nkv)
    failures, logs = [], []

    def make(i):
        rt = Shadowed(i, nkv.M12Config(**m12))
        logs.append([])
        rt.setup(ocfg, failures, logs[-1])
        return rt
    model = H.Qwen3SparseModel(arch, make, device=DEV, seed=0)

    # ---- arm A, every call shadowed by the oracle ------------------------------------
    tok = model.prefill(prompt, CHUNK)
    toks_a = [int(tok)]
    for _ in range(STEPS):
        tok = model.decode_step(tok)
        toks_a.append(int(tok))
    model.check_errors()
    assert all(sum(w == "prefill" for w, _ in lg) == PROMPT // CHUNK - 1 for lg in logs)
    assert all(sum(w == "decode" for w, _ in lg) == STEPS for lg in logs)
    assert not failures, f"{len(failures)} calls outside the parity bounds: {failures[:6]}"
    prefill_ids = [[ids for w, ids in lg if w == "prefill"] for lg in logs]
    decode_ids = [[ids for w, ids in lg if w == "decode"] for lg in logs]
    for layer in model.layers:
        layer.rt = None
    gc.collect()
    torch.cuda.empty_cache()

    # ---- arm B: oracle runtime on arm A's tokens and blocks ----------------------
    for i, layer in enumerate(model.layers):
        layer.rt = ForcedOracle(OracleAttentionRuntime(ocfg, DEV), prefill_ids[i], decode_ids[i])
    model.position = 0
    tok_b, logits = model.prefill(prompt, CHUNK, return_logits=True)
    rows = [(int(tok_b), logits[0].float())]
    for j in range(STEPS):
        tok_b, logits = model.decode_step(torch.tensor([toks_a[j]], device=DEV), return_logits=True)
        rows.append((int(tok_b), logits[0].float()))
    model.check_errors()
    differ = [(j, ta, tb, float(lg[tb] - lg[ta])) for j, ((tb, lg), ta) in enumerate(zip(rows, toks_a)) if tb != ta]
    print(f"\n{len(rows) - len(differ)}/{len(rows)} greedy tokens identical; the rest are near-ties "
          f"(step, arm A, arm B, logit gap in B): {differ[:12]}")
    outside = [d for d in differ if d[3] > TIE_BAND]
    assert not outside, f"token differences outside the tie band: {outside[:8]}"


def test_greedy_tokens_c2_hbm_history():
    _run_parity({}, {})


def test_greedy_tokens_c3_int8_host_history():
    _run_parity({"quant_history": True, "kv_residency": "host"}, {"quant_history": True})


def test_decode_loop_matches_eager_decode():
    """Two identical models (same weights, same prompt): greedy decode replayed
    from the CUDA graph and eager decode steps emit the same tokens, and every
    layer's recent window holds the same bytes afterwards."""
    nkv = pkg()
    from importlib import import_module
    H = import_module(nkv.__name__ + ".qwen3_harness")
    arch = H.Qwen3Arch(num_layers=6)
    prompt = torch.randint(0, arch.vocab_size, (8192 + 333,), generator=torch.Generator().manual_seed(5))

    def mk(i):
        return nkv.M12LayerRuntime(i, nkv.M12Config(max_model_len=16384, device=DEV))
    G = H.Qwen3SparseModel(arch, mk, device=DEV, seed=3)
    E = H.Qwen3SparseModel(arch, mk, device=DEV, seed=3)
    with torch.inference_mode():
        tg, te = G.prefill(prompt), E.prefill(prompt)
        assert int(tg) == int(te)
        tg, te = G.decode_step(tg), E.decode_step(te)
        loop = H.DecodeLoop(G, tg, max_steps=64)
        graph_toks = loop.run(40)
        eager_toks = []
        for _ in range(40):
            te = E.decode_step(te)
            eager_toks.append(int(te))
    assert graph_toks == eager_toks
    for a, b in zip(G.runtimes, E.runtimes):
        assert a.valid_len == b.valid_len
        assert torch.equal(a.recent_k, b.recent_k) and torch.equal(a.recent_v, b.recent_v)
