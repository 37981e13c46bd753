"""CPU restatement of the reference's M12 block-sparse attention path.

(The same torch code also runs on a CUDA device, in fp32 with TF32 off, for
the full-model token-parity runs; ``OracleConfig.device`` places the state.)

TEST INFRASTRUCTURE ONLY.  Nothing in the product package imports this module;
only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its ``cpu_baseline``
leg and ``--impl reference`` arm) may use it, and there only as the checker or as
the timed CPU baseline.

Every function restates one piece of ``nanovllm/sparse/m12_runtime.py`` (and
``quant_kv.py``) from the reference project, in float32 torch on the host.  The
citation of the reference line range is in each docstring.  Parity pin: the
state machine below is checked against fixtures produced by running the
reference's own ``M12LayerRuntime`` on the CPU (``tests/golden/make_golden.py``),
see ``tests/test_oracle_golden.py``.

Ordering convention: the reference ranks blocks with ``torch.topk``; ties in the
fp32 block score are ordered by torch internals.  This oracle ranks by
(score descending, block id ascending), a total order the CUDA kernels reproduce.
Equal-score blocks are the only place the two may differ.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

QMAX = 127  # reference quant_kv.py:21


# ----------------------------------------------------------------------------
# Pure helpers
# ----------------------------------------------------------------------------
def recent_slice(valid_len: int, sink_tokens: int, recent_tokens: int):
    """Segment of the left-aligned prefill recent buffer not covered by the sink.

    Reference: m12_runtime.py:32-50 (``prefill_recent_slice``).
    Returns (buffer_start, buffer_offset, length).
    """
    assert valid_len >= 0 and sink_tokens >= 0 and recent_tokens >= 0
    sink_len = min(sink_tokens, valid_len)
    buf_len = min(recent_tokens, valid_len)
    buf_start = valid_len - buf_len
    first = max(sink_len, buf_start)
    return buf_start, first - buf_start, valid_len - first


def query_summaries(q: torch.Tensor, nseg: int) -> torch.Tensor:
    """Per-segment mean of the chunk queries.  Reference: m12_runtime.py:53-67."""
    assert q.ndim == 3 and nseg > 0
    nseg = min(nseg, q.shape[0])
    if nseg == 1:
        return q.mean(dim=0, keepdim=True)
    parts = torch.tensor_split(q, nseg)
    return torch.stack([p.mean(dim=0) for p in parts])


def dynamic_budget(top_scores: torch.Tensor, max_k: int, mass: float) -> int:
    """Half / three-quarter / full budget choice.  Reference: m12_runtime.py:70-95."""
    n = top_scores.numel()
    if n < max_k or n <= 1 or not bool(torch.isfinite(top_scores).all()):
        return n
    sd = top_scores.std(unbiased=False)
    if float(sd) <= 1e-6:
        return n
    w = torch.softmax((top_scores - top_scores[0]) / sd, dim=0).cumsum(0)
    for c in sorted({max(1, (max_k + 1) // 2), max(1, (3 * max_k + 3) // 4), max_k}):
        if float(w[c - 1]) >= mass:
            return c
    return max_k


def rank_blocks(scores: torch.Tensor) -> torch.Tensor:
    """Block ids ordered by (score desc, id asc)."""
    n = scores.numel()
    ids = torch.arange(n, device=scores.device)
    # stable sort on -score keeps ascending ids among equal scores
    order = torch.sort(-scores.double(), stable=True).indices
    return ids[order]


# ----------------------------------------------------------------------------
# Representatives (reference m12_runtime.py:354-395)
# ----------------------------------------------------------------------------
def build_reps(k_blocks: torch.Tensor, r: int):
    """Pick r real keys per (block, kv head) by mean-direction + farthest point.

    k_blocks: [N, B, H, D] (any float dtype).  Returns (reps [H, N, r, D] in the
    input dtype, token index [H, N, r] int64, margins [H, N, r] float64).
    ``margins`` is the gap between the chosen token's criterion and the runner-up,
    used by tests to recognise fp32 near-ties.
    """
    N, B, H, D = k_blocks.shape
    kf = k_blocks.float().permute(2, 0, 1, 3)             # [H, N, B, D]
    norm = kf.norm(dim=-1, keepdim=True).clamp_min(1e-12)
    kd = kf / norm                                       # unit directions
    mean = kd.mean(dim=2)                                # [H, N, D]
    mean = mean / mean.norm(dim=-1, keepdim=True).clamp_min(1e-12)
    crit = (kd * mean.unsqueeze(2)).sum(-1)              # [H, N, B] cos to mean dir
    dev = k_blocks.device
    chosen = torch.empty(H, N, r, dtype=torch.long, device=dev)
    margins = torch.empty(H, N, r, dtype=torch.float64, device=dev)

    # step 0: first token of maximal cosine to the mean direction
    top2 = torch.topk(crit, min(2, B), dim=-1).values
    chosen[..., 0] = crit.argmax(-1)
    margins[..., 0] = (top2[..., 0] - top2[..., -1]).double() if B > 1 else math.inf

    # steps 1..r-1: the reference raises the running max-cosine to at least 0
    # (``torch.maximum(max_cos, mask)`` with a zero mask, m12_runtime.py:386-389)
    # and sets already-chosen tokens to 2.0, then takes the FIRST argmin.  So the
    # pick is the first token whose max-cosine is <= 0, else the smallest one.
    worst = torch.full((H, N, B), -math.inf, device=dev)
    taken = torch.zeros(H, N, B, dtype=torch.bool, device=dev)
    pos = torch.arange(B, device=dev)
    for s in range(1, r):
        prev = chosen[..., s - 1]
        taken.scatter_(2, prev.unsqueeze(-1), True)
        pdir = torch.gather(kd, 2, prev[..., None, None].expand(H, N, 1, D))
        cos = (kd * pdir).sum(-1)                         # [H, N, B]
        worst = torch.maximum(worst, cos)
        crit_s = torch.where(taken, torch.full_like(worst, 2.0), worst.clamp_min(0.0))
        c = crit_s.argmin(-1)
        chosen[..., s] = c
        # sensitivity of the decision to fp32 rounding of ``worst``
        raw = torch.where(taken, torch.full_like(worst, 2.0), worst).double()
        rc = torch.gather(raw, 2, c.unsqueeze(-1)).squeeze(-1)
        clamped = rc <= 0
        earlier = torch.where((pos < c.unsqueeze(-1)) & ~taken, raw,
                              torch.full_like(raw, math.inf)).amin(-1)
        others = torch.where(pos == c.unsqueeze(-1), torch.full_like(raw, math.inf),
                             (raw - rc.unsqueeze(-1)).abs()).amin(-1)
        margins[..., s] = torch.where(clamped, torch.minimum(rc.abs(), earlier), others)
    src = k_blocks.permute(2, 0, 1, 3)                    # [H, N, B, D]
    reps = torch.gather(src, 2, chosen[..., None].expand(H, N, r, D))
    return reps, chosen, margins


# ----------------------------------------------------------------------------
# Block scores and selection (reference m12_runtime.py:959-1087)
# ----------------------------------------------------------------------------
def block_scores(q: torch.Tensor, reps: torch.Tensor, nblocks: int) -> torch.Tensor:
    """score[b] = max over query rows, query heads and reps of q·rep (fp32).

    q: [nq, Hq, D]; reps: [Hkv, >=nblocks, r, D].  Reference m12_runtime.py:999-1003.
    """
    nq, hq, d = q.shape
    hkv = reps.shape[0]
    g = hq // hkv
    qf = q.float().view(nq, hkv, g, d)
    rf = reps[:, :nblocks].float()                        # [Hkv, n, r, D]
    s = torch.einsum("qhgd,hbrd->qhgbr", qf, rf)
    return s.amax(dim=(0, 1, 2, 4))


def per_query_scores(q: torch.Tensor, reps: torch.Tensor, nblocks: int) -> torch.Tensor:
    """[Tq, nblocks] per-query block scores.  Reference m12_runtime.py:1071-1075."""
    nq, hq, d = q.shape
    hkv = reps.shape[0]
    qf = q.float().view(nq, hkv, hq // hkv, d)
    s = torch.einsum("qhgd,hbrd->qhgbr", qf, reps[:, :nblocks].float())
    return s.amax(dim=(1, 2, 4))


def mask_protected(scores: torch.Tensor, protected, nblocks: int) -> torch.Tensor:
    out = scores.clone()
    ids = [p for p in protected if 0 <= p < nblocks]
    if ids:
        out[torch.tensor(ids, dtype=torch.long, device=out.device)] = -math.inf
    return out


def select_k(nblocks: int, protected, requested: int) -> int:
    """Budget after protection.  Reference m12_runtime.py:984-988."""
    avail = nblocks - len([p for p in protected if p < nblocks])
    return min(requested, max(1, avail))


def select_blocks(q, reps, nblocks, protected, requested):
    """Returns (ids [k] int64, masked scores [nblocks] fp32)."""
    if q.ndim == 2:
        q = q.unsqueeze(0)
    s = mask_protected(block_scores(q, reps, nblocks), protected, nblocks)
    k = select_k(nblocks, protected, requested)
    return rank_blocks(s)[:k].clone(), s


def select_per_query(q, reps, nblocks, protected, requested):
    """Lossless-verify selection: per-query top-k, sorted union, allowed mask.

    Reference m12_runtime.py:1057-1087.  Returns (union [U], allowed [Tq, U] bool,
    per-query masked scores [Tq, nblocks]).
    """
    s = per_query_scores(q, reps, nblocks)
    s = torch.stack([mask_protected(row, protected, nblocks) for row in s])
    k = select_k(nblocks, protected, requested)
    top = torch.stack([rank_blocks(row)[:k] for row in s])          # [Tq, k]
    union = torch.unique(top.flatten())
    pos = torch.searchsorted(union, top.flatten()).view(top.shape)
    allowed = torch.zeros(q.shape[0], union.numel(), dtype=torch.bool, device=q.device)
    allowed.scatter_(1, pos, True)
    return union, allowed, s


# ----------------------------------------------------------------------------
# Attention (reference m12_runtime.py:845-896)
# ----------------------------------------------------------------------------
def attention(q, k, v, scale, causal_from=None, disallow=None):
    """fp32 softmax attention of q [Tq,Hq,D] over packed k,v [S,Hkv,D].

    Keys at index >= causal_from are the current chunk: query t sees chunk keys
    up to causal_from + t.  ``disallow`` [Tq, S] bool masks extra keys.  Output in
    float32 [Tq, Hq, D].
    """
    tq, hq, d = q.shape
    s_len, hkv, _ = k.shape
    g = hq // hkv
    qf = q.float().view(tq, hkv, g, d)
    logits = torch.einsum("thgd,shd->thgs", qf, k.float()) * scale
    if q.is_cuda and torch.backends.cuda.matmul.allow_tf32:
        raise RuntimeError("the oracle's fp32 attention needs TF32 matmuls disabled")
    mask = torch.zeros(tq, s_len, dtype=torch.bool, device=q.device)
    if disallow is not None:
        mask |= disallow
    if causal_from is not None and causal_from < s_len:
        col = torch.arange(s_len, device=q.device).unsqueeze(0)
        row = torch.arange(tq, device=q.device).unsqueeze(1) + causal_from
        mask |= (col > row) & (col >= causal_from)
    if mask.any():
        logits = logits.masked_fill(mask[:, None, None, :], -math.inf)
    p = torch.softmax(logits, dim=-1)
    o = torch.einsum("thgs,shd->thgd", p, v.float())
    return o.reshape(tq, hq, d)


# ----------------------------------------------------------------------------
# Quantisation, reference scheme (reference m12_runtime.py:460-474, quant_kv.py)
# ----------------------------------------------------------------------------
def k_channel_scale(k_blocks):
    """[Hkv, D] fp32 scale from a [N, B, Hkv, D] window."""
    return k_blocks.float().abs().amax(dim=(0, 1)).clamp_min(1e-8) / QMAX


def quant_k(k_blocks, k_scale):
    return torch.round(k_blocks.float() / k_scale).clamp(-QMAX, QMAX).to(torch.int8)


def quant_v_blocks(v_blocks):
    """Returns (int8 [N,B,Hkv,D], scale [N,Hkv] fp32)."""
    vs = v_blocks.float().abs().amax(dim=(1, 3)).clamp_min(1e-8) / QMAX
    vq = torch.round(v_blocks.float() / vs[:, None, :, None]).clamp(-QMAX, QMAX)
    return vq.to(torch.int8), vs


# Per-token per-kv-head scheme (the variant BASELINE config 3 names): scale is
# amax over D for each (token, head), stored as bf16; dequant = int8 * bf16 scale.
def quant_token_head(x):
    """x [T, Hkv, D] -> (int8 [T,Hkv,D], scale [T,Hkv] bf16)."""
    xf = x.float()
    sc = (xf.abs().amax(dim=-1).clamp_min(1e-8) / QMAX).to(torch.bfloat16)
    q = torch.round(xf / sc.float()[..., None]).clamp(-QMAX, QMAX).to(torch.int8)
    return q, sc


# ----------------------------------------------------------------------------
# The per-layer state machine (reference M12LayerRuntime)
# ----------------------------------------------------------------------------
@dataclass
class OracleConfig:
    block_size: int = 64
    r: int = 4
    recent_tokens: int = 512
    sink_tokens: int = 64
    top_k_blocks: int = 32
    prefill_top_k_blocks: int | None = None
    decode_top_k_blocks: int | None = None
    num_heads: int = 32
    num_kv_heads: int = 8
    head_dim: int = 128
    dtype: torch.dtype = torch.bfloat16
    scale: float = 128.0 ** -0.5
    quant_history: bool = False
    prefill_query_segments: int = 1
    gather_sort: bool = False
    # decode selection variants (reference M12Config fields, m12_runtime.py:110-121)
    dynamic_top_k: bool = False
    dynamic_top_k_mass: float = 0.90
    decode_relative_a: float | None = None
    decode_relative_max_blocks: int = 48
    decode_relative_union: bool = False
    decode_query_window: int = 1
    # where the layer state lives ("cpu", or a CUDA device for full-model runs)
    device: str = "cpu"


def relative_select(scores: torch.Tensor, nblocks: int, protected, k: int, a: float, scale: float,
                    max_blocks: int, union: bool) -> torch.Tensor:
    """Relative-threshold decode selection.  Reference m12_runtime.py:1015-1031:
    candidates are the best ``min(max_blocks, avail)`` blocks; keep those whose
    masked score is within ln(a)/scale of the best (with ``union``, also every
    candidate ranked below k); if none qualifies, the first k."""
    avail = nblocks - len([p for p in protected if p < nblocks])
    threshold = float(scores.amax()) + math.log(a) / scale
    cap = min(max_blocks, max(1, avail))
    order = rank_blocks(scores)
    cand = order[:cap]
    above = scores[cand] >= threshold
    if union:
        above = above | (torch.arange(cand.numel(), device=scores.device) < k)
    keep = cand[above]
    if keep.numel() == 0:
        keep = order[:k]
    return keep.clone()


@dataclass
class OracleLayer:
    """Reference-semantics layer state (m12_runtime.py:169-292, 420-513, 1141-1346)."""

    cfg: OracleConfig
    k_hist: list = field(default_factory=list)   # per block [B, Hkv, D] (dtype or int8)
    v_hist: list = field(default_factory=list)
    v_scale: list = field(default_factory=list)   # per block [Hkv] fp32 (quant)
    reps: torch.Tensor | None = None              # [Hkv, nblocks, r, D]
    rep_idx: torch.Tensor | None = None
    rep_margin: torch.Tensor | None = None
    k_scale: torch.Tensor | None = None
    sink_k: torch.Tensor | None = None
    sink_v: torch.Tensor | None = None
    recent_k: torch.Tensor | None = None          # [R, Hkv, D] logical, left-aligned
    recent_v: torch.Tensor | None = None
    valid_len: int = 0
    prefill_len: int = 0
    nblocks: int = 0
    protected: set = field(default_factory=set)
    last_ids: torch.Tensor | None = None
    last_scores: torch.Tensor | None = None
    own_ids: torch.Tensor | None = None           # selection before any override
    force_ids: torch.Tensor | None = None         # test hook: ids to use for the next step
    pending: tuple | None = None
    q_window: list = field(default_factory=list)  # decode routing queries (decode_query_window > 1)

    def __post_init__(self):
        c = self.cfg
        z = lambda n: torch.zeros(n, c.num_kv_heads, c.head_dim, dtype=c.dtype, device=c.device)
        self.sink_k, self.sink_v = z(c.sink_tokens), z(c.sink_tokens)
        self.recent_k, self.recent_v = z(c.recent_tokens), z(c.recent_tokens)
        self.reps = torch.zeros(c.num_kv_heads, 0, c.r, c.head_dim, dtype=c.dtype, device=c.device)
        self.rep_idx = torch.zeros(c.num_kv_heads, 0, c.r, dtype=torch.long, device=c.device)
        self.rep_margin = torch.zeros(c.num_kv_heads, 0, c.r, dtype=torch.float64, device=c.device)

    # -- store (m12_runtime.py:420-513) ------------------------------------
    def store(self, k, v):
        c = self.cfg
        B = c.block_size
        T = k.shape[0]
        assert T >= 2
        nb = -(-T // B)
        pad = nb * B - T
        kp = torch.cat([k, k.new_zeros(pad, *k.shape[1:])]) if pad else k
        vp = torch.cat([v, v.new_zeros(pad, *v.shape[1:])]) if pad else v
        kb = kp.reshape(nb, B, c.num_kv_heads, c.head_dim)
        vb = vp.reshape(nb, B, c.num_kv_heads, c.head_dim)
        if c.quant_history:
            if self.k_scale is None:
                self.k_scale = k_channel_scale(kb)
            kq = quant_k(kb, self.k_scale)
            vq, vs = quant_v_blocks(vb)
            self.k_hist += list(kq)
            self.v_hist += list(vq)
            self.v_scale += list(vs)
        else:
            self.k_hist += list(kb.clone())
            self.v_hist += list(vb.clone())
        reps, idx, marg = build_reps(kb, c.r)
        self.reps = torch.cat([self.reps, reps], dim=1)
        self.rep_idx = torch.cat([self.rep_idx, idx], dim=1)
        self.rep_margin = torch.cat([self.rep_margin, marg], dim=1)
        if self.prefill_len == 0:
            n = min(c.sink_tokens, T)
            self.sink_k[:n] = k[:n]
            self.sink_v[:n] = v[:n]
        self._recent_append(k, v)
        self.prefill_len += T
        need = self.nblocks + nb
        self.nblocks = need
        nrb = c.recent_tokens // B
        self.protected = {0} | set(range(max(1, need - nrb), need))

    def _recent_append(self, k, v):
        """Left-aligned recent window update shared by store and commit.

        Reference m12_runtime.py:488-503 and 788-802.  Advances valid_len.
        """
        R = self.cfg.recent_tokens
        T = k.shape[0]
        new_len = min(R, self.valid_len + T)
        if T >= new_len:
            self.recent_k[:new_len] = k[T - new_len:]
            self.recent_v[:new_len] = v[T - new_len:]
        else:
            carry = new_len - T
            old_len = min(R, self.valid_len)
            self.recent_k[:carry] = self.recent_k[old_len - carry:old_len].clone()
            self.recent_v[:carry] = self.recent_v[old_len - carry:old_len].clone()
            self.recent_k[carry:new_len] = k
            self.recent_v[carry:new_len] = v
        self.valid_len += T

    # -- history gather -------------------------------------------------------
    def gather(self, ids):
        c = self.cfg
        if ids.numel() == 0:
            e = torch.zeros(0, c.num_kv_heads, c.head_dim, dtype=c.dtype, device=c.device)
            return e, e.clone()
        if c.quant_history:
            ks = torch.stack([self.k_hist[i].float() * self.k_scale for i in ids.tolist()])
            vs = torch.stack([self.v_hist[i].float() * self.v_scale[i][None, :, None]
                              for i in ids.tolist()])
            ks, vs = ks.to(c.dtype), vs.to(c.dtype)
        else:
            ks = torch.stack([self.k_hist[i] for i in ids.tolist()])
            vs = torch.stack([self.v_hist[i] for i in ids.tolist()])
        return (ks.reshape(-1, c.num_kv_heads, c.head_dim),
                vs.reshape(-1, c.num_kv_heads, c.head_dim))

    def _select(self, q, budget):
        c = self.cfg
        req = c.top_k_blocks if budget is None else budget
        ids, s = select_blocks(q, self.reps, self.nblocks, self.protected, req)
        if c.gather_sort and ids.numel() > 1:
            ids = ids.sort().values
        return self._adopt(ids, s)

    def _adopt(self, ids, scores):
        self.own_ids, self.last_scores = ids, scores
        if self.force_ids is not None:
            ids, self.force_ids = torch.as_tensor(self.force_ids, dtype=torch.long).to(ids.device), None
        self.last_ids = ids
        return ids

    def _history_pack(self, ids, k, v):
        """[selected | sink | recent (sink-deduplicated) | current]; m12_runtime.py:589-636."""
        c = self.cfg
        hk, hv = self.gather(ids)
        sink_len = min(c.sink_tokens, self.valid_len)
        _, off, rlen = recent_slice(self.valid_len, c.sink_tokens, c.recent_tokens)
        kk = [hk, self.sink_k[:sink_len], self.recent_k[off:off + rlen], k]
        vv = [hv, self.sink_v[:sink_len], self.recent_v[off:off + rlen], v]
        causal_from = hk.shape[0] + sink_len + rlen
        return torch.cat(kk), torch.cat(vv), causal_from

    # -- prefill --------------------------------------------------------------
    def prefill_first(self, q, k, v):
        """m12_runtime.py:518-523 (store only) + the caller's dense causal attention."""
        assert self.prefill_len == 0
        o = attention(q, k, v, self.cfg.scale, causal_from=0)
        self.store(k, v)
        return o

    def prefill_chunk(self, q, k, v, forced_ids=None):
        """m12_runtime.py:528-651 with the torch backend (mask of :875-896)."""
        c = self.cfg
        assert self.prefill_len > 0
        if forced_ids is None:
            qs = query_summaries(q, c.prefill_query_segments)
            ids = self._select(qs, c.prefill_top_k_blocks)
        else:
            ids = torch.as_tensor(forced_ids, dtype=torch.long).to(q.device)
            self.last_ids = ids
        kp, vp, cf = self._history_pack(ids, k, v)
        o = attention(q, kp, vp, c.scale, causal_from=cf)
        self.store(k, v)
        return o

    # -- verify (m12_runtime.py:656-807) -------------------------------------
    def verify(self, q, k, v, lossless: bool):
        c = self.cfg
        B = c.block_size
        if lossless:
            ids, allowed, s = select_per_query(q, self.reps, self.nblocks,
                                               self.protected, c.top_k_blocks)
            self.own_ids, self.last_scores, self.last_ids = ids, s, ids
        else:
            ids = self._select(q, None)
        kp, vp, cf = self._history_pack(ids, k, v)
        dis = None
        if lossless:
            dis = torch.zeros(q.shape[0], kp.shape[0], dtype=torch.bool, device=q.device)
            dis[:, :ids.numel() * B] = ~allowed.repeat_interleave(B, dim=1)
        o = attention(q, kp, vp, c.scale, causal_from=cf, disallow=dis)
        self.pending = (k, v)
        return o

    def commit(self, n):
        if n > 0:
            k, v = self.pending
            self._recent_append(k[:n], v[:n])
        self.pending = None

    # -- decode (m12_runtime.py:1141-1346) ------------------------------------
    def _decode_select(self, q_route):
        """Decode block choice with the configured variant (reference
        m12_runtime.py:1193-1198 -> _gpu_select :959-1055)."""
        c = self.cfg
        req = c.top_k_blocks if c.decode_top_k_blocks is None else c.decode_top_k_blocks
        s = mask_protected(block_scores(q_route.unsqueeze(0), self.reps, self.nblocks),
                           self.protected, self.nblocks)
        k = select_k(self.nblocks, self.protected, req)
        if c.decode_relative_a is not None:
            ids = relative_select(s, self.nblocks, self.protected, k, c.decode_relative_a, c.scale,
                                  c.decode_relative_max_blocks, c.decode_relative_union)
        else:
            ids = rank_blocks(s)[:k].clone()
            if c.dynamic_top_k and k == req:
                ids = ids[:dynamic_budget(s[ids], req, c.dynamic_top_k_mass)]
        if c.gather_sort and ids.numel() > 1:
            ids = ids.sort().values
        return self._adopt(ids, s)

    def _routing_query(self, q):
        """Mean of the last decode_query_window queries (reference :1181-1190)."""
        c = self.cfg
        if c.decode_query_window <= 1:
            return q[0]
        self.q_window.append(q[0])
        while len(self.q_window) > c.decode_query_window:
            self.q_window.pop(0)
        if len(self.q_window) == 1:
            return self.q_window[0]
        return torch.stack(self.q_window, dim=0).mean(dim=0)

    def decode(self, q, k, v):
        c = self.cfg
        # shift-left-and-append on the full R-slot window (m12_runtime.py:1169-1172)
        self.recent_k = torch.cat([self.recent_k[1:], k[:1]])
        self.recent_v = torch.cat([self.recent_v[1:], v[:1]])
        ids = self._decode_select(self._routing_query(q))
        hk, hv = self.gather(ids)
        sink_len = min(c.sink_tokens, self.valid_len)
        rlen = min(c.recent_tokens, self.valid_len + 1)
        R = c.recent_tokens
        kp = torch.cat([hk, self.sink_k[:sink_len], self.recent_k[R - rlen:]])
        vp = torch.cat([hv, self.sink_v[:sink_len], self.recent_v[R - rlen:]])
        o = attention(q, kp, vp, c.scale)
        self.valid_len += 1
        return o
