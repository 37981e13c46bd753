"""Full-model harness: a Qwen3 decoder whose attention layers call the sparse
runtime exactly as the reference's ``Attention.forward`` does.

The reference runs its sparse path inside ``nanovllm/models/qwen3.py``
(``Qwen3Attention.forward`` :85-101 -> ``Attention.forward``,
``nanovllm/layers/attention.py:64-99``), with one ``M12LayerRuntime`` per layer
installed by ``ModelRunner.allocate_kv_cache`` (``nanovllm/engine/model_runner.py:134-185``).
This module is that caller, built for B200:

* the dense projections are cuBLAS GEMMs (``torch.nn.functional.linear``)
  for chunks, and this package's weight-streaming GEMV (``nkv_gemv_bf16``) for
  one to four tokens (decode);
* the elementwise work around them is this package's kernels: residual add +
  RMSNorm (``nkv_add_rms_norm``), the per-head q/k RMSNorm fused with the YaRN
  rotary embedding in place on the qkv projection output (``nkv_qk_norm_rope``,
  whose q/k/v views are what the sparse runtime reads), SwiGLU (``nkv_silu_mul``);
* prefill runs in chunks: the first chunk's dense causal attention
  (the reference's FA2 varlen call, attention.py:80-85) then ``prefill_first``,
  later chunks ``prefill_chunk``; decode calls ``decode`` per layer;
* a decode step of the whole model (36 layers, logits, greedy argmax, token
  feedback) can be recorded once in a CUDA graph and replayed per token
  (``DecodeLoop``), the recent windows advancing on the device
  (``DeviceRingHeads``); the reference runs sparse decode eagerly
  (``nanovllm/config.py:180``).

The attention runtime of each layer comes from a factory, so the same model can
run this package's ``M12LayerRuntime`` or any object with its methods
(``first_chunk_attention``, ``prefill_first``, ``prefill_chunk``, ``decode``,
``verify_tokens``, ``commit_verified``, ``rollback_verified``, ``prefill_len``).

Weights are random (seeded N(0, 0.02), norm weights one, embeddings tied to the
LM head as in Qwen3-4B): there are no checkpoints here.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

from . import _lib
from ._lib import call


@dataclass
class Qwen3Arch:
    """Qwen3-4B architecture."""

    vocab_size: int = 151936
    hidden_size: int = 2560
    num_layers: int = 36
    num_heads: int = 32
    num_kv_heads: int = 8
    head_dim: int = 128
    intermediate_size: int = 9728
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1e6
    rope_scaling: dict = field(default_factory=lambda: {"rope_type": "yarn", "factor": 4.0,
                                                        "original_max_position_embeddings": 32768})
    max_position: int = 131072 + 2048


def rope_cos_sin(arch: Qwen3Arch, device, max_position: int | None = None) -> torch.Tensor:
    """cos/sin table [P, head_dim] fp32 (cos in the first half, sin in the second).

    YaRN as the reference computes it (layers/rotary_embedding.py:46-126, the
    HuggingFace parameterisation): the inverse frequencies blended between
    interpolation (1 / (factor * base^(2i/d))) and extrapolation by a linear ramp
    between the correction dims of beta_fast=32 / beta_slow=1 (floor/ceil),
    cos and sin scaled by mscale = 0.1 ln(factor) + 1; plain RoPE when
    ``rope_scaling`` is None.
    """
    d = arch.head_dim
    base = arch.rope_theta
    P = max_position or arch.max_position
    rs = arch.rope_scaling
    pos_freqs = base ** (torch.arange(0, d, 2, dtype=torch.float, device=device) / d)
    if rs and rs.get("rope_type", rs.get("type")) == "yarn":
        factor = float(rs.get("factor", 1.0))
        orig = int(rs.get("original_max_position_embeddings", P))
        beta_fast, beta_slow = float(rs.get("beta_fast", 32)), float(rs.get("beta_slow", 1))

        def corr_dim(rot):
            return (d * math.log(orig / (rot * 2 * math.pi))) / (2 * math.log(base))
        low, high = math.floor(corr_dim(beta_fast)), math.ceil(corr_dim(beta_slow))
        low, high = max(low, 0), min(high, d - 1)
        if low == high:
            high += 0.001
        ramp = torch.clamp((torch.arange(d // 2, dtype=torch.float, device=device) - low) / (high - low), 0.0, 1.0)
        extra = 1.0 - ramp
        inv_freq = (1.0 / (factor * pos_freqs)) * (1.0 - extra) + (1.0 / pos_freqs) * extra
        att = rs.get("attention_factor")
        mscale = float(att) if att is not None else (0.1 * math.log(factor) + 1.0 if factor > 1 else 1.0)
    else:
        inv_freq = 1.0 / pos_freqs
        mscale = 1.0
    t = torch.arange(P, dtype=torch.float, device=device)
    freqs = torch.einsum("i,j -> ij", t, inv_freq)
    return torch.cat((freqs.cos() * mscale, freqs.sin() * mscale), dim=-1).contiguous()


class _Layer:
    __slots__ = ("w_in", "wqkv", "q_norm", "k_norm", "wo", "w_post", "wgu", "wd", "rt")


def _stream(dev) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


class Qwen3SparseModel:
    """Random-init Qwen3 decoder with one sparse attention runtime per layer.

    ``make_runtime(layer_id)`` returns the layer's runtime (an ``M12LayerRuntime``
    or any object with its methods).  All tensors live on ``device``.
    """

    def __init__(self, arch: Qwen3Arch, make_runtime, device="cuda", seed: int = 0, init_std: float = 0.02):
        _lib.load()
        self.arch = a = arch
        dev = torch.device(device)
        if dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        if a.head_dim != 128:
            raise _lib.NanoKVUnsupported("Qwen3SparseModel", _lib.NKV_ERR_UNSUPPORTED, "head_dim must be 128")
        g = torch.Generator(device=dev).manual_seed(seed)

        def w(*shape):
            t = torch.empty(*shape, dtype=torch.bfloat16, device=dev)
            t.normal_(0.0, init_std, generator=g)
            return t

        def ones(n):
            return torch.ones(n, dtype=torch.bfloat16, device=dev)
        H, D = a.hidden_size, a.head_dim
        self.q_size, self.kv_size = a.num_heads * D, a.num_kv_heads * D
        self.embed = w(a.vocab_size, H)      # tied LM head (tie_word_embeddings)
        self.layers: list[_Layer] = []
        for i in range(a.num_layers):
            L = _Layer()
            L.w_in, L.w_post = ones(H), ones(H)
            L.wqkv = w(self.q_size + 2 * self.kv_size, H)
            L.q_norm, L.k_norm = ones(D), ones(D)
            L.wo = w(H, self.q_size)
            L.wgu = w(2 * a.intermediate_size, H)
            L.wd = w(H, a.intermediate_size)
            L.rt = make_runtime(i)
            self.layers.append(L)
        self.w_final = ones(H)
        self.cos_sin = rope_cos_sin(a, dev)
        self.err = torch.zeros(4, dtype=torch.int32, device=dev)
        self.position = 0
        # with record_ids set, every eager prefill-chunk and decode call appends
        # the layer's selected block ids (host int64): record[mode][layer]
        self.record_ids = False
        self.record = {"prefill": [[] for _ in self.layers], "decode": [[] for _ in self.layers]}
        self.decode_queries = None  # set by DecodeLoop(record_ids=True) while it records
        self.use_gemv = True  # decode-time projections on nkv_gemv_bf16 (cuBLAS when False)

    @property
    def runtimes(self):
        return [L.rt for L in self.layers]

    # ------------------------------------------------------------------
    # kernels
    # ------------------------------------------------------------------
    def _norm(self, x, residual, weight, out, has_residual):
        T, H = x.shape
        call("nkv_add_rms_norm", _stream(self.device), x.data_ptr(), residual.data_ptr(), weight.data_ptr(),
             out.data_ptr(), T, H, self.arch.rms_norm_eps, 1 if has_residual else 0)

    def _qk_norm_rope(self, qkv, positions, L):
        a = self.arch
        call("nkv_qk_norm_rope", _stream(self.device), qkv.data_ptr(), qkv.stride(0), qkv.shape[0], a.num_heads,
             a.num_kv_heads, a.head_dim, L.q_norm.data_ptr(), L.k_norm.data_ptr(), self.cos_sin.data_ptr(),
             positions.data_ptr(), self.cos_sin.shape[0], a.rms_norm_eps, self.err.data_ptr())

    def _linear(self, x, w):
        """x [T, K] @ w[N, K]^T: the library's weight-streaming GEMV for up to 4
        rows (decode), cuBLAS through torch otherwise."""
        T = x.shape[0]
        if T > 4 or not self.use_gemv or x.stride(-1) != 1:
            return F.linear(x, w)
        N, K = w.shape
        y = torch.empty(T, N, dtype=torch.bfloat16, device=self.device)
        call("nkv_gemv_bf16", _stream(self.device), x.data_ptr(), x.stride(0), T, w.data_ptr(), w.stride(0), N, K,
             y.data_ptr(), y.stride(0))
        return y

    def _silu_mul(self, gu):
        T = gu.shape[0]
        I = self.arch.intermediate_size
        out = torch.empty(T, I, dtype=torch.bfloat16, device=self.device)
        call("nkv_silu_mul", _stream(self.device), gu.data_ptr(), out.data_ptr(), T, I)
        return out

    # ------------------------------------------------------------------
    # forward
    # ------------------------------------------------------------------
    def forward(self, input_ids: torch.Tensor, positions: torch.Tensor, mode: str,
                last_only: bool = True) -> torch.Tensor:
        """Hidden states after the final norm.  ``mode`` selects the attention
        call of every layer: "prefill", "decode" or "verify"."""
        a = self.arch
        T = input_ids.shape[0]
        h = F.embedding(input_ids, self.embed)
        residual = torch.empty_like(h)
        xn = torch.empty_like(h)
        for i, L in enumerate(self.layers):
            self._norm(h, residual, L.w_in, xn, has_residual=i > 0)
            qkv = self._linear(xn, L.wqkv)
            self._qk_norm_rope(qkv, positions, L)
            q = qkv[:, :self.q_size].view(T, a.num_heads, a.head_dim)
            k = qkv[:, self.q_size:self.q_size + self.kv_size].view(T, a.num_kv_heads, a.head_dim)
            v = qkv[:, self.q_size + self.kv_size:].view(T, a.num_kv_heads, a.head_dim)
            o = self._attention(L.rt, q, k, v, mode)
            if mode == "decode" and self.decode_queries is not None:
                self.decode_queries[i] = q
            if self.record_ids and mode != "verify" and (mode == "decode" or L.rt.prefill_len > T):
                self.record[mode][i].append(L.rt.last_block_ids.clone().cpu())
            h = self._linear(o.reshape(T, self.q_size), L.wo)
            self._norm(h, residual, L.w_post, xn, has_residual=True)
            h = self._linear(self._silu_mul(self._linear(xn, L.wgu)), L.wd)
        if last_only:
            h, residual = h[-1:].contiguous(), residual[-1:].contiguous()
        out = torch.empty_like(h)
        self._norm(h, residual, self.w_final, out, has_residual=True)
        return out

    def _attention(self, rt, q, k, v, mode):
        """The reference's Attention.forward dispatch for the sparse runtime
        (attention.py:64-99)."""
        if mode == "verify":
            return rt.verify_tokens(q, k, v, q.device)
        if mode == "prefill":
            if rt.prefill_len == 0:
                o = rt.first_chunk_attention(q, k, v)
                rt.prefill_first(q, k, v)
                return o
            return rt.prefill_chunk(q, k, v, q.device)
        assert q.shape[0] == 1, "sparse decode supports a single query token"
        return rt.decode(q, k, v, q.device)

    def logits(self, hidden: torch.Tensor) -> torch.Tensor:
        return self._linear(hidden, self.embed)

    # ------------------------------------------------------------------
    # generation
    # ------------------------------------------------------------------
    @torch.inference_mode()
    def prefill(self, prompt_ids: torch.Tensor, chunk: int = 4096, return_logits: bool = False):
        """Chunked prefill of the prompt; returns the greedy next token [1] int64
        (and the last position's logits with ``return_logits``)."""
        dev = self.device
        ids = prompt_ids.to(dev)
        n = ids.shape[0]
        hidden = None
        for s in range(0, n, chunk):
            e = min(n, s + chunk)
            pos = torch.arange(s, e, dtype=torch.int64, device=dev)
            hidden = self.forward(ids[s:e], pos, "prefill", last_only=True)
        self.position = n
        logits = self.logits(hidden)
        tok = logits.argmax(dim=-1)
        return (tok, logits) if return_logits else tok

    @torch.inference_mode()
    def decode_step(self, token: torch.Tensor, return_logits: bool = False):
        """One eager decode step; returns the greedy next token [1] int64 (and
        the logits with ``return_logits``)."""
        pos = torch.full((1,), self.position, dtype=torch.int64, device=self.device)
        hidden = self.forward(token.view(1).to(self.device), pos, "decode")
        self.position += 1
        logits = self.logits(hidden)
        tok = logits.argmax(dim=-1)
        return (tok, logits) if return_logits else tok

    @torch.inference_mode()
    def generate(self, prompt_ids: torch.Tensor, steps: int, chunk: int = 4096, graph: bool = True) -> list[int]:
        """Greedy generation: the prefill's token plus ``steps`` decode steps."""
        tok = self.prefill(prompt_ids, chunk)
        out = [tok]
        if steps > 0 and graph:
            tok = self.decode_step(tok)  # one eager step sets up every layer's decode state
            out.append(tok)
            loop = DecodeLoop(self, tok)
            toks = loop.run(steps - 1)
            loop.close()
            return [int(t) for t in torch.cat(out).tolist()] + toks
        for _ in range(steps):
            tok = self.decode_step(tok)
            out.append(tok)
        return [int(t) for t in torch.cat(out).tolist()]

    # ------------------------------------------------------------------
    # speculative decoding: verify, commit, rollback
    # ------------------------------------------------------------------
    @torch.inference_mode()
    def verify(self, tokens) -> torch.Tensor:
        """One sparse verification pass over Tq tokens at positions
        ``position .. position + Tq - 1`` (the first is the current unprocessed
        token, the rest are draft proposals): every layer runs its runtime's
        ``verify_tokens`` (shared or per-query selection over the frozen
        history, nothing committed).  Returns the logits [Tq, vocab]; row i
        predicts the token after ``tokens[i]``.  Reference:
        ``ModelRunner.run_verify`` (model_runner.py:478-507)."""
        ids = torch.as_tensor(tokens, dtype=torch.int64).view(-1).to(self.device)
        Tq = ids.numel()
        pos = torch.arange(self.position, self.position + Tq, dtype=torch.int64, device=self.device)
        rts = self.runtimes
        for rt in rts:
            rt.verify_mode = True
        try:
            hidden = self.forward(ids, pos, "verify", last_only=False)
        finally:
            for rt in rts:
                rt.verify_mode = False
        return self.logits(hidden)

    def commit_verified(self, n: int) -> None:
        """Make the first n tokens of the last verify pass part of the sequence
        (their K/V enter every layer's recent window); the rest are dropped."""
        for rt in self.runtimes:
            rt.commit_verified(n)
        self.position += max(0, int(n))

    def rollback_verified(self) -> None:
        """Discard the last verify pass."""
        for rt in self.runtimes:
            rt.rollback_verified()

    @torch.inference_mode()
    def speculative_generate(self, prompt_ids: torch.Tensor, steps: int, proposer, k: int = 4,
                             chunk: int = 4096, lossless: bool = False) -> tuple[list[int], dict]:
        """Greedy speculative decoding: the prefill's token plus ``steps`` more.

        Every round the proposer drafts up to k tokens after the current one;
        one verify pass over [current, drafts] gives the target's greedy token
        after each; the drafts are accepted while they equal it, the accepted
        prefix (and the current token) is committed, and the target's token
        after the last accepted one becomes the next current token, so a round
        emits between 1 and k + 1 tokens.  A round without drafts is a plain
        decode step.  ``lossless`` selects the per-query (union + mask)
        verification.  Proposer interface (the reference's, proposers.py):
        ``prefill(prompt_ids)``, ``propose(last_token, k, pos) -> list[int]``,
        ``note_accepted(tokens)``.  Returns (tokens, stats)."""
        for rt in self.runtimes:
            rt.verify_lossless = bool(lossless)
        tok = int(self.prefill(prompt_ids, chunk))
        proposer.prefill([int(t) for t in prompt_ids.view(-1).tolist()])
        out = [tok]
        stats = {"rounds": 0, "verify_rounds": 0, "proposed": 0, "accepted": 0}
        while len(out) < steps + 1:
            want = min(k, steps + 1 - len(out) - 1)
            drafts = [int(t) for t in proposer.propose(tok, want, self.position)][:max(0, want)] if want > 0 else []
            stats["rounds"] += 1
            if not drafts:
                tok = int(self.decode_step(torch.tensor([tok], device=self.device)))
                out.append(tok)
                continue
            logits = self.verify([tok] + drafts)
            target = logits.argmax(dim=-1).tolist()
            n = 0
            while n < len(drafts) and drafts[n] == target[n]:
                n += 1
            self.commit_verified(n + 1)
            proposer.note_accepted(drafts[:n])
            out.extend(drafts[:n])
            tok = int(target[n])
            out.append(tok)
            stats["verify_rounds"] += 1
            stats["proposed"] += len(drafts)
            stats["accepted"] += n
        return out[:steps + 1], stats

    def check_errors(self):
        word = int(self.err[0].item())
        if word:
            raise _lib.NanoKVError("Qwen3SparseModel", _lib.NKV_ERR_DEVICE, f"kernel error word {word}")


class DecodeLoop:
    """Greedy decode of a ``Qwen3SparseModel`` replayed from one CUDA graph.

    One replay = one token: embedding of the current token, the 36 layers (each
    with its sparse runtime's decode step), final norm, LM head, argmax, and the
    argmax fed back as the next input; the token is also appended to a device
    history and the position advanced, so nothing returns to the host between
    tokens.  Every layer's runtime must be a graph-replayable ``M12LayerRuntime``
    that has decoded once eagerly (``DeviceRingHeads``' conditions).
    """

    def __init__(self, model: Qwen3SparseModel, token: torch.Tensor, max_steps: int = 4096,
                 record_ids: bool = False):
        from .decode_graph import DeviceRingHeads

        self.model = m = model
        dev = m.device
        self.tok = token.view(1).to(dev).clone()
        self.pos = torch.full((1,), m.position, dtype=torch.int64, device=dev)
        self.hist = torch.zeros(max_steps, dtype=torch.int64, device=dev)
        self.count = torch.zeros(1, dtype=torch.int64, device=dev)
        self.max_steps = max_steps
        self.heads = DeviceRingHeads(m.runtimes)
        # with record_ids, every replay also stores each layer's selected block
        # ids and its decode query: ids_hist[layer][step] (the layer's device id
        # buffer after its decode in that replay), q_hist[layer][step]
        self.ids_hist = self.q_hist = None
        if record_ids:
            self.ids_hist = [torch.zeros(max_steps, rt._ids_view.numel(), dtype=torch.int64, device=dev)
                             for rt in m.runtimes]
            self.q_hist = [torch.zeros(max_steps, m.arch.num_heads, m.arch.head_dim, dtype=torch.bfloat16,
                                       device=dev) for _ in m.runtimes]
            m.decode_queries = [None] * len(m.runtimes)
        self.stream = torch.cuda.Stream(dev)
        self.stream.wait_stream(torch.cuda.current_stream(dev))
        self.graph = torch.cuda.CUDAGraph()
        with torch.inference_mode(), torch.cuda.stream(self.stream):
            with self.heads.recording(), torch.cuda.graph(self.graph, stream=self.stream):
                hidden = m.forward(self.tok, self.pos, "decode")
                nxt = m.logits(hidden).argmax(dim=-1)
                self.tok.copy_(nxt)
                self.hist.index_copy_(0, self.count, nxt)
                if self.ids_hist is not None:
                    for buf, rt in zip(self.ids_hist, m.runtimes):
                        buf.index_copy_(0, self.count, rt._ids_view.view(1, -1))
                    for buf, q in zip(self.q_hist, m.decode_queries):
                        buf.index_copy_(0, self.count, q)
                    m.decode_queries = None
                self.pos.add_(1)
                self.count.add_(1)
        self.steps_done = 0

    def replay(self):
        if self.steps_done >= self.max_steps:
            raise RuntimeError("DecodeLoop history is full")
        self.heads.before_replay()
        self.graph.replay()
        self.heads.after_replay()
        self.steps_done += 1
        self.model.position += 1

    def run(self, steps: int) -> list[int]:
        """``steps`` replays; returns the tokens they produced."""
        start = self.steps_done
        cur = torch.cuda.current_stream(self.model.device)
        self.stream.wait_stream(cur)
        with torch.cuda.stream(self.stream):
            for _ in range(steps):
                self.replay()
        cur.wait_stream(self.stream)
        return [int(t) for t in self.hist[start:self.steps_done].tolist()]

    def close(self):
        self.graph = None
