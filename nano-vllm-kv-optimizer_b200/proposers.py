"""Draft proposers for the speculative loop of ``Qwen3SparseModel.speculative_generate``.

The loop needs three calls from a proposer (the reference's interface,
``nanovllm/sparse/proposers.py``):

    prefill(prompt_ids)            # state for a new prompt (a list of token ids)
    propose(last_token, k, pos)    # up to k candidate tokens after last_token at position pos
    note_accepted(tokens)          # the drafts the target accepted in this round

* ``NgramProposer``: no model; continues the context by the most frequent
  continuation of its last n tokens seen earlier in the context (prompt
  lookup).
* ``DraftModelProposer``: a small Qwen3-architecture draft model
  (``StaticDraftModel``) whose one-token step runs over a static window of
  keys and values and is replayed from a CUDA graph, as the reference's
  ``StaticDraft`` (static_draft.py) does.  Its weights are random (seeded):
  there are no checkpoints here.
"""
from __future__ import annotations

import math
from collections import Counter
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from . import _lib
from ._lib import call
from .qwen3_harness import Qwen3Arch, rope_cos_sin


class NgramProposer:
    """Prompt-lookup drafter: after the context's last n tokens, propose what
    most often followed the same n tokens earlier in the context, token by
    token, up to ``max_k`` (reference proposers.py: ``NgramProposer``)."""

    def __init__(self, n: int = 4, max_k: int = 8):
        self.n, self.max_k = int(n), int(max_k)
        self.context: list[int] = []
        self.follow: dict[tuple, Counter] = {}
        self._indexed = 0  # context positions whose n-gram is in the index

    def reset(self) -> None:
        self.context, self.follow, self._indexed = [], {}, 0

    def _index(self) -> None:
        # every n-gram that has a following token, from where indexing stopped
        n, ctx = self.n, self.context
        for i in range(self._indexed, len(ctx) - n):
            self.follow.setdefault(tuple(ctx[i:i + n]), Counter())[ctx[i + n]] += 1
        self._indexed = max(self._indexed, len(ctx) - n)

    def prefill(self, prompt_ids) -> None:
        self.reset()
        self.context = [int(t) for t in prompt_ids]
        self._index()

    def note_accepted(self, tokens) -> None:
        self.context.extend(int(t) for t in tokens)
        self._index()

    def propose(self, last_token: int, k: int, pos: int) -> list[int]:
        k = min(int(k), self.max_k)
        if len(self.context) < self.n:
            return []
        if self.context[-1] != int(last_token):
            self.note_accepted([last_token])  # the current token belongs to the context
        out: list[int] = []
        tail = self.context[-self.n:]
        for _ in range(k):
            c = self.follow.get(tuple(tail))
            if not c:
                break
            # the most frequent continuation; ties go to the one seen first
            best = max(c.items(), key=lambda kv: kv[1])[0]
            out.append(best)
            tail = tail[1:] + [best]
        return out


@dataclass
class DraftArch:
    """A Qwen3-0.6B-like draft (the reference's default draft model)."""

    vocab_size: int = 151936
    hidden_size: int = 1024
    num_layers: int = 28
    num_heads: int = 16
    num_kv_heads: int = 8
    head_dim: int = 128
    intermediate_size: int = 3072
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1e6
    max_position: int = 131072 + 2048


class StaticDraftModel:
    """Draft decoder with a static key/value window of ``window`` slots per
    layer (slot = position % window) and a one-token step whose buffers never
    move, so that it is captured once in a CUDA graph and replayed per token.

    A slot is visible to the query at position p iff the position it holds
    lies in (p - window, p].  Norms, the q/k RMSNorm + RoPE and SwiGLU are this
    package's kernels; the window attention and projections are torch ops (the
    draft is not the sparse path)."""

    def __init__(self, arch: DraftArch, window: int = 2048, device="cuda", seed: int = 1,
                 init_std: float = 0.02):
        _lib.load()
        self.arch = a = arch
        dev = torch.device(device)
        if dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        self.device, self.window = dev, int(window)
        g = torch.Generator(device=dev).manual_seed(seed)

        def w(*shape):
            t = torch.empty(*shape, dtype=torch.bfloat16, device=dev)
            t.normal_(0.0, init_std, generator=g)
            return t
        H, D = a.hidden_size, a.head_dim
        self.q_size, self.kv_size = a.num_heads * D, a.num_kv_heads * D
        self.embed = w(a.vocab_size, H)
        self.wqkv = [w(self.q_size + 2 * self.kv_size, H) for _ in range(a.num_layers)]
        self.wo = [w(H, self.q_size) for _ in range(a.num_layers)]
        self.wgu = [w(2 * a.intermediate_size, H) for _ in range(a.num_layers)]
        self.wd = [w(H, a.intermediate_size) for _ in range(a.num_layers)]
        self.ones_h = torch.ones(H, dtype=torch.bfloat16, device=dev)
        self.ones_d = torch.ones(D, dtype=torch.bfloat16, device=dev)
        rope_arch = Qwen3Arch(vocab_size=a.vocab_size, hidden_size=H, num_layers=a.num_layers,
                              num_heads=a.num_heads, num_kv_heads=a.num_kv_heads, head_dim=D,
                              intermediate_size=a.intermediate_size, rms_norm_eps=a.rms_norm_eps,
                              rope_theta=a.rope_theta, rope_scaling=None, max_position=a.max_position)
        self.cos_sin = rope_cos_sin(rope_arch, dev)
        W = self.window
        self.kcache = torch.zeros(a.num_layers, W, a.num_kv_heads, D, dtype=torch.bfloat16, device=dev)
        self.vcache = torch.zeros_like(self.kcache)
        self.slot_pos = torch.full((W,), -1, dtype=torch.int64, device=dev)
        self.in_id = torch.zeros(1, dtype=torch.int64, device=dev)
        self.in_pos = torch.zeros(1, dtype=torch.int64, device=dev)
        self.out_logits = torch.empty(1, a.vocab_size, dtype=torch.bfloat16, device=dev)
        self.err = torch.zeros(4, dtype=torch.int32, device=dev)
        self.graph = None

    def _stream(self) -> int:
        return torch.cuda.current_stream(self.device).cuda_stream

    def _norm(self, x, residual, out, has_residual):
        T, H = x.shape
        call("nkv_add_rms_norm", self._stream(), x.data_ptr(), residual.data_ptr(), self.ones_h.data_ptr(),
             out.data_ptr(), T, H, self.arch.rms_norm_eps, 1 if has_residual else 0)

    def _forward(self, ids: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
        """Hidden states after the final norm for T tokens at positions pos
        (consecutive); their keys and values are written into the window
        first, so each token sees itself and the earlier window."""
        a = self.arch
        T, W, D, G = ids.shape[0], self.window, a.head_dim, a.num_heads // a.num_kv_heads
        slots = torch.remainder(pos, W)
        self.slot_pos.index_copy_(0, slots, pos)
        sp = self.slot_pos.view(1, W)
        visible = (sp >= 0) & (sp <= pos.view(T, 1)) & (sp > pos.view(T, 1) - W)  # [T, W]
        bias = torch.zeros(T, W, dtype=torch.float32, device=self.device).masked_fill_(~visible, float("-inf"))
        h = F.embedding(ids, self.embed)
        residual = torch.empty_like(h)
        xn = torch.empty_like(h)
        scale = 1.0 / math.sqrt(D)
        for l in range(a.num_layers):
            self._norm(h, residual, xn, has_residual=l > 0)
            qkv = F.linear(xn, self.wqkv[l])
            call("nkv_qk_norm_rope", self._stream(), qkv.data_ptr(), qkv.stride(0), T, a.num_heads, a.num_kv_heads,
                 D, self.ones_d.data_ptr(), self.ones_d.data_ptr(), self.cos_sin.data_ptr(), pos.data_ptr(),
                 self.cos_sin.shape[0], a.rms_norm_eps, self.err.data_ptr())
            q = qkv[:, :self.q_size].view(T, a.num_kv_heads, G, D)
            self.kcache[l].index_copy_(0, slots, qkv[:, self.q_size:self.q_size + self.kv_size].view(T, -1, D))
            self.vcache[l].index_copy_(0, slots, qkv[:, self.q_size + self.kv_size:].view(T, -1, D))
            s = torch.einsum("thgd,whd->thgw", q.float(), self.kcache[l].float()) * scale
            p = torch.softmax(s + bias.view(T, 1, 1, W), dim=-1)
            o = torch.einsum("thgw,whd->thgd", p, self.vcache[l].float()).to(torch.bfloat16)
            h = F.linear(o.reshape(T, self.q_size), self.wo[l])
            self._norm(h, residual, xn, has_residual=True)
            gu = F.linear(xn, self.wgu[l])
            act = torch.empty(T, a.intermediate_size, dtype=torch.bfloat16, device=self.device)
            call("nkv_silu_mul", self._stream(), gu.data_ptr(), act.data_ptr(), T, a.intermediate_size)
            h = F.linear(act, self.wd[l])
        out = torch.empty_like(h)
        self._norm(h, residual, out, has_residual=True)
        return out

    @torch.inference_mode()
    def prefill(self, prompt_ids, chunk: int = 256) -> None:
        """The prompt's last ``window`` tokens into the window (chunked), then
        the step is captured once."""
        ids = torch.as_tensor(prompt_ids, dtype=torch.int64).view(-1).to(self.device)
        n = ids.numel()
        self.kcache.zero_()
        self.vcache.zero_()
        self.slot_pos.fill_(-1)
        for s in range(max(0, n - self.window), n, chunk):
            e = min(n, s + chunk)
            self._forward(ids[s:e], torch.arange(s, e, dtype=torch.int64, device=self.device))
        if self.graph is None:
            self._capture()

    def _capture(self) -> None:
        keep = (self.kcache.clone(), self.vcache.clone(), self.slot_pos.clone())
        stream = torch.cuda.Stream(self.device)
        stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(stream):
            for _ in range(2):  # warm-up outside the capture
                self.out_logits.copy_(F.linear(self._forward(self.in_id, self.in_pos), self.embed))
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph, stream=stream):
                self.out_logits.copy_(F.linear(self._forward(self.in_id, self.in_pos), self.embed))
        torch.cuda.current_stream(self.device).wait_stream(stream)
        # the warm-up and capture steps wrote one slot: put the window back
        self.kcache.copy_(keep[0])
        self.vcache.copy_(keep[1])
        self.slot_pos.copy_(keep[2])

    @torch.inference_mode()
    def step(self, token: int, pos: int) -> torch.Tensor:
        """Logits [1, vocab] after ``token`` at absolute position ``pos``."""
        if not 0 <= int(pos) < self.cos_sin.shape[0]:
            raise _lib.NanoKVError("StaticDraftModel.step", _lib.NKV_ERR_ARG, f"position {pos} outside the RoPE table")
        self.in_id.fill_(int(token))
        self.in_pos.fill_(int(pos))
        if self.graph is not None:
            self.graph.replay()
        else:
            self.out_logits.copy_(F.linear(self._forward(self.in_id, self.in_pos), self.embed))
        return self.out_logits


class DraftModelProposer:
    """Greedy proposals from a ``StaticDraftModel``: feed the current token at
    its position, then each proposal at the next (reference proposers.py:
    ``DraftModelProposer`` over ``StaticDraftRunner``).  The draft needs no
    rollback: a slot holding a rejected proposal is overwritten when its
    position comes round again, and positions above the query are masked."""

    def __init__(self, draft: StaticDraftModel):
        self.draft = draft

    def reset(self) -> None:
        pass

    def prefill(self, prompt_ids) -> None:
        self.draft.prefill(prompt_ids)

    def note_accepted(self, tokens) -> None:
        pass

    def propose(self, last_token: int, k: int, pos: int) -> list[int]:
        out: list[int] = []
        tok = int(last_token)
        for i in range(int(k)):
            tok = int(self.draft.step(tok, pos + i).argmax(dim=-1))
            out.append(tok)
        return out
