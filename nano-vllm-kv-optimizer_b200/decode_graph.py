"""Decode steps of sparse layers replayed from a CUDA graph.

The reference's model runner captures its dense decode step in CUDA graphs
(``nanovllm/engine/model_runner.py:458-475``) but runs the sparse decode
eagerly (``nanovllm/config.py:180``), so every layer pays its host launch cost
on every token.  Here the decode of a layer can be recorded in a CUDA graph
and replayed per token:

* the inputs are fixed device tensors (a model's qkv projection output
  buffers); the caller writes each token's q/k/v into them before a replay;
* the outputs are fixed device tensors, overwritten by every replay;
* the recent window's head lives on the device (``nkv_decode_args.ring_head``),
  so each replay appends its token one slot further, exactly as the eager
  ``decode`` would; the host-side state (``valid_len``, ring head, last ids)
  advances with every replay, so eager calls can be mixed in between.

A layer qualifies once its recent window is full (``valid_len >=
recent_tokens - 1`` and ``>= sink_tokens``: the attended window then has a
fixed length), it uses the single-call decode (no relative threshold,
dynamic budget, gather sort or query window), it records neither ids nor
queries, and it has run one eager ``decode`` (which sets up its workspaces
and kernel attributes outside the capture).  The non-finite output check
(``check_finite_outputs``) needs a host synchronisation and is not recorded.
A change of a layer's history (another prefill chunk, ``reset``) makes the
recording invalid: the next replay raises.

``DeviceRingHeads`` is the part a model runner uses to record the decode
calls inside its own graph of the whole model (layers interleaved with the
projections and MLPs); ``DecodeGraph`` is the stand-alone form for a stack of
attention layers.
"""
from __future__ import annotations

from contextlib import contextmanager

import torch

from .m12_runtime import M12LayerRuntime


class DeviceRingHeads:
    """Device-resident recent-window heads for a set of layers' decode calls.

    ``recording()`` wraps a CUDA graph capture that contains one ``decode``
    call per layer (in any order, with any other work between them): inside
    it the layers' decode steps read and advance the head on the device
    (``nkv_decode_args.ring_head``), and the host state the capture moved is
    put back afterwards.  Around every replay of that graph call
    ``before_replay()`` (re-uploads the heads when eager calls moved a
    window, raises when a layer's history changed) and ``after_replay()``
    (advances each layer's host state by one token).  Replays and eager calls
    go to the same stream.
    """

    def __init__(self, layers: list[M12LayerRuntime]):
        assert len(layers) > 0
        dev = layers[0].device
        for rt in layers:
            cfg = rt.cfg
            assert rt.device == dev, "all layers on one device"
            assert rt._fast_ok and not rt.record_q and not rt.record_ids, \
                "graph replay needs the single-call decode without id or query recording"
            assert rt._k_store is not None and rt._dargs is not None, \
                "run one eager decode on every layer before recording"
            assert rt.valid_len + 1 >= cfg.recent_tokens and rt.valid_len >= cfg.sink_tokens, \
                "graph replay needs a full recent window (valid_len >= recent_tokens - 1)"
        self.layers = list(layers)
        self.device = dev
        # {head, arrivals} per layer: 8-byte aligned rows; arrivals start at 0
        self._ring = torch.zeros(len(layers), 2, dtype=torch.int32, device=dev)
        self._R = [rt.cfg.recent_tokens for rt in layers]
        self._nb = [rt.nblocks_filled for rt in layers]
        self._heads = [rt._ring_head for rt in layers]
        self._upload()

    def _upload(self):
        self._ring[:, 0].copy_(torch.tensor(self._heads, dtype=torch.int32))

    @contextmanager
    def recording(self, outputs=None):
        """``outputs[i]`` (optional): the [1, Hq, D] tensor layer i's recorded
        decode writes its output into, instead of a new tensor."""
        layers = self.layers
        saved = [(rt.valid_len, rt._ring_head, rt._last_ids_dev, rt._last_ids_host, rt.timings,
                  rt.cfg.check_finite_outputs) for rt in layers]
        try:
            for i, rt in enumerate(layers):
                rt._ring_dev_ptr = self._ring[i].data_ptr()
                rt.cfg.check_finite_outputs = False  # a host synchronisation: not recordable
                if outputs is not None:
                    o = outputs[i]
                    assert (o.is_contiguous() and o.dtype == torch.bfloat16 and o.device == rt.device
                            and tuple(o.shape) == (1, rt.cfg.num_heads, rt.cfg.head_dim))
                    rt._out_override = o
            yield self
        finally:
            for rt, sv in zip(layers, saved):
                rt._ring_dev_ptr = 0
                rt._out_override = None
                (rt.valid_len, rt._ring_head, rt._last_ids_dev, rt._last_ids_host, rt.timings,
                 rt.cfg.check_finite_outputs) = sv

    def before_replay(self):
        heads, stale = self._heads, False
        for i, rt in enumerate(self.layers):
            if rt.nblocks_filled != self._nb[i]:
                raise RuntimeError(f"layer {rt.layer_id}: history changed since the recording; "
                                   "record a new graph")
            if rt._ring_head != heads[i]:
                stale = True
        if stale:  # eager calls moved a window: the host state is the truth
            for i, rt in enumerate(self.layers):
                heads[i] = rt._ring_head
            self._upload()

    def after_replay(self):
        heads, R = self._heads, self._R
        for i, rt in enumerate(self.layers):
            h = heads[i] + 1
            if h == R[i]:
                h = 0
            heads[i] = rt._ring_head = h
            rt.valid_len += 1
            rt._last_ids_dev, rt._last_ids_host = rt._ids_view, None


class DecodeGraph:
    """One decode token through ``layers``, recorded once, replayed per token.

    ``inputs[i] = (q, k, v)`` are layer i's device inputs ([1, Hq, D],
    [1, Hkv, D], [1, Hkv, D] bf16), read by every replay.  ``outputs[i]`` is
    layer i's [1, Hq, D] output; with ``stack=True`` they are the rows of
    ``out`` ([L, 1, Hq, D]), which the layers' decode steps write directly.
    """

    def __init__(self, layers: list[M12LayerRuntime], inputs, stream: torch.cuda.Stream | None = None,
                 stack: bool = True):
        assert len(layers) == len(inputs)
        self.heads = DeviceRingHeads(layers)
        dev = self.heads.device
        for q, k, v in inputs:
            assert q.dtype == torch.bfloat16 and q.shape[0] == 1 and k.shape[0] == 1 and v.shape[0] == 1
            assert q.device == dev and k.device == dev and v.device == dev
        self.layers = self.heads.layers
        self.inputs = list(inputs)
        self.graph = torch.cuda.CUDAGraph()
        # stacked: every layer's decode writes its row of `out` directly
        self.out = None
        if stack:
            hq, d = layers[0].cfg.num_heads, layers[0].cfg.head_dim
            assert all(rt.cfg.num_heads == hq and rt.cfg.head_dim == d for rt in layers)
            self.out = torch.empty(len(layers), 1, hq, d, dtype=torch.bfloat16, device=dev)
        rows = list(self.out) if stack else None
        with self.heads.recording(rows), torch.cuda.graph(self.graph, stream=stream):
            self.outputs = [rt.decode(q, k, v, dev) for rt, (q, k, v) in zip(layers, inputs)]

    def replay(self):
        """Decode one token through every layer; returns ``out`` (or ``outputs``)."""
        self.heads.before_replay()
        self.graph.replay()
        self.heads.after_replay()
        return self.out if self.out is not None else self.outputs
