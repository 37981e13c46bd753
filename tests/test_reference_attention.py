"""The reference's own Attention.forward driving this package's runtime.

The reference installs its sparse runtime on each attention layer
(``model_runner.py:183``: ``attn.sparse_rt = M12LayerRuntime(...)``) and
``Attention.forward`` (``nanovllm/layers/attention.py:64-99``) dispatches on the
global context: a later prefill chunk to ``prefill_chunk``, a decode token to
``decode``, a verify pass (``verify_mode``) to ``verify_tokens``.  Here the
reference's unmodified module (installed under ``baseline/_ref``) gets this
package's ``M12LayerRuntime`` as its ``sparse_rt``, and every output it
returns is checked against the oracle on the same inputs (selected ids equal
modulo 1e-3 score ties, outputs within max-abs 2e-2 / rel 1e-2).  The first
chunk is stored directly: its dense attention is the caller's FA2 call, not
part of the sparse path.  Skipped when the reference is not installed.
"""
import sys

import pytest
import torch

from helpers import ids_match_modulo_ties, orc, pkg, qkv
from oracle import ref_shim

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-2, 1e-2
DEV = "cuda"


def _reference_attention():
    if not ref_shim.reference_available():
        pytest.skip("the reference is not installed under baseline/_ref")
    if ref_shim.REFERENCE_ROOT not in sys.path:
        sys.path.insert(0, ref_shim.REFERENCE_ROOT)
    try:
        from nanovllm.layers.attention import Attention
        from nanovllm.utils.context import reset_context, set_context
    except ImportError as e:  # its imports (triton, flash_attn) are part of the image
        pytest.skip(f"reference attention module not importable: {e}")
    return Attention, set_context, reset_context


def _close(got, want):
    torch.testing.assert_close(got.float().cpu(), want.float().cpu(), atol=ATOL, rtol=RTOL)


def test_reference_attention_forward_drives_this_runtime():
    Attention, set_context, reset_context = _reference_attention()
    nkv = pkg()
    g = torch.Generator().manual_seed(1234)
    cfg = nkv.M12Config(max_model_len=16384, device=DEV)
    rt = nkv.M12LayerRuntime(0, cfg)
    attn = Attention(32, 128, cfg.scale, 8)
    attn.sparse_rt = rt
    layer = orc.OracleLayer(orc.OracleConfig())
    try:
        # history: two chunks stored (the first chunk's dense attention is the caller's)
        _, k, v = qkv(g, 4096)
        rt.prefill_first(None, k.to(DEV), v.to(DEV))
        layer.store(k, v)
        # a later prefill chunk through Attention.forward -> prefill_chunk
        q, k, v = qkv(g, 2048)
        set_context(True, max_seqlen_q=2048, max_seqlen_k=2048)
        o = attn(q.to(DEV), k.to(DEV), v.to(DEV))
        layer.force_ids = rt.last_prefill_block_ids.cpu()
        _close(o, layer.prefill_chunk(q, k, v))
        # decode tokens -> decode
        set_context(False)
        for _ in range(3):
            q, k, v = qkv(g, 1)
            o = attn(q.to(DEV), k.to(DEV), v.to(DEV))
            layer.force_ids = rt.last_block_ids
            want = layer.decode(q, k, v)
            ok, why = ids_match_modulo_ties(rt.last_block_ids, layer.own_ids, layer.last_scores)
            assert ok, why
            _close(o, want)
        # a verify pass over [current + 4 drafts] (verify_mode) -> verify_tokens, then commit 3
        rt.verify_mode = True
        q, k, v = qkv(g, 5)
        o = attn(q.to(DEV), k.to(DEV), v.to(DEV))
        rt.verify_mode = False
        layer.force_ids = rt.last_verify_block_ids
        _close(o, layer.verify(q, k, v, lossless=False))
        rt.commit_verified(3)
        layer.commit(3)
        assert rt.valid_len == layer.valid_len
        # the next decode sees the committed tokens in the recent window
        q, k, v = qkv(g, 1)
        o = attn(q.to(DEV), k.to(DEV), v.to(DEV))
        layer.force_ids = rt.last_block_ids
        _close(o, layer.decode(q, k, v))
    finally:
        reset_context()
