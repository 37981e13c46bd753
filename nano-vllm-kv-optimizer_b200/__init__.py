"""NanoKV block-sparse attention hot path, B200-native (sm_100a).

Drop-in for the reference's per-layer sparse runtime
(``nanovllm/sparse/m12_runtime.py``): ``M12Config`` / ``M12LayerRuntime`` with
the same methods, backed by hand-written CUDA kernels behind the C ABI in
``include/nanokv.h`` (``libnanokv.so``, built in-tree by ``build.py``).

The directory name is not a Python identifier; import it with
``importlib.import_module("nano-vllm-kv-optimizer_b200")``.
"""
from . import _lib
from .m12_runtime import (
    M12Config,
    M12LayerRuntime,
    dynamic_top_k_from_scores,
    prefill_query_summaries,
    prefill_recent_slice,
)
from .decode_graph import DecodeGraph, DeviceRingHeads
from .qwen3_harness import DecodeLoop, Qwen3Arch, Qwen3SparseModel
from .proposers import DraftArch, DraftModelProposer, NgramProposer, StaticDraftModel
from .segmented_prefill import SegmentedPrefillAdapter
from .sharded import KVHeadShardedLayer
from . import torch_ops  # registers torch.ops.nanokv.*

__all__ = [
    "DecodeGraph",
    "DecodeLoop",
    "DraftArch",
    "DraftModelProposer",
    "DeviceRingHeads",
    "KVHeadShardedLayer",
    "M12Config",
    "M12LayerRuntime",
    "NgramProposer",
    "Qwen3Arch",
    "Qwen3SparseModel",
    "SegmentedPrefillAdapter",
    "StaticDraftModel",
    "dynamic_top_k_from_scores",
    "prefill_query_summaries",
    "prefill_recent_slice",
]
