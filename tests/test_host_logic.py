"""CPU tests: the C ABI library loads and exports every declared symbol, and the
host-side logic of the runtime follows the reference's semantics."""
import os
import random
import re

import pytest
import torch

from helpers import ROOT, orc, pkg


def _declared_functions():
    text = open(os.path.join(ROOT, "include", "nanokv.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(nkv_[a-z_0-9]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    nkv = pkg()
    lib = nkv._lib.load()
    names = _declared_functions()
    assert len(names) >= 14
    for name in names:
        assert hasattr(lib, name), name
        assert name in nkv._lib.SIGNATURES, f"{name} has no ctypes signature"
    assert lib.nkv_version() >= 1


def test_workspace_queries_are_host_only():
    lib = pkg()._lib.load()
    assert lib.nkv_select_workspace_bytes(2048, 1) >= 2048 * 4
    assert lib.nkv_attend_workspace_bytes(8, 32, 1, 2624) > 0


def test_static_scratch_limit_at_reference_geometry():
    """The largest key count nkv_attend_static takes at hkv 8 / hq 32 / one
    query is the one the header states (8048 keys)."""
    lib = pkg()._lib.load()
    cap = 8 << 20
    assert lib.nkv_attend_workspace_bytes(8, 32, 1, 8048) <= cap
    assert lib.nkv_attend_workspace_bytes(8, 32, 1, 8049) > cap
    assert lib.nkv_attend_workspace_bytes(8, 32, 1, 116 * 64 + 64 + 512 + 1) <= cap


def test_argument_errors_need_no_gpu():
    nkv = pkg()
    lib = nkv._lib
    with pytest.raises(lib.NanoKVUnsupported):
        lib.call("nkv_select", None, 1, 1, 0, 0, 32, 8, 64, 1, 4, 16, 8, None, 0, 4,
                 1, None, None, 1, 1 << 20)
    with pytest.raises(lib.NanoKVError):
        lib.call("nkv_select", None, 0, 1, 0, 0, 32, 8, 128, 0, 4, 16, 8, None, 0, 4,
                 1, None, None, 1, 1 << 20)
    a = lib.AttendArgs()
    a.head_dim, a.hq, a.hkv, a.nq = 128, 32, 8, 1
    with pytest.raises(lib.NanoKVError):
        import ctypes
        lib.call("nkv_attend", None, ctypes.byref(a))


# ----------------------------------------------------------------------------
# recent ring vs the reference's left-aligned shifting window
# ----------------------------------------------------------------------------
class LeftAligned:
    """The reference's recent buffer (m12_runtime.py:488-503, 788-802, 1169-1172)."""

    def __init__(self, R):
        self.R, self.buf, self.valid = R, [None] * R, 0

    def append(self, toks):
        R, T = self.R, len(toks)
        new_len = min(R, self.valid + T)
        if T >= new_len:
            self.buf[:new_len] = toks[T - new_len:]
        else:
            carry, old_len = new_len - T, min(R, self.valid)
            self.buf[:carry] = self.buf[old_len - carry:old_len]
            self.buf[carry:new_len] = toks
        self.valid += T

    def decode(self, tok):
        self.buf = self.buf[1:] + [tok]
        rlen = min(self.R, self.valid + 1)
        window = self.buf[self.R - rlen:]
        self.valid += 1
        return window

    def prefill_slice(self, sink):
        _, off, n = orc.recent_slice(self.valid, sink, self.R)
        return self.buf[off:off + n]


class Ring:
    """The runtime's ring arithmetic, applied to a Python list."""

    def __init__(self, R):
        self.nkv = pkg().m12_runtime
        self.R, self.ring, self.head, self.valid = R, [None] * R, 0, 0

    def append(self, toks):
        pos0, first, new_head = self.nkv.ring_append_plan(self.head, self.valid, len(toks), self.R)
        for i in range(first, len(toks)):
            self.ring[(pos0 + i) % self.R] = toks[i]
        self.head, self.valid = new_head, self.valid + len(toks)

    def decode(self, tok):
        w, start, n, new_head = self.nkv.ring_decode_plan(self.head, self.valid, self.R)
        window = [self.ring[(start + j) % self.R] for j in range(n)] + [tok]
        self.ring[w] = tok
        self.head, self.valid = new_head, self.valid + 1
        return window

    def prefill_slice(self, sink):
        _, off, n = orc.recent_slice(self.valid, sink, self.R)
        s = self.nkv.ring_slice_start(self.head, off, self.R)
        return [self.ring[(s + j) % self.R] for j in range(n)]


@pytest.mark.parametrize("seed", range(12))
def test_ring_matches_left_aligned_window(seed):
    rnd = random.Random(seed)
    R = rnd.choice([1, 2, 5, 8, 64, 512])
    sink = rnd.choice([0, 2, 64])
    ref, ring = LeftAligned(R), Ring(R)
    counter = 0
    for _ in range(60):
        op = rnd.random()
        if op < 0.35:
            T = rnd.choice([1, 2, 3, R - 1, R, R + 3, 2 * R + 1])
            T = max(1, T)
            toks = list(range(counter, counter + T))
            counter += T
            ref.append(toks)
            ring.append(toks)
        else:
            assert ref.decode(counter) == ring.decode(counter)
            counter += 1
        assert ref.prefill_slice(sink) == ring.prefill_slice(sink)


# ----------------------------------------------------------------------------
# helpers and config with the reference's semantics
# ----------------------------------------------------------------------------
def test_recent_slice_and_dynamic_budget():
    nkv = pkg()
    assert nkv.prefill_recent_slice(4096, 64, 512) == (3584, 0, 512)
    assert nkv.prefill_recent_slice(128, 64, 512) == (0, 64, 64)
    assert nkv.prefill_recent_slice(64, 64, 512) == (0, 64, 0)
    for v in range(0, 700, 7):
        assert nkv.prefill_recent_slice(v, 64, 512) == orc.recent_slice(v, 64, 512)
    f = nkv.dynamic_top_k_from_scores
    assert f(torch.ones(32), 32, 0.90) == 32
    assert f(torch.arange(10, 0, -1).float(), 32, 0.90) == 10
    assert f(torch.tensor([float("inf")] + [0.0] * 31), 32, 0.90) == 32
    assert f(torch.tensor([10.0] + [0.0] * 31), 32, 0.90) == 16


def test_host_query_summaries_match_oracle():
    nkv = pkg()
    q = torch.randn(10, 4, 8)
    for n in (1, 3, 4, 10, 20):
        torch.testing.assert_close(nkv.prefill_query_summaries(q, n), orc.query_summaries(q, n))


@pytest.mark.parametrize("kw", [
    dict(decode_kv_pipeline=True, use_index_select=False),
    dict(prefill_top_k_blocks=0), dict(decode_top_k_blocks=33),
    dict(decode_relative_a=1.5), dict(decode_relative_a=0.5, decode_relative_max_blocks=0),
    dict(decode_query_window=0), dict(fused_dequant=True),
    dict(kv_residency="disk"), dict(quant_scheme="x"), dict(prefill_attention_backend="x"),
])
def test_config_validation_errors(kw):
    with pytest.raises(ValueError):
        pkg().M12Config(**kw)
