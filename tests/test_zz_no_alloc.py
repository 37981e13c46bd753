"""nkv_attend_static (workspace = scratch inside the library) against nkv_attend
(workspace from the caller), on the GPU.

Both run the same kernels on the same arguments; the outputs must agree within
the GPU parity tolerance (max-abs 2e-2 / rel 1e-2) on two calls in a row, for
the single-query decode kernel with either split merge and for the multi-query
kernel, and the scratch form's output agrees with the fp32 oracle's attention
over the same keys (selected blocks, sink, ring slice, current tokens).  A call
whose workspace would not fit the scratch is refused, and an
error the kernels record in the scratch (here: a block id outside the store,
which the kernels' bounds check replaces by block 0 and reports) is readable
through nkv_attend_static_check.
"""
import ctypes as C
import os

import pytest
import torch

from helpers import orc, pkg

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-2, 1e-2
DEV = "cuda"


def _layer(nkv, seed):
    """A layer runtime with 8192 stored tokens (bf16 block store in HBM)."""
    rt = nkv.M12LayerRuntime(0, nkv.M12Config(max_model_len=16384, device=DEV))
    g = torch.Generator(device=DEV).manual_seed(seed)
    for c in range(4):
        k = torch.randn(2048, 8, 128, generator=g, device=DEV).bfloat16()
        v = torch.randn(2048, 8, 128, generator=g, device=DEV).bfloat16()
        if c == 0:
            rt.prefill_first(None, k, v)
        else:
            rt._store_kv(k, v)
    torch.cuda.synchronize()
    return rt


def _attend_args(nkv, rt, nq, seed):
    """Run rt._attend once through nkv_attend; return its output, a copy of its
    args and the input tensors those args point into (keep them alive)."""
    g = torch.Generator(device=DEV).manual_seed(seed)
    q = torch.randn(nq, 32, 128, generator=g, device=DEV).bfloat16()
    kc = torch.randn(nq, 8, 128, generator=g, device=DEV).bfloat16()
    vc = torch.randn(nq, 8, 128, generator=g, device=DEV).bfloat16()
    n_sel = 32
    ids = torch.randperm(rt.nblocks_filled, generator=torch.Generator().manual_seed(seed))[:n_sel]
    ids = ids.to(DEV)
    captured = []
    orig = nkv.m12_runtime.call

    def spy(name, stream, argp):
        if name == "nkv_attend":
            captured.append(nkv._lib.AttendArgs.from_buffer_copy(argp._obj))
        return orig(name, stream, argp)

    nkv.m12_runtime.call = spy
    try:
        out = rt._attend(q, ids, n_sel, 64, 0, 300, kc, vc)  # no ring write: calls are repeatable
    finally:
        nkv.m12_runtime.call = orig
    torch.cuda.synchronize()
    assert len(captured) == 1
    return out, captured[0], (q, kc, vc, ids)


def _static(nkv, args, like):
    lib = nkv._lib.load()
    out = torch.full_like(like, float("nan"))
    b = nkv._lib.AttendArgs.from_buffer_copy(args)
    b.out = out.data_ptr()
    b.workspace, b.workspace_bytes = None, 0
    rc = lib.nkv_attend_static(torch.cuda.current_stream().cuda_stream, C.byref(b))
    assert rc == 0, lib.nkv_last_error().decode()
    return out


@pytest.mark.parametrize("nq,merge", [(1, "1"), (1, "0"), (3, "1")])
def test_static_scratch_matches_caller_workspace(nq, merge):
    nkv = pkg()
    old = os.environ.get("NKV_ATTEND_MERGE")
    nkv._lib.load()
    nkv._lib.set_env("NKV_ATTEND_MERGE", merge)
    try:
        rt = _layer(nkv, 5)
        ref, args, _keep = _attend_args(nkv, rt, nq, 11)
        for _ in range(2):  # two calls in a row: the scratch is reused
            got = _static(nkv, args, ref)
            torch.cuda.synchronize()
            torch.testing.assert_close(got.float().cpu(), ref.float().cpu(), atol=ATOL, rtol=RTOL)
        # the caller-workspace path is unaffected by the static calls
        lib = nkv._lib.load()
        out = torch.full_like(ref, float("nan"))
        b = nkv._lib.AttendArgs.from_buffer_copy(args)
        b.out = out.data_ptr()
        assert lib.nkv_attend(torch.cuda.current_stream().cuda_stream, C.byref(b)) == 0
        torch.cuda.synchronize()
        torch.testing.assert_close(out.float().cpu(), ref.float().cpu(), atol=ATOL, rtol=RTOL)
    finally:
        nkv._lib.set_env("NKV_ATTEND_MERGE", old)


def test_static_scratch_rejects_oversize():
    nkv = pkg()
    rt = _layer(nkv, 6)
    _, args, _keep = _attend_args(nkv, rt, 1, 12)
    lib = nkv._lib.load()
    b = nkv._lib.AttendArgs.from_buffer_copy(args)
    b.n_sel = 1 << 16  # 4M keys: a workspace far beyond the scratch
    need = lib.nkv_attend_workspace_bytes(8, 32, 1, b.n_sel * 64 + 64 + 300 + 1)
    assert need > (8 << 20)
    rc = lib.nkv_attend_static(torch.cuda.current_stream().cuda_stream, C.byref(b))
    assert rc == nkv._lib.NKV_ERR_ARG
    assert "static scratch" in lib.nkv_last_error().decode()


def test_static_scratch_error_word_is_readable():
    nkv = pkg()
    rt = _layer(nkv, 7)
    ref, args, keep = _attend_args(nkv, rt, 1, 13)
    lib = nkv._lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    _static(nkv, args, ref)
    assert lib.nkv_attend_static_check(stream) == 0, lib.nkv_last_error().decode()
    # slot 3 names a block beyond the store's capacity: the kernel's id check
    # records the error and loads block 0 in its place
    bad_ids = keep[3].clone()
    bad_ids[3] = rt.cpu_blocks_cap + 7
    b = nkv._lib.AttendArgs.from_buffer_copy(args)
    b.block_ids = bad_ids.data_ptr()
    out = torch.empty_like(ref)
    b.out = out.data_ptr()
    b.workspace, b.workspace_bytes = None, 0
    assert lib.nkv_attend_static(stream, C.byref(b)) == 0, lib.nkv_last_error().decode()
    assert lib.nkv_attend_static_check(stream) == nkv._lib.NKV_ERR_DEVICE
    assert "out of range" in lib.nkv_last_error().decode()
    # reading the word cleared it
    assert lib.nkv_attend_static_check(stream) == 0
    # and the next good call reports nothing
    got = _static(nkv, args, ref)
    assert lib.nkv_attend_static_check(stream) == 0
    torch.testing.assert_close(got.float().cpu(), ref.float().cpu(), atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("nq", [1, 3])
def test_static_scratch_matches_oracle(nq):
    """The scratch form against the CPU oracle directly: the keys the call
    attends (its selected blocks read back from the block store, the sink, the
    ring slice and the current tokens, causal among themselves) packed in the
    reference's order and attended in fp32."""
    nkv = pkg()
    rt = _layer(nkv, 8)
    ref, args, (q, kc, vc, ids) = _attend_args(nkv, rt, nq, 14)
    for _ in range(2):
        got = _static(nkv, args, ref)
        torch.cuda.synchronize()
    hist_k = rt.k_cpu[ids.cpu()].reshape(-1, 8, 128).cpu()     # [n_sel * 64, Hkv, D]
    hist_v = rt.v_cpu[ids.cpu()].reshape(-1, 8, 128).cpu()
    ring_k = rt._ring_k.permute(1, 0, 2)[:300].cpu()           # physical slots [0, 300)
    ring_v = rt._ring_v.permute(1, 0, 2)[:300].cpu()
    kp = torch.cat([hist_k, rt._sink_k.permute(1, 0, 2)[:64].cpu(), ring_k, kc.cpu()])
    vp = torch.cat([hist_v, rt._sink_v.permute(1, 0, 2)[:64].cpu(), ring_v, vc.cpu()])
    want = orc.attention(q.cpu(), kp, vp, rt.cfg.scale, causal_from=kp.shape[0] - nq)
    torch.testing.assert_close(got.float().cpu(), want, atol=ATOL, rtol=RTOL)
