"""The dense-model kernels of the full-model harness against torch fp32
restatements of the reference's eager expressions (needs a B200).

nkv_qk_norm_rope: Qwen3Attention's q/k RMSNorm + rotary embedding
(reference nanovllm/models/qwen3.py:91-98, layers/layernorm.py:16-26,
layers/rotary_embedding.py:7-15); nkv_add_rms_norm: RMSNorm with and without
the residual add (layernorm.py:16-39); nkv_silu_mul: SiluAndMul
(activation.py:6-11).  Outputs are bf16 roundings of the same fp32 math; the
reductions sum in a different order, so a value may land one bf16 step away
(after the rotary embedding's subtraction such a step can be several ulps of
a small result): at least 99.5 % of elements identical, the rest within
max-abs 2e-2 / rel 8e-3.
"""
import pytest
import torch

from helpers import pkg

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _ulps(a, b):
    """Distance in bf16 steps between two bf16 tensors of the same sign pattern."""
    ai = a.view(torch.int16).int()
    bi = b.view(torch.int16).int()
    # map the sign-magnitude encoding to an ordered integer line
    ai = torch.where(ai < 0, -32768 - ai, ai)
    bi = torch.where(bi < 0, -32768 - bi, bi)
    return (ai - bi).abs()


def _check(got, want):
    d = _ulps(got.contiguous(), want.contiguous())
    assert float((d == 0).float().mean()) >= 0.995
    torch.testing.assert_close(got.float(), want.float(), atol=2e-2, rtol=8e-3)


def _ref_norm(x, w, eps):
    xf = x.float()
    var = xf.pow(2).mean(dim=-1, keepdim=True)
    xf = xf * torch.rsqrt(var + eps)
    return xf.to(torch.bfloat16) * w


def _ref_rope(x, cos, sin):
    x1, x2 = torch.chunk(x.float(), 2, dim=-1)
    return torch.cat((x1 * cos - x2 * sin, x2 * cos + x1 * sin), dim=-1).to(x.dtype)


@pytest.mark.parametrize("T", [1, 7, 4096])
def test_qk_norm_rope_matches_reference_math(T):
    nkv = pkg()
    from importlib import import_module
    h = import_module(nkv.__name__ + ".qwen3_harness")
    arch = h.Qwen3Arch()
    g = torch.Generator(device=DEV).manual_seed(T)
    hq, hkv, d = 32, 8, 128
    qkv = (torch.randn(T, (hq + 2 * hkv) * d, generator=g, device=DEV) * 1.7).bfloat16()
    qw = (1 + 0.1 * torch.randn(d, generator=g, device=DEV)).bfloat16()
    kw = (1 + 0.1 * torch.randn(d, generator=g, device=DEV)).bfloat16()
    cs = h.rope_cos_sin(arch, DEV, max_position=40000)
    pos = torch.randint(0, 40000, (T,), generator=g, device=DEV)
    q = qkv[:, :hq * d].view(T, hq, d)
    k = qkv[:, hq * d:(hq + hkv) * d].view(T, hkv, d)
    cos, sin = cs[pos].chunk(2, dim=-1)
    want_q = _ref_rope(_ref_norm(q, qw, 1e-6), cos.unsqueeze(1), sin.unsqueeze(1))
    want_k = _ref_rope(_ref_norm(k, kw, 1e-6), cos.unsqueeze(1), sin.unsqueeze(1))
    v_before = qkv[:, (hq + hkv) * d:].clone()
    err = torch.zeros(4, dtype=torch.int32, device=DEV)
    nkv._lib.call("nkv_qk_norm_rope", torch.cuda.current_stream().cuda_stream, qkv.data_ptr(), qkv.stride(0), T,
                  hq, hkv, d, qw.data_ptr(), kw.data_ptr(), cs.data_ptr(), pos.data_ptr(), cs.shape[0], 1e-6,
                  err.data_ptr())
    torch.cuda.synchronize()
    assert int(err[0]) == 0
    _check(q, want_q)
    _check(k, want_k)
    assert torch.equal(qkv[:, (hq + hkv) * d:], v_before)


@pytest.mark.parametrize("T,residual", [(1, True), (1, False), (333, True), (4096, True)])
def test_add_rms_norm_matches_reference_math(T, residual):
    nkv = pkg()
    g = torch.Generator(device=DEV).manual_seed(T + residual)
    H = 2560
    x = torch.randn(T, H, generator=g, device=DEV).bfloat16()
    r = (3 * torch.randn(T, H, generator=g, device=DEV)).bfloat16()
    w = (1 + 0.1 * torch.randn(H, generator=g, device=DEV)).bfloat16()
    if residual:
        s = x.float() + r.float()
        want_r = s.to(torch.bfloat16)
        var = s.pow(2).mean(dim=-1, keepdim=True)
        want = (s * torch.rsqrt(var + 1e-6)).to(torch.bfloat16) * w
    else:
        want_r = x.clone()
        want = _ref_norm(x, w, 1e-6)
    out = torch.empty_like(x)
    rr = r.clone()
    nkv._lib.call("nkv_add_rms_norm", torch.cuda.current_stream().cuda_stream, x.data_ptr(), rr.data_ptr(),
                  w.data_ptr(), out.data_ptr(), T, H, 1e-6, 1 if residual else 0)
    torch.cuda.synchronize()
    assert torch.equal(rr, want_r)
    _check(out, want)


def test_silu_mul_matches_reference_math():
    nkv = pkg()
    g = torch.Generator(device=DEV).manual_seed(5)
    T, I = 37, 9728
    gu = (2 * torch.randn(T, 2 * I, generator=g, device=DEV)).bfloat16()
    x, y = gu.float().chunk(2, -1)
    want = (torch.nn.functional.silu(x) * y).to(torch.bfloat16)
    out = torch.empty(T, I, dtype=torch.bfloat16, device=DEV)
    nkv._lib.call("nkv_silu_mul", torch.cuda.current_stream().cuda_stream, gu.data_ptr(), out.data_ptr(), T, I)
    torch.cuda.synchronize()
    _check(out, want)


@pytest.mark.parametrize("rows,N,K", [(1, 6144, 2560), (1, 2560, 9728), (2, 2560, 4096), (4, 1000, 2560),
                                      (1, 151936, 2560), (3, 77, 136)])
def test_gemv_matches_fp32(rows, N, K):
    """nkv_gemv_bf16 against the fp32 product of the same bf16 operands,
    rounded to bf16 (the kernel sums in fp32 in its own order: each output
    within one bf16 step of the fp32 reference, or 1e-3 absolute)."""
    nkv = pkg()
    g = torch.Generator(device=DEV).manual_seed(N + K + rows)
    x = torch.randn(rows, K, generator=g, device=DEV).bfloat16()
    w = (torch.randn(N, K, generator=g, device=DEV) * 0.05).bfloat16()
    y = torch.empty(rows, N, dtype=torch.bfloat16, device=DEV)
    nkv._lib.call("nkv_gemv_bf16", torch.cuda.current_stream().cuda_stream, x.data_ptr(), x.stride(0), rows,
                  w.data_ptr(), w.stride(0), N, K, y.data_ptr(), y.stride(0))
    torch.cuda.synchronize()
    want = x.float() @ w.float().T
    err = (y.float() - want).abs()
    tol = torch.maximum(want.abs() * 2.0 ** -7, torch.full_like(want, 1e-3))
    assert bool((err <= tol).all()), float((err - tol).max())
