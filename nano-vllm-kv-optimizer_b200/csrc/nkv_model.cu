// Dense-model kernels around the sparse attention path (the callers on either
// side of it in a Qwen3 decoder layer), for the full-model harness:
//
//   nkv_qk_norm_rope  per-head RMSNorm of q and k followed by the rotary
//                     embedding, in place on the fused qkv projection output
//                     (reference nanovllm/models/qwen3.py:91-98 with
//                     layers/layernorm.py:16-26 and layers/rotary_embedding.py:7-15,
//                     138-151); its outputs are the q/k the sparse runtime reads
//   nkv_add_rms_norm  residual add + RMSNorm of a hidden row
//                     (layers/layernorm.py:16-39, qwen3.py:145-152)
//   nkv_silu_mul      SwiGLU activation silu(gate) * up (layers/activation.py:6-11)
//
// All three are HBM/latency-bound elementwise passes: one warp per 128-wide
// head row, or one CTA per hidden row, 16-byte or 4-byte vector accesses.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "nkv_common.cuh"
#include "nkv_host.h"

namespace nkv {
namespace {

__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// One warp per (token, head) row of 128 elements.  Lane l holds the pairs
// x[2l, 2l+1] (first half) and x[64+2l, 64+2l+1] (second half): the rotary
// embedding rotates element j with element j+64, so both sit in one lane.
// Arithmetic follows the reference's eager expressions: sum of squares in
// fp32, mean, x * rsqrt(mean + eps) rounded to bf16, times the bf16 weight
// rounded to bf16, then y1 = x1*cos - x2*sin, y2 = x2*cos + x1*sin in fp32
// (products rounded separately: no fused multiply-add) rounded to bf16.
__global__ void __launch_bounds__(256) qk_norm_rope_kernel(__nv_bfloat16* __restrict__ qkv, long long row_stride,
                                                           int T, int hq, int hkv,
                                                           const __nv_bfloat16* __restrict__ qw,
                                                           const __nv_bfloat16* __restrict__ kw,
                                                           const float* __restrict__ cos_sin,
                                                           const long long* __restrict__ pos, long long max_pos,
                                                           float eps, int* __restrict__ err) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int heads = hq + hkv;
  const long long r = (long long)blockIdx.x * 8 + warp;
  if (r >= (long long)T * heads) return;
  const int t = (int)(r / heads), j = (int)(r % heads);
  __nv_bfloat16* row = qkv + (long long)t * row_stride + (long long)j * NKV_D;
  const __nv_bfloat16* w = j < hq ? qw : kw;
  const __nv_bfloat162 a2 = *reinterpret_cast<const __nv_bfloat162*>(row + 2 * lane);
  const __nv_bfloat162 b2 = *reinterpret_cast<const __nv_bfloat162*>(row + 64 + 2 * lane);
  float x[4] = {__low2float(a2), __high2float(a2), __low2float(b2), __high2float(b2)};
  float ss = __fmul_rn(x[0], x[0]);
  ss = __fadd_rn(ss, __fmul_rn(x[1], x[1]));
  ss = __fadd_rn(ss, __fmul_rn(x[2], x[2]));
  ss = __fadd_rn(ss, __fmul_rn(x[3], x[3]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
  const float inv = rsqrtf(__fadd_rn(__fdiv_rn(ss, (float)NKV_D), eps));
  const int col[4] = {2 * lane, 2 * lane + 1, 64 + 2 * lane, 64 + 2 * lane + 1};
#pragma unroll
  for (int e = 0; e < 4; ++e) x[e] = bf16_round(__fmul_rn(bf16_round(__fmul_rn(x[e], inv)), __bfloat162float(w[col[e]])));
  long long p = pos[t];
  if (p < 0 || p >= max_pos) {  // position outside the cos/sin table
    if (err) atomicExch(err, ERR_BAD_INDEX);
    p = 0;
  }
  const float* cs = cos_sin + p * NKV_D;
  float y[4];
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const float c = cs[2 * lane + e], s = cs[64 + 2 * lane + e];
    const float x1 = x[e], x2 = x[2 + e];
    y[e] = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
    y[2 + e] = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
  }
  *reinterpret_cast<__nv_bfloat162*>(row + 2 * lane) = __floats2bfloat162_rn(y[0], y[1]);
  *reinterpret_cast<__nv_bfloat162*>(row + 64 + 2 * lane) = __floats2bfloat162_rn(y[2], y[3]);
}

// One CTA per hidden row; thread i owns 8 consecutive elements (one 16-byte
// access).  With a residual: s = x + residual in fp32, residual <- bf16(s),
// out <- bf16(bf16(s * rsqrt(mean(s^2) + eps)) * w); without: residual <- x
// and the same normalisation of x (reference layernorm.py:16-39).
__global__ void __launch_bounds__(512) add_rms_norm_kernel(const __nv_bfloat16* __restrict__ x,
                                                           __nv_bfloat16* __restrict__ residual,
                                                           const __nv_bfloat16* __restrict__ w,
                                                           __nv_bfloat16* __restrict__ out, int H, float eps,
                                                           int has_residual) {
  const long long row = blockIdx.x;
  const int i = threadIdx.x * 8;
  __shared__ float red[16];
  float s[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  float ss = 0.f;
  const bool on = i < H;
  if (on) {
    const uint4 xv = *reinterpret_cast<const uint4*>(x + row * H + i);
    const __nv_bfloat16* xb = reinterpret_cast<const __nv_bfloat16*>(&xv);
    if (has_residual) {
      const uint4 rv = *reinterpret_cast<const uint4*>(residual + row * H + i);
      const __nv_bfloat16* rb = reinterpret_cast<const __nv_bfloat16*>(&rv);
#pragma unroll
      for (int e = 0; e < 8; ++e) s[e] = __fadd_rn(__bfloat162float(xb[e]), __bfloat162float(rb[e]));
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) s[e] = __bfloat162float(xb[e]);
    }
    uint4 ro;
    __nv_bfloat16* rob = reinterpret_cast<__nv_bfloat16*>(&ro);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      rob[e] = __float2bfloat16_rn(s[e]);
      ss = __fadd_rn(ss, __fmul_rn(s[e], s[e]));
    }
    *reinterpret_cast<uint4*>(residual + row * H + i) = ro;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = (blockDim.x + 31) >> 5;
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  if (warp == 0) {
    float v = lane < nw ? red[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (lane == 0) red[0] = v;
  }
  __syncthreads();
  if (!on) return;
  const float inv = rsqrtf(__fadd_rn(__fdiv_rn(red[0], (float)H), eps));
  const uint4 wv = *reinterpret_cast<const uint4*>(w + i);
  const __nv_bfloat16* wb = reinterpret_cast<const __nv_bfloat16*>(&wv);
  uint4 yo;
  __nv_bfloat16* yb = reinterpret_cast<__nv_bfloat16*>(&yo);
#pragma unroll
  for (int e = 0; e < 8; ++e)
    yb[e] = __float2bfloat16_rn(__fmul_rn(bf16_round(__fmul_rn(s[e], inv)), __bfloat162float(wb[e])));
  *reinterpret_cast<uint4*>(out + row * H + i) = yo;
}

// out[t, j] = bf16(silu(g) * u) with g = gu[t, j], u = gu[t, I + j] in fp32;
// silu(g) = g / (1 + exp(-g)).  Eight elements per thread.
__global__ void __launch_bounds__(256) silu_mul_kernel(const __nv_bfloat16* __restrict__ gu,
                                                       __nv_bfloat16* __restrict__ out, int T, int I) {
  const long long idx = ((long long)blockIdx.x * blockDim.x + threadIdx.x) * 8;
  const long long total = (long long)T * I;
  if (idx >= total) return;
  const long long t = idx / I, j = idx % I;
  const uint4 gv = *reinterpret_cast<const uint4*>(gu + t * 2 * I + j);
  const uint4 uv = *reinterpret_cast<const uint4*>(gu + t * 2 * I + I + j);
  const __nv_bfloat16* gb = reinterpret_cast<const __nv_bfloat16*>(&gv);
  const __nv_bfloat16* ub = reinterpret_cast<const __nv_bfloat16*>(&uv);
  uint4 ov;
  __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(&ov);
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float g = __bfloat162float(gb[e]);
    const float sg = __fdiv_rn(g, __fadd_rn(1.f, expf(-g)));
    ob[e] = __float2bfloat16_rn(__fmul_rn(sg, __bfloat162float(ub[e])));
  }
  *reinterpret_cast<uint4*>(out + t * I + j) = ov;
}

}  // namespace
}  // namespace nkv

using namespace nkv;

extern "C" int nkv_qk_norm_rope(nkv_stream_t stream, void* qkv, long long row_stride, int T, int hq, int hkv,
                                int head_dim, const void* q_weight, const void* k_weight, const float* cos_sin,
                                const long long* positions, long long max_positions, float eps, int* err) {
  NKV_REQUIRE(qkv && q_weight && k_weight && cos_sin && positions, "qk_norm_rope: null pointer");
  NKV_REQUIRE(T >= 0 && hq >= 1 && hkv >= 1 && max_positions >= 1, "qk_norm_rope: bad shape");
  if (head_dim != NKV_D) {
    set_error("qk_norm_rope: head_dim %d (only %d)", head_dim, NKV_D);
    return NKV_ERR_UNSUPPORTED;
  }
  NKV_REQUIRE(row_stride >= (long long)(hq + 2 * hkv) * NKV_D && row_stride % 2 == 0 &&
                  (reinterpret_cast<uintptr_t>(qkv) & 3) == 0,
              "qk_norm_rope: qkv rows must hold q, k and v heads, 4-byte aligned");
  if (T == 0) return NKV_OK;
  const long long rows = (long long)T * (hq + hkv);
  const long long blocks = (rows + 7) / 8;
  NKV_REQUIRE(blocks < (1ll << 31), "qk_norm_rope: too many rows");
  qk_norm_rope_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<__nv_bfloat16*>(qkv), row_stride, T, hq, hkv, reinterpret_cast<const __nv_bfloat16*>(q_weight),
      reinterpret_cast<const __nv_bfloat16*>(k_weight), cos_sin, positions, max_positions, eps, err);
  return check_launch("qk_norm_rope");
}

extern "C" int nkv_add_rms_norm(nkv_stream_t stream, const void* x, void* residual, const void* weight, void* out,
                                int T, int H, float eps, int has_residual) {
  NKV_REQUIRE(x && residual && weight && out, "add_rms_norm: null pointer");
  NKV_REQUIRE(T >= 0 && H >= 8 && H % 8 == 0 && H <= 8 * 512, "add_rms_norm: H must be a multiple of 8, <= 4096");
  NKV_REQUIRE(((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(residual) |
                reinterpret_cast<uintptr_t>(weight) | reinterpret_cast<uintptr_t>(out)) & 15) == 0,
              "add_rms_norm: pointers must be 16-byte aligned");
  if (T == 0) return NKV_OK;
  const int threads = ((H / 8 + 31) / 32) * 32;
  add_rms_norm_kernel<<<T, threads, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(x), reinterpret_cast<__nv_bfloat16*>(residual),
      reinterpret_cast<const __nv_bfloat16*>(weight), reinterpret_cast<__nv_bfloat16*>(out), H, eps, has_residual);
  return check_launch("add_rms_norm");
}

extern "C" int nkv_silu_mul(nkv_stream_t stream, const void* gate_up, void* out, int T, int I) {
  NKV_REQUIRE(gate_up && out, "silu_mul: null pointer");
  NKV_REQUIRE(T >= 0 && I >= 8 && I % 8 == 0, "silu_mul: I must be a multiple of 8");
  NKV_REQUIRE(((reinterpret_cast<uintptr_t>(gate_up) | reinterpret_cast<uintptr_t>(out)) & 15) == 0,
              "silu_mul: pointers must be 16-byte aligned");
  if (T == 0) return NKV_OK;
  const long long n8 = (long long)T * I / 8;
  silu_mul_kernel<<<(unsigned)((n8 + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(gate_up), reinterpret_cast<__nv_bfloat16*>(out), T, I);
  return check_launch("silu_mul");
}
