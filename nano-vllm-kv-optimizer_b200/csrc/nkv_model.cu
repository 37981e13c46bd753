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
//   nkv_gemv_bf16     y = W x for one token (the decode-time projections and LM
//                     head, layers/linear.py, embed_head.py): HBM-bound weight
//                     streaming
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
  pdl_launch_dependents();  // the next kernel may become resident; it waits for this one
  pdl_wait();               // inputs of the preceding kernel complete past this point
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
  pdl_launch_dependents();  // the next kernel may become resident; it waits for this one
  pdl_wait();               // inputs of the preceding kernel complete past this point
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
  pdl_launch_dependents();  // the next kernel may become resident; it waits for this one
  pdl_wait();               // inputs of the preceding kernel complete past this point
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

// y[r][n] = sum_k x[r][k] W[n][k] for R <= 4 rows of x (bf16 in, fp32
// accumulate, bf16 out).  One warp per output column n (a weight row), a CTA of
// GV_WARPS warps takes consecutive weight rows; x is staged in shared memory as
// fp32 once per CTA.  Lane l streams 16-byte chunks l, l + 32, ... of its
// weight row with GV_U chunks in flight per iteration (non-allocating loads:
// the weights are read once per token), and the dot product ends with a warp
// shuffle reduction.
constexpr int GV_WARPS = 8;
constexpr int GV_U = 8;
template <int R>
__global__ void __launch_bounds__(GV_WARPS * 32) gemv_kernel(const __nv_bfloat16* __restrict__ x, long long ldx,
                                                           const __nv_bfloat16* __restrict__ W, long long ldw,
                                                           int N, int K, __nv_bfloat16* __restrict__ y,
                                                           long long ldy) {
  pdl_launch_dependents();  // the next kernel may become resident; it waits for this one
  pdl_wait();               // inputs of the preceding kernel complete past this point
  extern __shared__ __align__(16) float xs[];  // [R][K]
  for (int i = threadIdx.x; i < R * (K >> 3); i += blockDim.x) {
    const int r = i / (K >> 3), c = i % (K >> 3);
    float v[8];
    unpack8(*reinterpret_cast<const uint4*>(x + r * ldx + c * 8), v);
    *reinterpret_cast<float4*>(xs + r * K + c * 8) = make_float4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<float4*>(xs + r * K + c * 8 + 4) = make_float4(v[4], v[5], v[6], v[7]);
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nch = K >> 3;
  // the CTAs stride over the weight rows, so that the staging of x is paid once per CTA
  for (int n = blockIdx.x * GV_WARPS + warp; n < N; n += gridDim.x * GV_WARPS) {
  const uint4* wr = reinterpret_cast<const uint4*>(W + (long long)n * ldw);
  float acc[R];
#pragma unroll
  for (int r = 0; r < R; ++r) acc[r] = 0.f;
  for (int c0 = lane; c0 < nch; c0 += 32 * GV_U) {
    uint4 w[GV_U];
#pragma unroll
    for (int u = 0; u < GV_U; ++u) {
      const int c = c0 + u * 32;
      w[u] = c < nch ? ldg_nc_v4(wr + c) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int u = 0; u < GV_U; ++u) {
      const int c = c0 + u * 32;
      if (c >= nch) break;
      const uint32_t wv[4] = {w[u].x, w[u].y, w[u].z, w[u].w};
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const float4 xa = *reinterpret_cast<const float4*>(xs + r * K + c * 8);
        const float4 xb = *reinterpret_cast<const float4*>(xs + r * K + c * 8 + 4);
        const float xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          acc[r] = fmaf(__uint_as_float(wv[e] << 16), xv[2 * e], acc[r]);
          acc[r] = fmaf(__uint_as_float(wv[e] & 0xffff0000u), xv[2 * e + 1], acc[r]);
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < R; ++r) {
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], m);
  }
  if (lane == 0) {
#pragma unroll
    for (int r = 0; r < R; ++r) y[r * ldy + n] = __float2bfloat16_rn(acc[r]);
  }
  }
}

// The same product with each weight row split over a whole CTA: CTA b takes
// rows [b * RPC, (b + 1) * RPC) and thread t the 16-byte chunks t, t + 256, ...
// (CH of them) of every one of those rows and of every x row, so a warp reads
// 512 contiguous bytes of a row and every load of the CTA is issued before the
// first product: one DRAM round trip per CTA, RPC x CH loads in flight per
// thread, x read straight into registers (no staging, no barrier before the
// products).  Sums: per thread in chunk order, a warp shuffle tree, then the 8
// warps in order.  RPC = 16 / CH keeps 64 registers of weights in flight.
constexpr int GS_THREADS = 256;
template <int R, int CH>
__global__ void __launch_bounds__(GS_THREADS) gemv_split_kernel(const __nv_bfloat16* __restrict__ x, long long ldx,
                                                                const __nv_bfloat16* __restrict__ W, long long ldw,
                                                                int N, int K, __nv_bfloat16* __restrict__ y,
                                                                long long ldy) {
  constexpr int RPC = CH >= 16 ? 1 : 16 / CH;
  constexpr int NW = GS_THREADS / 32;
  __shared__ float red[NW][R * RPC];
  pdl_launch_dependents();
  pdl_wait();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nch = K >> 3;
  const int n0 = blockIdx.x * RPC;
  uint4 w[RPC][CH];
#pragma unroll
  for (int r = 0; r < RPC; ++r) {
    const int n = n0 + r;
#pragma unroll
    for (int i = 0; i < CH; ++i) {
      const int c = tid + i * GS_THREADS;
      w[r][i] = (n < N && c < nch) ? ldg_nc_v4(W + (long long)n * ldw + c * 8) : make_uint4(0u, 0u, 0u, 0u);
    }
  }
  uint4 xv[R][CH];
#pragma unroll
  for (int q = 0; q < R; ++q)
#pragma unroll
    for (int i = 0; i < CH; ++i) {
      const int c = tid + i * GS_THREADS;
      xv[q][i] = c < nch ? __ldg(reinterpret_cast<const uint4*>(x + q * ldx + c * 8)) : make_uint4(0u, 0u, 0u, 0u);
    }
  float acc[R][RPC];
#pragma unroll
  for (int q = 0; q < R; ++q)
#pragma unroll
    for (int r = 0; r < RPC; ++r) acc[q][r] = 0.f;
#pragma unroll
  for (int i = 0; i < CH; ++i) {
#pragma unroll
    for (int q = 0; q < R; ++q) {
      float xf[8];
      unpack8(xv[q][i], xf);
#pragma unroll
      for (int r = 0; r < RPC; ++r) {
        const uint32_t wv[4] = {w[r][i].x, w[r][i].y, w[r][i].z, w[r][i].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          acc[q][r] = fmaf(__uint_as_float(wv[e] << 16), xf[2 * e], acc[q][r]);
          acc[q][r] = fmaf(__uint_as_float(wv[e] & 0xffff0000u), xf[2 * e + 1], acc[q][r]);
        }
      }
    }
  }
#pragma unroll
  for (int q = 0; q < R; ++q)
#pragma unroll
    for (int r = 0; r < RPC; ++r) {
#pragma unroll
      for (int m = 16; m > 0; m >>= 1) acc[q][r] += __shfl_xor_sync(0xffffffffu, acc[q][r], m);
      if (lane == 0) red[warp][q * RPC + r] = acc[q][r];
    }
  __syncthreads();
  if (tid < R * RPC) {
    const int q = tid / RPC, r = tid % RPC, n = n0 + r;
    float s = 0.f;
#pragma unroll
    for (int v = 0; v < NW; ++v) s += red[v][tid];
    if (n < N) y[q * ldy + n] = __float2bfloat16_rn(s);
  }
}

// Launch in plain stream order, or with programmatic dependent launch allowed
// (NKV_MODEL_PDL=1): every kernel above waits for its predecessor before
// touching memory, so that form only hides launch latency between the dense
// kernels.  It measured slower in the full-model decode step (3.40 against
// 2.87 ms per token: the early-resident dependents crowd the running grid), so
// it is off by default.
template <typename... KArgs, typename... Args>
int launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, const char* what,
               Args... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = knob("NKV_MODEL_PDL", 0) != 0 ? 1 : 0;
  cudaLaunchConfig_t lc = {};
  lc.gridDim = grid;
  lc.blockDim = block;
  lc.dynamicSmemBytes = smem;
  lc.stream = st;
  lc.attrs = attr;
  lc.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&lc, kernel, args...);
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error("%s: launch failed: %s", what, cudaGetErrorString(e));
    return NKV_ERR_CUDA;
  }
  return check_launch(what);
}

}  // namespace
}  // namespace nkv

using namespace nkv;

extern "C" int nkv_gemv_bf16(nkv_stream_t stream, const void* x, long long x_row_stride, int rows, const void* w,
                             long long w_row_stride, int N, int K, void* y, long long y_row_stride) {
  NKV_REQUIRE(x && w && y, "gemv: null pointer");
  NKV_REQUIRE(rows >= 1 && rows <= 4 && N >= 1 && K >= 8 && K % 8 == 0, "gemv: rows 1..4, K a multiple of 8");
  NKV_REQUIRE(w_row_stride >= K && w_row_stride % 8 == 0 && (reinterpret_cast<uintptr_t>(w) & 15) == 0,
              "gemv: weight rows must be 16-byte aligned");
  NKV_REQUIRE(x_row_stride >= K && y_row_stride >= N, "gemv: bad row strides");
  const size_t smem = (size_t)rows * K * sizeof(float);
  NKV_REQUIRE(smem <= 200 * 1024, "gemv: rows x K too large for the staged x (%zu bytes)", smem);
  NKV_REQUIRE(x_row_stride % 8 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0,
              "gemv: x rows must be 16-byte aligned");
  const auto* xs_ = reinterpret_cast<const __nv_bfloat16*>(x);
  const auto* ws_ = reinterpret_cast<const __nv_bfloat16*>(w);
  auto* ys_ = reinterpret_cast<__nv_bfloat16*>(y);
  // rows split over a CTA (up to K = 16384) below 64 K rows; one warp per row
  // above that (the LM head: there staging x once per CTA for many rows pays,
  // 131 against 136 us at 151936 x 2560) or with NKV_GEMV_SPLIT=0
  const int nch = K >> 3;
  const int ch = (nch + GS_THREADS - 1) / GS_THREADS;
  if (ch <= 8 && N <= 65536 && knob("NKV_GEMV_SPLIT", 1) != 0) {
    const int chc = ch == 7 ? 8 : ch;
    const int rpc = 16 / chc;
    const dim3 g((unsigned)((N + rpc - 1) / rpc));
#define NKV_GS(RR, CC)                                                                                      \
  if (rows == RR && chc == CC)                                                                              \
    return launch_pdl(gemv_split_kernel<RR, CC>, g, dim3(GS_THREADS), 0, (cudaStream_t)stream, "gemv", xs_, \
                      (long long)x_row_stride, ws_, (long long)w_row_stride, N, K, ys_, (long long)y_row_stride);
#define NKV_GS_R(RR) NKV_GS(RR, 1) NKV_GS(RR, 2) NKV_GS(RR, 3) NKV_GS(RR, 4) NKV_GS(RR, 5) NKV_GS(RR, 6) NKV_GS(RR, 8)
    NKV_GS_R(1)
    NKV_GS_R(2)
    NKV_GS_R(3)
    NKV_GS_R(4)
#undef NKV_GS_R
#undef NKV_GS
  }
  // enough CTAs to keep every SM streaming, few enough that each stages x once
  // for many rows
  const long long want = (N + GV_WARPS - 1) / GV_WARPS;
  const long long cap = (long long)sm_count() * knob("NKV_GEMV_CTAS_PER_SM", 4);
  const unsigned grid = (unsigned)(want < cap ? want : cap);
  const auto* xb = reinterpret_cast<const __nv_bfloat16*>(x);
  const auto* wb = reinterpret_cast<const __nv_bfloat16*>(w);
  auto* yb = reinterpret_cast<__nv_bfloat16*>(y);
  switch (rows) {
#define NKV_GV_CASE(RR)                                                                                 \
  case RR:                                                                                              \
    if (ensure_smem(gemv_kernel<RR>, smem, "gemv")) return NKV_ERR_CUDA;                               \
    return launch_pdl(gemv_kernel<RR>, dim3(grid), dim3(GV_WARPS * 32), smem, (cudaStream_t)stream, "gemv", xb, \
                      (long long)x_row_stride, wb, (long long)w_row_stride, N, K, yb, (long long)y_row_stride);
    NKV_GV_CASE(1)
    NKV_GV_CASE(2)
    NKV_GV_CASE(3)
    NKV_GV_CASE(4)
#undef NKV_GV_CASE
  }
  return NKV_ERR_ARG;
}

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
  return launch_pdl(qk_norm_rope_kernel, dim3((unsigned)blocks), dim3(256), 0, (cudaStream_t)stream, "qk_norm_rope",
                    reinterpret_cast<__nv_bfloat16*>(qkv), row_stride, T, hq, hkv,
                    reinterpret_cast<const __nv_bfloat16*>(q_weight), reinterpret_cast<const __nv_bfloat16*>(k_weight),
                    cos_sin, positions, (long long)max_positions, eps, err);
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
  return launch_pdl(add_rms_norm_kernel, dim3(T), dim3(threads), 0, (cudaStream_t)stream, "add_rms_norm",
                    reinterpret_cast<const __nv_bfloat16*>(x), reinterpret_cast<__nv_bfloat16*>(residual),
                    reinterpret_cast<const __nv_bfloat16*>(weight), reinterpret_cast<__nv_bfloat16*>(out), H, eps,
                    has_residual);
}

extern "C" int nkv_silu_mul(nkv_stream_t stream, const void* gate_up, void* out, int T, int I) {
  NKV_REQUIRE(gate_up && out, "silu_mul: null pointer");
  NKV_REQUIRE(T >= 0 && I >= 8 && I % 8 == 0, "silu_mul: I must be a multiple of 8");
  NKV_REQUIRE(((reinterpret_cast<uintptr_t>(gate_up) | reinterpret_cast<uintptr_t>(out)) & 15) == 0,
              "silu_mul: pointers must be 16-byte aligned");
  if (T == 0) return NKV_OK;
  const long long n8 = (long long)T * I / 8;
  return launch_pdl(silu_mul_kernel, dim3((unsigned)((n8 + 255) / 256)), dim3(256), 0, (cudaStream_t)stream,
                    "silu_mul", reinterpret_cast<const __nv_bfloat16*>(gate_up), reinterpret_cast<__nv_bfloat16*>(out),
                    T, I);
}
