// Kernel (5): KV store + representative refresh for one prefill chunk, plus the
// small helpers around it (K channel scale, query-segment means, and the dense
// paged-cache row scatter that twins the reference's Triton store_kvcache).
//
// Store: one CTA per (block, kv head).  One pass over the chunk's rows writes
// the bf16 block store, sink and recent-ring rows from the registers and
// stages the 64 x 128 key tile in shared memory (the value tile too for the
// int8 kinds, whose scales need the whole tile).  The key directions are
// computed once into shared memory (fp32, 32 KiB) and every pass of the
// representative choice reads them; per warp four tokens are reduced at a
// time (interleaved butterflies).  The r representatives are chosen in-CTA
// exactly as the reference does (m12_runtime.py:354-395):
//   dir_t   = k_t / max(|k_t|, 1e-12)                 (true division, as F.normalize)
//   mean    = sum_t dir_t / B ;  mdir = mean / max(|mean|, 1e-12)
//   pick_0  = first argmax_t dir_t . mdir
//   pick_s  = first argmin_t of (taken ? 2 : max(0, max_{s'<s} dir_t . dir_pick_s'))
// The stored representative is the raw bf16 key row of each pick.
#include "nkv_common.cuh"
#include "nkv_host.h"

namespace nkv {

constexpr int ST_THREADS = 256;
constexpr int ST_MAXB = 128;

struct StoreParams {
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  long long k_row, k_head, v_row, v_head;
  int T, hkv, B, r, start_block, max_blocks, store_kind;  // max_blocks: reps block dim
  void* k_store;
  void* v_store;
  const float* k_chan_scale;
  float* v_block_scale;
  __nv_bfloat16* k_tok_scale;
  __nv_bfloat16* v_tok_scale;
  __nv_bfloat16* reps;
  short* rep_index;
  __nv_bfloat16* sink_k;
  __nv_bfloat16* sink_v;
  int sink_cap, sink_write;
  __nv_bfloat16* ring_k;
  __nv_bfloat16* ring_v;
  int ring_cap, ring_pos0, ring_first;
};

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) x += __shfl_xor_sync(FULL, x, m);
  return x;
}
__device__ __forceinline__ float warp_max(float x) {
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) x = fmaxf(x, __shfl_xor_sync(FULL, x, m));
  return x;
}

// x / n, correctly rounded, given y = RN(1/n) (n a positive normal float):
// q0 = RN(x * y) is within an ulp of x / n, the remainder r = x - q0 * n is
// exact in one fma, and RN(q0 + r * y) is the correctly rounded quotient
// (Markstein, "Computation of elementary functions on the IBM RISC System/6000
// processor", IBM J. Res. Dev. 34(1), 1990).  The argument needs a quotient
// in the normal range: tiny quotients (and zeros, for the sign) take the
// division itself.  Checked against the division operator by nkv_selftest_div.
__device__ __forceinline__ float div_rcp(float x, float n, float y) {
  const float q0 = x * y;
  if (fabsf(q0) < 0x1p-100f) return __fdiv_rn(x, n);
  const float r = fmaf(-q0, n, x);
  return fmaf(r, y, q0);
}

// quantize one float with a given scale, reference rounding (half to even)
__device__ __forceinline__ signed char q8(float x, float s) {
  float y = rintf(__fdiv_rn(x, s));
  y = fminf(fmaxf(y, -127.f), 127.f);
  return (signed char)(int)y;
}

__global__ void __launch_bounds__(ST_THREADS) store_kernel(StoreParams p) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int B = p.B;
  // V is staged only for the int8 store kinds (its scales need the whole tile)
  const bool stage_v = p.k_store != nullptr && p.store_kind != NKV_STORE_BF16;
  __nv_bfloat16* ks = reinterpret_cast<__nv_bfloat16*>(smem);           // [B][D] raw keys
  float* dir = reinterpret_cast<float*>(ks + B * NKV_D);                 // [B][D] k_t / |k_t|
  __nv_bfloat16* vs = reinterpret_cast<__nv_bfloat16*>(dir + B * NKV_D); // [B][D] (int8 kinds)
  float* crit = reinterpret_cast<float*>(vs + (stage_v ? B * NKV_D : 0)); // [B]
  float* worst = crit + ST_MAXB;                                         // [B]
  float* mdir = worst + ST_MAXB;                                         // [D]
  float* red = mdir + NKV_D;                                             // [8 warps]
  __shared__ int picks[8];
  __shared__ float s_vscale;

  const int bl = blockIdx.x, h = blockIdx.y;
  const int blk = p.start_block + bl;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const long long tile = ((long long)blk * p.hkv + h) * B;  // row index into the store
  const bool bf16_store = p.k_store != nullptr && p.store_kind == NKV_STORE_BF16;

  // ---- one pass over the chunk's rows: stage K (and V for int8 kinds); the
  // bf16 block store (zero rows past T), sink and recent-ring rows are written
  // straight from the registers ------------------------------------------------
  // Loads of ST_BATCH rows per thread are all issued before their stores (the
  // compiler may not move a load above a store to another global pointer).
  constexpr int ST_BATCH = 4;
  for (int base = 0; base < B * (NKV_D / 8); base += ST_BATCH * ST_THREADS) {
    uint4 kr[ST_BATCH], vr[ST_BATCH];
#pragma unroll
    for (int j = 0; j < ST_BATCH; ++j) {
      const int i = base + j * ST_THREADS + tid;
      const int gt = bl * B + i / (NKV_D / 8), c = i % (NKV_D / 8);
      kr[j] = vr[j] = make_uint4(0, 0, 0, 0);
      if (i < B * (NKV_D / 8) && gt < p.T) {
        kr[j] = __ldg(reinterpret_cast<const uint4*>(p.k + gt * p.k_row + h * p.k_head + c * 8));
        vr[j] = __ldg(reinterpret_cast<const uint4*>(p.v + gt * p.v_row + h * p.v_head + c * 8));
      }
    }
#pragma unroll
    for (int j = 0; j < ST_BATCH; ++j) {
      const int i = base + j * ST_THREADS + tid;
      if (i >= B * (NKV_D / 8)) break;
      const int gt = bl * B + i / (NKV_D / 8), c = i % (NKV_D / 8);
      const uint4 kv = kr[j], vv = vr[j];
      reinterpret_cast<uint4*>(ks)[i] = kv;
      if (stage_v) reinterpret_cast<uint4*>(vs)[i] = vv;
      if (bf16_store) {
        reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.k_store) + tile * NKV_D)[i] = kv;
        reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.v_store) + tile * NKV_D)[i] = vv;
      }
      if (gt < p.T) {
        if (gt < p.sink_write) {
          const long long o = ((long long)h * p.sink_cap + gt) * NKV_D + c * 8;
          *reinterpret_cast<uint4*>(p.sink_k + o) = kv;
          *reinterpret_cast<uint4*>(p.sink_v + o) = vv;
        }
        if (gt >= p.ring_first && p.ring_cap > 0) {
          const int slot = (p.ring_pos0 + gt) % p.ring_cap;
          const long long o = ((long long)h * p.ring_cap + slot) * NKV_D + c * 8;
          *reinterpret_cast<uint4*>(p.ring_k + o) = kv;
          *reinterpret_cast<uint4*>(p.ring_v + o) = vv;
        }
      }
    }
  }
  __syncthreads();

  // ---- int8 block store ------------------------------------------------------
  if (!stage_v) {
    // bf16 store (written above) or representatives only
  } else if (p.store_kind == NKV_STORE_INT8_REF) {
    // V block scale: max |v| over the block's tokens and dims
    float m = 0.f;
    for (int i = tid; i < B * NKV_D; i += ST_THREADS) m = fmaxf(m, fabsf(__bfloat162float(vs[i])));
    m = warp_max(m);
    if (lane == 0) red[warp] = m;
    __syncthreads();
    if (tid == 0) {
      float mm = 0.f;
      for (int w = 0; w < ST_THREADS / 32; ++w) mm = fmaxf(mm, red[w]);
      s_vscale = __fdiv_rn(fmaxf(mm, 1e-8f), 127.f);
      p.v_block_scale[(long long)blk * p.hkv + h] = s_vscale;
    }
    __syncthreads();
    const float vsc = s_vscale;
    signed char* ko = reinterpret_cast<signed char*>(p.k_store) + tile * NKV_D;
    signed char* vo = reinterpret_cast<signed char*>(p.v_store) + tile * NKV_D;
    for (int i = tid; i < B * NKV_D / 4; i += ST_THREADS) {
      const int e = i * 4, d = e % NKV_D;
      char4 kq, vq;
      kq.x = q8(__bfloat162float(ks[e + 0]), p.k_chan_scale[h * NKV_D + d + 0]);
      kq.y = q8(__bfloat162float(ks[e + 1]), p.k_chan_scale[h * NKV_D + d + 1]);
      kq.z = q8(__bfloat162float(ks[e + 2]), p.k_chan_scale[h * NKV_D + d + 2]);
      kq.w = q8(__bfloat162float(ks[e + 3]), p.k_chan_scale[h * NKV_D + d + 3]);
      vq.x = q8(__bfloat162float(vs[e + 0]), vsc);
      vq.y = q8(__bfloat162float(vs[e + 1]), vsc);
      vq.z = q8(__bfloat162float(vs[e + 2]), vsc);
      vq.w = q8(__bfloat162float(vs[e + 3]), vsc);
      reinterpret_cast<char4*>(ko)[i] = kq;
      reinterpret_cast<char4*>(vo)[i] = vq;
    }
  } else {  // NKV_STORE_INT8_TOKEN: bf16 scale per (token) for K and V
    signed char* ko = reinterpret_cast<signed char*>(p.k_store) + tile * NKV_D;
    signed char* vo = reinterpret_cast<signed char*>(p.v_store) + tile * NKV_D;
    for (int t = warp; t < B; t += ST_THREADS / 32) {
      float kx[4], vx[4], km = 0.f, vm = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        kx[i] = __bfloat162float(ks[t * NKV_D + lane * 4 + i]);
        vx[i] = __bfloat162float(vs[t * NKV_D + lane * 4 + i]);
        km = fmaxf(km, fabsf(kx[i]));
        vm = fmaxf(vm, fabsf(vx[i]));
      }
      km = warp_max(km);
      vm = warp_max(vm);
      const __nv_bfloat16 kscb = __float2bfloat16_rn(__fdiv_rn(fmaxf(km, 1e-8f), 127.f));
      const __nv_bfloat16 vscb = __float2bfloat16_rn(__fdiv_rn(fmaxf(vm, 1e-8f), 127.f));
      const float ksc = __bfloat162float(kscb), vsc = __bfloat162float(vscb);
      char4 kq, vq;
      kq.x = q8(kx[0], ksc); kq.y = q8(kx[1], ksc); kq.z = q8(kx[2], ksc); kq.w = q8(kx[3], ksc);
      vq.x = q8(vx[0], vsc); vq.y = q8(vx[1], vsc); vq.z = q8(vx[2], vsc); vq.w = q8(vx[3], vsc);
      reinterpret_cast<char4*>(ko + t * NKV_D)[lane] = kq;
      reinterpret_cast<char4*>(vo + t * NKV_D)[lane] = vq;
      if (lane == 0) {
        p.k_tok_scale[tile + t] = kscb;
        p.v_tok_scale[tile + t] = vscb;
      }
    }
  }

  // ---- representatives ---------------------------------------------------------
  // Four threads per token (t = tid / 4 + 64 g; quarter qd = tid % 4 holds dims
  // [32 qd, 32 qd + 32)), so a token's dot product is 32 fmas and two shuffles.
  // dir_t = k_t / max(|k_t|, 1e-12) is computed once into shared memory, its
  // 16-byte chunks XOR-swizzled within each quarter by (qd, row parity): the 8
  // lanes of a shared-memory phase then touch 8 different bank groups.  mdir
  // uses the same layout with row parity 0.
  const int qd = tid & 3;
  for (int tb = 0; tb < B; tb += ST_THREADS / 4) {
    const int t = tb + (tid >> 2);
    if (t >= B) break;  // warp-uniform (B is a multiple of 8)
    const int sw = qd | ((t & 1) << 2);
    float x[32];
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      unpack8(*reinterpret_cast<const uint4*>(ks + t * NKV_D + qd * 32 + c * 8), x + c * 8);
#pragma unroll
      for (int e = 0; e < 8; ++e) ss = fmaf(x[c * 8 + e], x[c * 8 + e], ss);
    }
    ss += __shfl_xor_sync(FULL, ss, 1);
    ss += __shfl_xor_sync(FULL, ss, 2);
    const float n = fmaxf(sqrtf(ss), 1e-12f);
    const float y = __frcp_rn(n);
#pragma unroll
    for (int i = 0; i < 8; ++i)
      *reinterpret_cast<float4*>(dir + t * NKV_D + qd * 32 + ((i ^ sw) << 2)) =
          make_float4(div_rcp(x[i * 4 + 0], n, y), div_rcp(x[i * 4 + 1], n, y), div_rcp(x[i * 4 + 2], n, y),
                      div_rcp(x[i * 4 + 3], n, y));
  }
  __syncthreads();
  // mean direction: thread (d, half) sums dir_t[d] over half of the tokens
  {
    const int d = tid & (NKV_D - 1), hf = tid >> 7;  // ST_THREADS == 2 * NKV_D
    const int dq = d >> 5, di = (d >> 2) & 7, de = d & 3;
    const int off0 = dq * 32 + ((di ^ dq) << 2) + de, off1 = dq * 32 + ((di ^ (dq | 4)) << 2) + de;
    const int h0 = hf * (B / 2), h1 = h0 + B / 2;
    float sm = 0.f;
    for (int t = h0; t < h1; ++t) sm += dir[t * NKV_D + ((t & 1) ? off1 : off0)];
    crit[tid] = sm;  // (crit and worst as scratch: 256 floats)
    __syncthreads();
    if (tid < NKV_D) mdir[off0] = __fdiv_rn(crit[tid] + crit[tid + NKV_D], (float)B);
  }
  __syncthreads();
  if (warp == 0) {  // normalise mdir (elementwise: layout-agnostic)
    float sq = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) sq = fmaf(mdir[lane * 4 + i], mdir[lane * 4 + i], sq);
    sq = warp_sum(sq);
    const float n = fmaxf(sqrtf(sq), 1e-12f);
#pragma unroll
    for (int i = 0; i < 4; ++i) mdir[lane * 4 + i] = __fdiv_rn(mdir[lane * 4 + i], n);
  }
  __syncthreads();

  for (int step = 0; step < p.r; ++step) {
    // criterion per token: dir_t . mdir (step 0), dir_t . dir_pick (later)
    const int pk = step == 0 ? 0 : picks[step - 1];
    const float* ref = step == 0 ? mdir : dir + pk * NKV_D;
    const int rsw = qd | ((pk & 1) << 2);  // mdir: row parity 0
    for (int tb = 0; tb < B; tb += ST_THREADS / 4) {
      const int t = tb + (tid >> 2);
      if (t >= B) break;  // warp-uniform
      const int sw = qd | ((t & 1) << 2);
      float sc = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 a4 = *reinterpret_cast<const float4*>(dir + t * NKV_D + qd * 32 + ((i ^ sw) << 2));
        const float4 r4 = *reinterpret_cast<const float4*>(ref + qd * 32 + ((i ^ rsw) << 2));
        sc = fmaf(a4.x, r4.x, sc);
        sc = fmaf(a4.y, r4.y, sc);
        sc = fmaf(a4.z, r4.z, sc);
        sc = fmaf(a4.w, r4.w, sc);
      }
      sc += __shfl_xor_sync(FULL, sc, 1);
      sc += __shfl_xor_sync(FULL, sc, 2);
      if (qd == 0) {
        if (step == 0) {
          crit[t] = sc;
        } else {
          const float w = step == 1 ? sc : fmaxf(worst[t], sc);
          worst[t] = w;
          bool taken = false;
          for (int q = 0; q < step; ++q) taken |= (picks[q] == t);
          crit[t] = taken ? 2.0f : fmaxf(w, 0.f);
        }
      }
    }
    __syncthreads();
    if (warp == 0) {
      // first index of the max (step 0) / min (later steps)
      float best = step == 0 ? -INFINITY : INFINITY;
      int bi = 0x7fffffff;
      for (int t = lane; t < B; t += 32) {
        const float c = crit[t];
        const bool better = step == 0 ? (c > best) : (c < best);
        if (better) { best = c; bi = t; }
      }
#pragma unroll
      for (int m = 16; m > 0; m >>= 1) {
        const float ob = __shfl_xor_sync(FULL, best, m);
        const int oi = __shfl_xor_sync(FULL, bi, m);
        const bool take = step == 0 ? (ob > best || (ob == best && oi < bi))
                                    : (ob < best || (ob == best && oi < bi));
        if (take) { best = ob; bi = oi; }
      }
      if (lane == 0) picks[step] = (bi >= 0 && bi < B) ? bi : 0;  // all-NaN guard
    }
    __syncthreads();
  }
  // write the chosen raw keys
  for (int i = tid; i < p.r * (NKV_D / 8); i += ST_THREADS) {
    const int j = i / (NKV_D / 8), c = i % (NKV_D / 8);
    const long long o = (((long long)h * p.max_blocks + blk) * p.r + j) * NKV_D + c * 8;
    *reinterpret_cast<uint4*>(p.reps + o) = reinterpret_cast<uint4*>(ks + picks[j] * NKV_D)[c];
  }
  if (p.rep_index && tid < p.r)
    p.rep_index[((long long)h * p.max_blocks + blk) * p.r + tid] = (short)picks[tid];
}

// Store + representatives for 64-token blocks into a bf16 block store (or
// representatives only), as two kernels that run at the same time: the copy
// (block store, sink and ring rows; bound by HBM) and the representative
// choice (bound by its chain of dependent steps), each over the same
// (block, head) grid.  The copy grid lets the representatives grid start at
// once (programmatic dependent launch); the representatives grid reads only
// the chunk's keys, which the copy does not write, and waits for the copy grid
// only at its very end, so that the pair completes together (a later kernel
// in the stream sees the store, the sink and the ring written).
//
// In both, thread t owns chunk c = t % 16 (dims 8c .. 8c + 7) of rows
// t / 16 + 16 j, j < 4, and issues all of its loads before its stores.
constexpr int SB64 = 64;
// The copy grid is smaller than the (block, head) grid and strides over it,
// so that it leaves room on every SM for the representatives CTAs beside it.
__global__ void __launch_bounds__(ST_THREADS) store_copy_b64(StoreParams p, int nblk) {
  pdl_launch_dependents();
  const int tid = threadIdx.x;
  const int c = tid & 15, rg = tid >> 4;
  const bool store = p.k_store != nullptr;
  for (int u = blockIdx.x; u < nblk * p.hkv; u += gridDim.x) {
  const int bl = u / p.hkv, h = u % p.hkv;
  const int blk = p.start_block + bl;
  const long long tile = ((long long)blk * p.hkv + h) * SB64;
  uint4 kr[4], vr[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int gt = bl * SB64 + rg + 16 * j;
    kr[j] = vr[j] = make_uint4(0, 0, 0, 0);
    if (gt < p.T) {
      kr[j] = __ldg(reinterpret_cast<const uint4*>(p.k + gt * p.k_row + h * p.k_head + c * 8));
      vr[j] = __ldg(reinterpret_cast<const uint4*>(p.v + gt * p.v_row + h * p.v_head + c * 8));
    }
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int row = rg + 16 * j, gt = bl * SB64 + row;
    if (store) {
      const long long o = (tile + row) * NKV_D + c * 8;
      *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.k_store) + o) = kr[j];
      *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.v_store) + o) = vr[j];
    }
    if (gt < p.T) {
      if (gt < p.sink_write) {
        const long long o = ((long long)h * p.sink_cap + gt) * NKV_D + c * 8;
        *reinterpret_cast<uint4*>(p.sink_k + o) = kr[j];
        *reinterpret_cast<uint4*>(p.sink_v + o) = vr[j];
      }
      if (gt >= p.ring_first && p.ring_cap > 0) {
        const int slot = (p.ring_pos0 + gt) % p.ring_cap;
        const long long o = ((long long)h * p.ring_cap + slot) * NKV_D + c * 8;
        *reinterpret_cast<uint4*>(p.ring_k + o) = kr[j];
        *reinterpret_cast<uint4*>(p.ring_v + o) = vr[j];
      }
    }
  }
  }
}

// Sum over the 16 lanes of a row group of four per-lane values x[j] (one per
// row j): a transposing butterfly (5 shuffles instead of 16).  Returns the
// full sum of row (lane >> 2) & 3; the 4 lanes that share bits 3..2 hold the
// same value.  The order of the additions is fixed.
__device__ __forceinline__ float rowsum16_t(const float (&x)[4], int lane) {
  const bool b3 = (lane >> 3) & 1, b2 = (lane >> 2) & 1;
  const float s0 = b3 ? x[0] : x[2], s1 = b3 ? x[1] : x[3];
  const float r0 = __shfl_xor_sync(FULL, s0, 8), r1 = __shfl_xor_sync(FULL, s1, 8);
  const float k0 = (b3 ? x[2] : x[0]) + r0, k1 = (b3 ? x[3] : x[1]) + r1;  // rows 2 b3, 2 b3 + 1
  const float r = __shfl_xor_sync(FULL, b2 ? k0 : k1, 4);
  float v = (b2 ? k1 : k0) + r;  // row 2 b3 + b2
  v += __shfl_xor_sync(FULL, v, 2);
  v += __shfl_xor_sync(FULL, v, 1);
  return v;
}

// The representatives: the general kernel's rule with the key directions held
// in registers.  Row norms by a transposing 16-lane shuffle sum, the division
// correctly rounded as above, the directions also written into a shared fp32
// tile from which the farthest-point steps read their reference direction;
// the mean direction is a fixed-order sum of the threads' partial sums.  A
// step is 8 fmas per row, one transposing row sum (lane l then holds row
// rg + 16 ((l >> 2) & 3)), a per-warp first-index arg-best by shuffles, one
// barrier, and the same shuffle reduction over the 8 warps' candidates in
// every warp (no second barrier: the candidate slots alternate by step).  The
// chosen raw key rows are read back from the input (L2) at the end.
template <bool COPY>
__global__ void __launch_bounds__(ST_THREADS, 4) store_reps_b64(StoreParams p) {
  __shared__ __align__(16) float dir_t[SB64 * NKV_D];  // [row][D] k_row / |k_row|
  __shared__ __align__(16) float part[16][NKV_D];      // per row group: sum of its 4 rows' directions
  __shared__ float md[NKV_D];
  __shared__ float red[4];
  __shared__ float s_bv[2][ST_THREADS / 32];
  __shared__ int s_bi[2][ST_THREADS / 32];
  const int bl = blockIdx.x, h = blockIdx.y;
  const int blk = p.start_block + bl;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int c = tid & 15, rg = tid >> 4;  // chunk; row group (rows rg + 16 j)
  const int my_j = (lane >> 2) & 3;      // the row of the group whose sums this lane ends with
  const int my_row = rg + 16 * my_j;

  uint4 kr[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int gt = bl * SB64 + rg + 16 * j;
    kr[j] = make_uint4(0, 0, 0, 0);
    if (gt < p.T) kr[j] = __ldg(reinterpret_cast<const uint4*>(p.k + gt * p.k_row + h * p.k_head + c * 8));
  }
  if constexpr (COPY) {  // the copy in the same CTA: V loads, then every store, from the registers
    uint4 vr[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int gt = bl * SB64 + rg + 16 * j;
      vr[j] = make_uint4(0, 0, 0, 0);
      if (gt < p.T) vr[j] = __ldg(reinterpret_cast<const uint4*>(p.v + gt * p.v_row + h * p.v_head + c * 8));
    }
    const long long tile = ((long long)blk * p.hkv + h) * SB64;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int row = rg + 16 * j, gt = bl * SB64 + row;
      if (p.k_store) {
        const long long o = (tile + row) * NKV_D + c * 8;
        *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.k_store) + o) = kr[j];
        *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.v_store) + o) = vr[j];
      }
      if (gt < p.T) {
        if (gt < p.sink_write) {
          const long long o = ((long long)h * p.sink_cap + gt) * NKV_D + c * 8;
          *reinterpret_cast<uint4*>(p.sink_k + o) = kr[j];
          *reinterpret_cast<uint4*>(p.sink_v + o) = vr[j];
        }
        if (gt >= p.ring_first && p.ring_cap > 0) {
          const int slot = (p.ring_pos0 + gt) % p.ring_cap;
          const long long o = ((long long)h * p.ring_cap + slot) * NKV_D + c * 8;
          *reinterpret_cast<uint4*>(p.ring_k + o) = kr[j];
          *reinterpret_cast<uint4*>(p.ring_v + o) = vr[j];
        }
      }
    }
  }

  // ---- directions (registers + shared tile) and partial mean sums -------------------
  float dr[4][8];
  {
    float ss[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      unpack8(kr[j], dr[j]);
      ss[j] = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) ss[j] = fmaf(dr[j][e], dr[j][e], ss[j]);
    }
    const float mine = rowsum16_t(ss, lane);
    float pm[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) pm[e] = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      // row j's sum sits in the lanes whose bits 3..2 are j
      const float tot = __shfl_sync(FULL, mine, (lane & ~15) | (j << 2));
      const float n = fmaxf(sqrtf(tot), 1e-12f);
      const float y = __frcp_rn(n);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        dr[j][e] = div_rcp(dr[j][e], n, y);
        pm[e] += dr[j][e];
      }
      float* dt = dir_t + (rg + 16 * j) * NKV_D + c * 8;
      *reinterpret_cast<float4*>(dt) = make_float4(dr[j][0], dr[j][1], dr[j][2], dr[j][3]);
      *reinterpret_cast<float4*>(dt + 4) = make_float4(dr[j][4], dr[j][5], dr[j][6], dr[j][7]);
    }
    *reinterpret_cast<float4*>(&part[rg][c * 8]) = make_float4(pm[0], pm[1], pm[2], pm[3]);
    *reinterpret_cast<float4*>(&part[rg][c * 8 + 4]) = make_float4(pm[4], pm[5], pm[6], pm[7]);
  }
  __syncthreads();
  if (tid < NKV_D) {  // mean direction (unnormalised) and its squared norm per warp
    float m = 0.f;
#pragma unroll
    for (int g = 0; g < 16; ++g) m += part[g][tid];
    m *= 1.0f / SB64;  // exact: a power of two
    md[tid] = m;
    const float sq = warp_sum(m * m);
    if (lane == 0) red[warp] = sq;
  }
  __syncthreads();
  const float nrm = fmaxf(sqrtf(((red[0] + red[1]) + red[2]) + red[3]), 1e-12f);
  const float nrm_y = __frcp_rn(nrm);
  float ref[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) ref[e] = div_rcp(md[c * 8 + e], nrm, nrm_y);

  // ---- r steps: step 0 max cosine to the mean direction, then farthest point --------
  float worst = 0.f;  // running max cosine of this lane's row to the picks
  bool taken = false;
  int pk[8];
#pragma unroll
  for (int s = 0; s < 8; ++s) {
    pk[s] = 0;
    if (s >= p.r) continue;  // uniform
    if (s > 0) {
      const float* pr = dir_t + pk[s - 1] * NKV_D + c * 8;
      const float4 a = *reinterpret_cast<const float4*>(pr), b = *reinterpret_cast<const float4*>(pr + 4);
      ref[0] = a.x; ref[1] = a.y; ref[2] = a.z; ref[3] = a.w;
      ref[4] = b.x; ref[5] = b.y; ref[6] = b.z; ref[7] = b.w;
    }
    float dd[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      dd[j] = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) dd[j] = fmaf(dr[j][e], ref[e], dd[j]);
    }
    const float d = rowsum16_t(dd, lane);  // row my_row
    float bv = d;
    if (s > 0) {
      worst = s == 1 ? d : fmaxf(worst, d);
      bv = taken ? 2.0f : fmaxf(worst, 0.f);
    }
    int bi = my_row;
    // first-index arg-best over the warp's 8 rows (lanes 4 apart hold other rows)
#pragma unroll
    for (int m = 4; m < 32; m <<= 1) {
      const float ob = __shfl_xor_sync(FULL, bv, m);
      const int oi = __shfl_xor_sync(FULL, bi, m);
      if (s == 0 ? (ob > bv || (ob == bv && oi < bi)) : (ob < bv || (ob == bv && oi < bi))) {
        bv = ob;
        bi = oi;
      }
    }
    if (lane == 0) {
      s_bv[s & 1][warp] = bv;
      s_bi[s & 1][warp] = bi;
    }
    __syncthreads();
    float fb = s_bv[s & 1][lane & 7];
    int fi = s_bi[s & 1][lane & 7];
#pragma unroll
    for (int m = 1; m < 8; m <<= 1) {
      const float ob = __shfl_xor_sync(FULL, fb, m);
      const int oi = __shfl_xor_sync(FULL, fi, m);
      if (s == 0 ? (ob > fb || (ob == fb && oi < fi)) : (ob < fb || (ob == fb && oi < fi))) {
        fb = ob;
        fi = oi;
      }
    }
    const int pick = (fi >= 0 && fi < SB64) ? fi : 0;  // all-NaN guard
    pk[s] = pick;
    taken |= pick == my_row;
  }
  // ---- the chosen raw key rows (from the input, an L2 read) --------------------------
#pragma unroll
  for (int s = 0; s < 8; ++s) {
    if (s >= p.r || (tid >> 4) != s) continue;
    const int gt = bl * SB64 + pk[s];
    uint4 kv = make_uint4(0, 0, 0, 0);
    if (gt < p.T) kv = __ldg(reinterpret_cast<const uint4*>(p.k + gt * p.k_row + h * p.k_head + c * 8));
    *reinterpret_cast<uint4*>(p.reps + (((long long)h * p.max_blocks + blk) * p.r + s) * NKV_D + c * 8) = kv;
  }
  if (p.rep_index && tid == 0)
    for (int s = 0; s < p.r && s < 8; ++s) p.rep_index[((long long)h * p.max_blocks + blk) * p.r + s] = (short)pk[s];
  // the copy grid (when there is one) has completed before this grid does
  if (!COPY) pdl_wait();
}

// K channel scale: one CTA per kv head, thread = channel.
__global__ void kscale_kernel(const __nv_bfloat16* k, int T, long long row, long long head,
                              float* out) {
  __shared__ float part[8][NKV_D];
  const int h = blockIdx.x;
  const int d = threadIdx.x & (NKV_D - 1), slice = threadIdx.x / NKV_D;  // 8 slices
  float m = 0.f;
  for (int t = slice; t < T; t += 8) m = fmaxf(m, fabsf(__bfloat162float(k[t * row + h * head + d])));
  part[slice][d] = m;
  __syncthreads();
  if (slice == 0) {
    for (int s = 1; s < 8; ++s) m = fmaxf(m, part[s][d]);
    out[h * NKV_D + d] = __fdiv_rn(fmaxf(m, 1e-8f), 127.f);
  }
}

// Query-segment means: grid (nseg, hq), thread = dim.
__global__ void qsum_kernel(const __nv_bfloat16* q, int T, long long row, long long head, int nseg,
                            __nv_bfloat16* out) {
  const int s = blockIdx.x, h = blockIdx.y, d = threadIdx.x;
  // torch.tensor_split: the first T % nseg segments hold one extra row
  const int base = T / nseg, extra = T % nseg;
  const int lo = s * base + min(s, extra);
  const int n = base + (s < extra ? 1 : 0);
  float acc = 0.f;
  for (int t = lo; t < lo + n; ++t) acc += __bfloat162float(q[t * row + h * head + d]);
  out[((long long)s * gridDim.y + h) * NKV_D + d] = __float2bfloat16_rn(__fdiv_rn(acc, (float)n));
}

// Paged-cache scatter: grid n rows.
__global__ void kvcache_kernel(const __nv_bfloat16* key, long long ks, const __nv_bfloat16* value,
                               long long vs, __nv_bfloat16* kc, __nv_bfloat16* vc,
                               const long long* slot, int row_elems) {
  const int i = blockIdx.x;
  const long long s = slot[i];
  if (s == -1) return;
  const bool vec = (row_elems % 8) == 0 && (ks % 8) == 0 && (vs % 8) == 0;
  if (vec) {
    for (int c = threadIdx.x; c < row_elems / 8; c += blockDim.x) {
      reinterpret_cast<uint4*>(kc + s * row_elems)[c] = reinterpret_cast<const uint4*>(key + i * ks)[c];
      reinterpret_cast<uint4*>(vc + s * row_elems)[c] = reinterpret_cast<const uint4*>(value + i * vs)[c];
    }
  } else {
    for (int c = threadIdx.x; c < row_elems; c += blockDim.x) {
      kc[s * row_elems + c] = key[i * ks + c];
      vc[s * row_elems + c] = value[i * vs + c];
    }
  }
}

// Recent-ring append: token i (i >= first) of a T-token run goes to slot
// (pos0 + i) % cap of every head.  grid (T - first), 2*hkv*16 threads max.
__global__ void ring_append_kernel(const __nv_bfloat16* k, const __nv_bfloat16* v, long long kr,
                                   long long kh, long long vr, long long vh, int first, int hkv,
                                   __nv_bfloat16* ring_k, __nv_bfloat16* ring_v, int cap, int pos0) {
  const int i = first + blockIdx.x;
  const int slot = (int)(((long long)pos0 + i) % cap);
  for (int e = threadIdx.x; e < hkv * 16; e += blockDim.x) {
    const int h = e / 16, c = e % 16;
    const long long o = ((long long)h * cap + slot) * NKV_D + c * 8;
    *reinterpret_cast<uint4*>(ring_k + o) = *reinterpret_cast<const uint4*>(k + i * kr + h * kh + c * 8);
    *reinterpret_cast<uint4*>(ring_v + o) = *reinterpret_cast<const uint4*>(v + i * vr + h * vh + c * 8);
  }
}

}  // namespace nkv

using namespace nkv;

extern "C" int nkv_ring_append(nkv_stream_t stream, const void* k, const void* v, int T,
                               int64_t k_row_stride, int64_t k_head_stride, int64_t v_row_stride,
                               int64_t v_head_stride, int hkv, int head_dim, void* ring_k,
                               void* ring_v, int ring_cap, int ring_pos0) {
  NKV_SUPPORTED(head_dim == NKV_D, "ring_append: head_dim %d unsupported", head_dim);
  NKV_REQUIRE(ring_cap >= 1 && ring_pos0 >= 0 && hkv >= 1, "ring_append: bad ring");
  if (T <= 0) return NKV_OK;
  NKV_REQUIRE(k && v && ring_k && ring_v, "ring_append: null pointer");
  NKV_REQUIRE(((uintptr_t)k & 15) == 0 && ((uintptr_t)v & 15) == 0 && k_row_stride % 8 == 0 &&
                  k_head_stride % 8 == 0 && v_row_stride % 8 == 0 && v_head_stride % 8 == 0,
              "ring_append: k/v must be 16-byte aligned with strides multiple of 8 elements");
  const int first = T > ring_cap ? T - ring_cap : 0;
  ring_append_kernel<<<T - first, 128, 0, (cudaStream_t)stream>>>(
      (const __nv_bfloat16*)k, (const __nv_bfloat16*)v, k_row_stride, k_head_stride, v_row_stride,
      v_head_stride, first, hkv, (__nv_bfloat16*)ring_k, (__nv_bfloat16*)ring_v, ring_cap, ring_pos0);
  return check_launch("ring_append");
}

extern "C" int nkv_store_chunk(nkv_stream_t stream, const nkv_store_args* a) {
  NKV_REQUIRE(a, "store: null args");
  NKV_SUPPORTED(a->head_dim == NKV_D, "store: head_dim %d unsupported (128 only)", a->head_dim);
  NKV_SUPPORTED(a->block_size == 16 || a->block_size == 32 || a->block_size == 64 ||
                    a->block_size == 128,
                "store: block_size %d unsupported", a->block_size);
  NKV_SUPPORTED(a->r >= 1 && a->r <= 8 && a->r <= a->block_size, "store: r=%d unsupported", a->r);
  NKV_REQUIRE(a->T >= 1 && a->hkv >= 1, "store: empty chunk");
  const int nb = (a->T + a->block_size - 1) / a->block_size;
  NKV_REQUIRE(a->start_block >= 0 && a->start_block + nb <= a->max_blocks,
              "store: blocks [%d, %d) exceed the representative capacity %d", a->start_block,
              a->start_block + nb, a->max_blocks);
  NKV_REQUIRE(!a->k_store || a->start_block + nb <= a->store_blocks,
              "store: blocks [%d, %d) exceed the block-store capacity %d", a->start_block,
              a->start_block + nb, a->store_blocks);
  NKV_REQUIRE(a->k && a->v && a->reps, "store: null k/v/reps");
  NKV_REQUIRE((a->k_store == nullptr) == (a->v_store == nullptr),
              "store: k_store and v_store must both be set or both be NULL (reps only)");
  NKV_REQUIRE(a->store_kind >= 0 && a->store_kind <= 2, "store: bad store_kind");
  NKV_REQUIRE(!a->k_store || a->store_kind != NKV_STORE_INT8_REF || (a->k_chan_scale && a->v_block_scale),
              "store: int8 reference scheme needs k_chan_scale and v_block_scale");
  NKV_REQUIRE(!a->k_store || a->store_kind != NKV_STORE_INT8_TOKEN || (a->k_tok_scale && a->v_tok_scale),
              "store: int8 token scheme needs k_tok_scale and v_tok_scale");
  NKV_REQUIRE(a->sink_write <= 0 || (a->sink_k && a->sink_v && a->sink_write <= a->sink_cap),
              "store: bad sink arguments");
  NKV_REQUIRE(a->ring_cap <= 0 || (a->ring_k && a->ring_v && a->ring_pos0 >= 0),
              "store: bad ring arguments");
  NKV_REQUIRE(((uintptr_t)a->k & 15) == 0 && ((uintptr_t)a->v & 15) == 0 &&
                  a->k_row_stride % 8 == 0 && a->k_head_stride % 8 == 0 &&
                  a->v_row_stride % 8 == 0 && a->v_head_stride % 8 == 0,
              "store: k/v must be 16-byte aligned with strides multiple of 8 elements");
  StoreParams p;
  p.k = (const __nv_bfloat16*)a->k;
  p.v = (const __nv_bfloat16*)a->v;
  p.k_row = a->k_row_stride;
  p.k_head = a->k_head_stride;
  p.v_row = a->v_row_stride;
  p.v_head = a->v_head_stride;
  p.T = a->T;
  p.hkv = a->hkv;
  p.B = a->block_size;
  p.r = a->r;
  p.start_block = a->start_block;
  p.max_blocks = a->max_blocks;
  p.store_kind = a->store_kind;
  p.k_store = a->k_store;
  p.v_store = a->v_store;
  p.k_chan_scale = a->k_chan_scale;
  p.v_block_scale = a->v_block_scale;
  p.k_tok_scale = (__nv_bfloat16*)a->k_tok_scale;
  p.v_tok_scale = (__nv_bfloat16*)a->v_tok_scale;
  p.reps = (__nv_bfloat16*)a->reps;
  p.rep_index = a->rep_index;
  p.sink_k = (__nv_bfloat16*)a->sink_k;
  p.sink_v = (__nv_bfloat16*)a->sink_v;
  p.sink_cap = a->sink_cap;
  p.sink_write = a->sink_write > 0 ? a->sink_write : 0;
  p.ring_k = (__nv_bfloat16*)a->ring_k;
  p.ring_v = (__nv_bfloat16*)a->ring_v;
  p.ring_cap = a->ring_cap > 0 ? a->ring_cap : 0;
  p.ring_pos0 = a->ring_pos0;
  p.ring_first = a->ring_first;
  // K tile (bf16) + directions (fp32) + V tile (bf16, int8 kinds) + per-token and per-dim scratch
  const bool stage_v = a->k_store != nullptr && a->store_kind != NKV_STORE_BF16;
  const size_t tile_b = (size_t)a->block_size * NKV_D;
  const size_t smem = tile_b * 2 + tile_b * 4 + (stage_v ? tile_b * 2 : 0) + (2 * ST_MAXB + NKV_D + 8) * 4;
  dim3 grid(nb, a->hkv);
  if (a->block_size == SB64 && (!a->k_store || a->store_kind == NKV_STORE_BF16) && knob("NKV_STORE_B64", 1)) {
    const bool copy = a->k_store || p.sink_write > 0 || p.ring_cap > 0;
    if (copy && knob("NKV_STORE_FUSED", 1)) {  // copy and representatives in one grid
      store_reps_b64<true><<<grid, ST_THREADS, 0, (cudaStream_t)stream>>>(p);
      return check_launch("store_chunk");
    }
    if (copy) {
      const int units = nb * a->hkv;
      int ctas = knob("NKV_STORE_COPY_CTAS", 0);
      if (ctas <= 0) ctas = sm_count();
      store_copy_b64<<<ctas < units ? ctas : units, ST_THREADS, 0, (cudaStream_t)stream>>>(p, nb);
      const int rc = check_launch("store_chunk copy");
      if (rc != NKV_OK) return rc;
    }
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = copy ? 1 : 0;
    cudaLaunchConfig_t lc = {};
    lc.gridDim = grid;
    lc.blockDim = dim3(ST_THREADS);
    lc.stream = (cudaStream_t)stream;
    lc.attrs = attr;
    lc.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&lc, store_reps_b64<false>, p);
    if (e != cudaSuccess) {
      cudaGetLastError();
      set_error("store_chunk reps: launch failed: %s", cudaGetErrorString(e));
      return NKV_ERR_CUDA;
    }
    return check_launch("store_chunk reps");
  }
  if (ensure_smem(store_kernel, smem, "store_chunk")) return NKV_ERR_CUDA;
  store_kernel<<<grid, ST_THREADS, smem, (cudaStream_t)stream>>>(p);
  return check_launch("store_chunk");
}

extern "C" int nkv_k_channel_scale(nkv_stream_t stream, const void* k, int T, int64_t row_stride,
                                   int64_t head_stride, int hkv, int head_dim, float* out_scale) {
  NKV_REQUIRE(k && out_scale && T >= 1 && hkv >= 1, "k_channel_scale: bad arguments");
  NKV_SUPPORTED(head_dim == NKV_D, "k_channel_scale: head_dim %d unsupported", head_dim);
  kscale_kernel<<<hkv, 8 * NKV_D, 0, (cudaStream_t)stream>>>((const __nv_bfloat16*)k, T, row_stride,
                                                            head_stride, out_scale);
  return check_launch("k_channel_scale");
}

extern "C" int nkv_query_summaries(nkv_stream_t stream, const void* q, int T, int64_t row_stride,
                                   int64_t head_stride, int hq, int head_dim, int nseg, void* out) {
  NKV_REQUIRE(q && out && T >= 1 && hq >= 1 && nseg >= 1, "query_summaries: bad arguments");
  NKV_SUPPORTED(head_dim == NKV_D, "query_summaries: head_dim %d unsupported", head_dim);
  if (nseg > T) nseg = T;
  dim3 grid(nseg, hq);
  qsum_kernel<<<grid, NKV_D, 0, (cudaStream_t)stream>>>((const __nv_bfloat16*)q, T, row_stride,
                                                       head_stride, nseg, (__nv_bfloat16*)out);
  return check_launch("query_summaries");
}

extern "C" int nkv_store_kvcache(nkv_stream_t stream, const void* key, int64_t key_stride,
                                 const void* value, int64_t value_stride, void* k_cache,
                                 void* v_cache, const int64_t* slot_mapping, int n, int row_elems) {
  NKV_REQUIRE(row_elems >= 1, "store_kvcache: bad row size");
  if (n <= 0) return NKV_OK;
  NKV_REQUIRE(key && value && k_cache && v_cache && slot_mapping, "store_kvcache: null pointer");
  kvcache_kernel<<<n, 128, 0, (cudaStream_t)stream>>>(
      (const __nv_bfloat16*)key, key_stride, (const __nv_bfloat16*)value, value_stride,
      (__nv_bfloat16*)k_cache, (__nv_bfloat16*)v_cache, (const long long*)slot_mapping, row_elems);
  return check_launch("store_kvcache");
}

// ---------------------------------------------------------------------------
// Self-test of div_rcp: out[i] = a[i] / b[i] by the store kernel's division
// (b[i] > 0 normal).  Tests compare it with the division operator.
// ---------------------------------------------------------------------------
namespace nkv {
__global__ void selftest_div_kernel(const float* a, const float* b, float* out, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = div_rcp(a[i], b[i], __frcp_rn(b[i]));
}
}  // namespace nkv

extern "C" int nkv_selftest_div(nkv_stream_t stream, const float* a, const float* b, float* out, int n) {
  NKV_REQUIRE(a && b && out && n >= 0, "selftest_div: bad arguments");
  if (n == 0) return NKV_OK;
  nkv::selftest_div_kernel<<<(n + 255) / 256, 256, 0, (cudaStream_t)stream>>>(a, b, out, n);
  return nkv::check_launch("selftest_div");
}
