// Kernel (4): segmented prefill attention on the tensor cores.
//
// One chunk of nq query positions (nq == n_cur) attends, per KV head, to the
// logical keys [selected blocks | sink | recent ring slice | current chunk]
// (the reference's pack order, m12_runtime.py:589-642), read in place from
// their four sources.  History keys are visible to every query; current key j
// is visible to query n when j <= n + (n_cur - nq) (causal, bottom-right
// aligned, as flash_attn_func(causal=True) at m12_runtime.py:834-839).
//
// Grid (position tiles, hkv).  A CTA owns 128 query rows = 128 / G positions
// x the G query heads of one KV head, so every K/V tile it loads serves all G
// heads.  Per 64-key tile:
//   loads:  K and V rows gathered by 16-byte cp.async into 128-byte-swizzled
//           [2][64][128 B] tiles (double buffered: tile t+1 loads while t is
//           computed); keys past the visible range read a valid stand-in row
//           and are masked.
//   math:   each of the 8 warps owns 16 query rows.  S = Q K^T with mma.sync
//           m16n8k16 (Q fragments held in registers for the whole loop, K via
//           ldmatrix), online softmax in the exp2 domain on the accumulator
//           fragments, O += P V with P re-packed as the bf16 A operand and V
//           via ldmatrix.trans.  fp32 accumulation throughout.
// Position tiles are scheduled last-first (they see the most keys).
#include <stdlib.h>
#include <string.h>

#include "nkv_common.cuh"
#include "nkv_host.h"

namespace nkv {

constexpr int PF_THREADS = 256;
constexpr int PF_ROWS = 128;  // query rows per CTA (positions x G)
constexpr int PF_KT = 64;     // keys per tile
constexpr size_t PF_SMEM = 1024 + PF_ROWS * 256 + 2 * 2 * PF_KT * 256;  // align + Q + 2 x (K, V)

struct PrefillParams {
  const __nv_bfloat16* q;
  long long q_row, q_head;
  int nq, hkv, B, log2B;
  float sl2;  // softmax scale * log2(e)
  const long long* ids;
  int n_sel, max_blocks, kind;
  const __nv_bfloat16* k_store;  // bf16 store (kind NKV_STORE_BF16)
  const __nv_bfloat16* v_store;
  const signed char* k_q;        // int8 store (the two int8 kinds)
  const signed char* v_q;
  const float* kcs;              // reference scheme: K scale [hkv][D], V scale [blocks][hkv]
  const float* vbs;
  const __nv_bfloat16* kts;      // token scheme: bf16 scale per (block, head, token)
  const __nv_bfloat16* vts;
  const __nv_bfloat16* sink_k;
  const __nv_bfloat16* sink_v;
  int sink_cap, sink_len;
  const __nv_bfloat16* ring_k;
  const __nv_bfloat16* ring_v;
  int ring_cap, ring_start, ring_len;
  const __nv_bfloat16* cur_k;
  const __nv_bfloat16* cur_v;
  long long cur_row, cur_head;
  int n_cur;
  __nv_bfloat16* out;
  long long out_row, out_head;
  int* err;
};

// Dequantised 8 values (16 bytes of bf16) of an int8 selected key: dims
// [c*8, c*8+8) of key `key` (< selEnd) of head h, in the reference's rounding
// (each product rounded to bf16, quant_kv.py / m12_runtime.py:1243-1278).
__device__ __forceinline__ void int8_chunk(const PrefillParams& p, int h, int key, int c, uint4* kout,
                                           uint4* vout) {
  long long id = __ldg(p.ids + (key >> p.log2B));
  if (id < 0 || id >= p.max_blocks) {
    if (p.err) atomicExch(p.err, ERR_BAD_INDEX);
    id = 0;
  }
  const int off = key & (p.B - 1);
  const long long o = ((id * p.hkv + h) * p.B + off) * NKV_D + c * 8;
  const uint2 kr = __ldg(reinterpret_cast<const uint2*>(p.k_q + o));
  const uint2 vr = __ldg(reinterpret_cast<const uint2*>(p.v_q + o));
  const signed char* kb = reinterpret_cast<const signed char*>(&kr);
  const signed char* vb = reinterpret_cast<const signed char*>(&vr);
  uint32_t kw[4], vw[4];
  if (p.kind == NKV_STORE_INT8_REF) {
    const float vsc = __ldg(p.vbs + id * p.hkv + h);
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
      const int d = c * 8 + e;
      kw[e / 2] = (uint32_t)f2bf((float)kb[e] * __ldg(p.kcs + h * NKV_D + d)) |
                  ((uint32_t)f2bf((float)kb[e + 1] * __ldg(p.kcs + h * NKV_D + d + 1)) << 16);
      vw[e / 2] = (uint32_t)f2bf((float)vb[e] * vsc) | ((uint32_t)f2bf((float)vb[e + 1] * vsc) << 16);
    }
  } else {
    const long long so = (id * p.hkv + h) * p.B + off;
    const float ksc = __bfloat162float(p.kts[so]), vsc = __bfloat162float(p.vts[so]);
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
      kw[e / 2] = (uint32_t)f2bf((float)kb[e] * ksc) | ((uint32_t)f2bf((float)kb[e + 1] * ksc) << 16);
      vw[e / 2] = (uint32_t)f2bf((float)vb[e] * vsc) | ((uint32_t)f2bf((float)vb[e + 1] * vsc) << 16);
    }
  }
  *kout = make_uint4(kw[0], kw[1], kw[2], kw[3]);
  *vout = make_uint4(vw[0], vw[1], vw[2], vw[3]);
}

// Source rows of logical key `key` of head h (K and V).
__device__ __forceinline__ void key_rows(const PrefillParams& p, int h, int key, int selEnd, int sinkEnd,
                                         int ringEnd, const __nv_bfloat16** kr, const __nv_bfloat16** vr) {
  if (key < selEnd) {
    long long id = __ldg(p.ids + (key >> p.log2B));
    if (id < 0 || id >= p.max_blocks) {
      if (p.err) atomicExch(p.err, ERR_BAD_INDEX);
      id = 0;
    }
    const long long o = ((id * p.hkv + h) * p.B + (key & (p.B - 1))) * NKV_D;
    *kr = p.k_store + o;
    *vr = p.v_store + o;
  } else if (key < sinkEnd) {
    const long long o = ((long long)h * p.sink_cap + (key - selEnd)) * NKV_D;
    *kr = p.sink_k + o;
    *vr = p.sink_v + o;
  } else if (key < ringEnd) {
    int phys = p.ring_start + (key - sinkEnd);
    if (phys >= p.ring_cap) phys -= p.ring_cap;
    const long long o = ((long long)h * p.ring_cap + phys) * NKV_D;
    *kr = p.ring_k + o;
    *vr = p.ring_v + o;
  } else {
    const long long o = (long long)(key - ringEnd) * p.cur_row + (long long)h * p.cur_head;
    *kr = p.cur_k + o;
    *vr = p.cur_v + o;
  }
}

template <int G>
__global__ void __launch_bounds__(PF_THREADS, 1) prefill_kernel(const PrefillParams p) {
  extern __shared__ __align__(16) unsigned char sm_raw[];
  unsigned char* sm = sm_raw + ((1024u - (smem_u32(sm_raw) & 1023u)) & 1023u);
  unsigned char* qs = sm;                   // [2][128][128 B]
  unsigned char* kvs = sm + PF_ROWS * 256;  // 2 buffers x (K [2][64][128 B], V [2][64][128 B])
  constexpr int P = PF_ROWS / G;            // positions per CTA

  const int tile = (int)gridDim.x - 1 - (int)blockIdx.x;
  const int h = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int p0 = tile * P;
  const int selEnd = p.n_sel * p.B, sinkEnd = selEnd + p.sink_len, ringEnd = sinkEnd + p.ring_len;
  const int off = p.n_cur - p.nq;  // current key j visible to position n iff j <= n + off
  const int last_pos = min(p.nq, p0 + P) - 1;
  const int visEnd = ringEnd + min(p.n_cur, last_pos + off + 1);  // keys the tile's last position sees
  const int allFrom = ringEnd + min(p.n_cur, max(0, p0 + off + 1));  // keys below: seen by every row
  const int ntk = (visEnd + PF_KT - 1) / PF_KT;

  // ---- Q tile: row r = position p0 + r / G, query head h * G + r % G ---------------------
  for (int i = tid; i < PF_ROWS * 16; i += PF_THREADS) {
    const int r = i >> 4, c = i & 15, pos = p0 + r / G;
    unsigned char* dst = qs + swz(PF_ROWS, r, c * 8);
    if (pos < p.nq)
      cp_async16(dst, p.q + (long long)pos * p.q_row + (long long)(h * G + r % G) * p.q_head + c * 8);
    else
      *reinterpret_cast<uint4*>(dst) = make_uint4(0u, 0u, 0u, 0u);
  }
  cp_async_commit();

  auto load_tile = [&](int t, int buf) {
    unsigned char* kt = kvs + buf * (2 * PF_KT * 256);
    unsigned char* vt = kt + PF_KT * 256;
#pragma unroll
    for (int it = 0; it < PF_KT * 16 / PF_THREADS; ++it) {
      const int i = tid + it * PF_THREADS;
      const int r = i >> 4, c = i & 15;
      int key = t * PF_KT + r;
      if (key >= visEnd) key = t * PF_KT;  // finite stand-in, masked below
      if (key < selEnd && p.kind != NKV_STORE_BF16) {  // int8 history: dequant on the way in
        uint4 kq, vq;
        int8_chunk(p, h, key, c, &kq, &vq);
        *reinterpret_cast<uint4*>(kt + swz(PF_KT, r, c * 8)) = kq;
        *reinterpret_cast<uint4*>(vt + swz(PF_KT, r, c * 8)) = vq;
        continue;
      }
      const __nv_bfloat16 *kr, *vr;
      key_rows(p, h, key, selEnd, sinkEnd, ringEnd, &kr, &vr);
      cp_async16(kt + swz(PF_KT, r, c * 8), kr + c * 8);
      cp_async16(vt + swz(PF_KT, r, c * 8), vr + c * 8);
    }
  };
  if (ntk > 0) load_tile(0, 0);
  cp_async_commit();
  cp_async_wait<1>();  // the Q tile
  __syncthreads();

  // Q fragments (A operand) of this warp's 16 rows, all 8 k-steps
  uint32_t qa[8][4];
  {
    const int row = warp * 16 + ((lane >> 3) & 1) * 8 + (lane & 7);
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) ldsm_x4(qa[kk], qs + swz(PF_ROWS, row, kk * 16 + (lane >> 4) * 8));
  }

  const int qg = lane >> 2, qt = lane & 3;
  const int mrow = lane & 7, msel = lane >> 3;
  const int pos0 = p0 + (warp * 16 + qg) / G, pos1 = p0 + (warp * 16 + qg + 8) / G;
  float o[16][4];
#pragma unroll
  for (int d = 0; d < 16; ++d) o[d][0] = o[d][1] = o[d][2] = o[d][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

  for (int t = 0; t < ntk; ++t) {
    const int buf = t & 1;
    if (t + 1 < ntk) load_tile(t + 1, buf ^ 1);
    cp_async_commit();
    cp_async_wait<1>();  // tile t
    __syncthreads();
    const unsigned char* kt = kvs + buf * (2 * PF_KT * 256);
    const unsigned char* vt = kt + PF_KT * 256;

    // S = Q K^T: 8 n-tiles of 8 keys
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 8; kk += 2) {
      uint32_t b[8][4];
#pragma unroll
      for (int j = 0; j < 8; ++j) ldsm_x4(b[j], kt + swz(PF_KT, j * 8 + mrow, (kk + (msel >> 1)) * 16 + (msel & 1) * 8));
#pragma unroll
      for (int j = 0; j < 8; ++j) mma_bf16(s[j], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b[j][0], b[j][1]);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        mma_bf16(s[j], qa[kk + 1][0], qa[kk + 1][1], qa[kk + 1][2], qa[kk + 1][3], b[j][2], b[j][3]);
    }
    // scale to the exp2 domain and mask; c0,c1 are row qg, c2,c3 row qg + 8
    const int kbase = t * PF_KT;
    const bool need_mask = kbase + PF_KT > allFrom;
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float x = s[j][e] * p.sl2;
        if (need_mask) {
          const int key = kbase + j * 8 + 2 * qt + (e & 1);
          const int pos = e < 2 ? pos0 : pos1;
          if (key >= ringEnd && key - ringEnd > pos + off) x = -INFINITY;
        }
        s[j][e] = x;
      }
    // online softmax
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      mx0 = fmaxf(mx0, fmaxf(s[j][0], s[j][1]));
      mx1 = fmaxf(mx1, fmaxf(s[j][2], s[j][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(FULL, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(FULL, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(FULL, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(FULL, mx1, 2));
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float base0 = mn0 == -INFINITY ? 0.f : mn0, base1 = mn1 == -INFINITY ? 0.f : mn1;
    const float al0 = exp2f(m0 - base0), al1 = exp2f(m1 - base1);  // 0 while m is -inf
    m0 = mn0;
    m1 = mn1;
    float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      s[j][0] = exp2f(s[j][0] - base0);
      s[j][1] = exp2f(s[j][1] - base0);
      s[j][2] = exp2f(s[j][2] - base1);
      s[j][3] = exp2f(s[j][3] - base1);
      rs0 += s[j][0] + s[j][1];
      rs1 += s[j][2] + s[j][3];
    }
    l0 = l0 * al0 + rs0;  // per-thread partial row sums (reduced over the quad at the end)
    l1 = l1 * al1 + rs1;
#pragma unroll
    for (int d = 0; d < 16; ++d) {
      o[d][0] *= al0;
      o[d][1] *= al0;
      o[d][2] *= al1;
      o[d][3] *= al1;
    }
    // O += P V: 4 k-steps of 16 keys
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      const uint32_t a0 = pack_bf16x2(s[2 * ks][0], s[2 * ks][1]);
      const uint32_t a1 = pack_bf16x2(s[2 * ks][2], s[2 * ks][3]);
      const uint32_t a2 = pack_bf16x2(s[2 * ks + 1][0], s[2 * ks + 1][1]);
      const uint32_t a3 = pack_bf16x2(s[2 * ks + 1][2], s[2 * ks + 1][3]);
      const int row = ks * 16 + (msel & 1) * 8 + mrow;
      uint32_t b[8][4];
#pragma unroll
      for (int dn2 = 0; dn2 < 8; ++dn2) ldsm_x4_t(b[dn2], vt + swz(PF_KT, row, dn2 * 16 + (msel >> 1) * 8));
#pragma unroll
      for (int dn2 = 0; dn2 < 8; ++dn2) {
        mma_bf16(o[2 * dn2], a0, a1, a2, a3, b[dn2][0], b[dn2][1]);
        mma_bf16(o[2 * dn2 + 1], a0, a1, a2, a3, b[dn2][2], b[dn2][3]);
      }
    }
    __syncthreads();  // buffer `buf` is refilled by the next iteration's prefetch
  }
  cp_async_wait<0>();

  l0 += __shfl_xor_sync(FULL, l0, 1);
  l0 += __shfl_xor_sync(FULL, l0, 2);
  l1 += __shfl_xor_sync(FULL, l1, 1);
  l1 += __shfl_xor_sync(FULL, l1, 2);
  const float inv0 = 1.f / l0, inv1 = 1.f / l1;
  const int g0 = (warp * 16 + qg) % G, g1 = (warp * 16 + qg + 8) % G;
  if (pos0 < p.nq) {
    __nv_bfloat16* dst = p.out + (long long)pos0 * p.out_row + (long long)(h * G + g0) * p.out_head + 2 * qt;
#pragma unroll
    for (int d = 0; d < 16; ++d)
      *reinterpret_cast<uint32_t*>(dst + d * 8) = pack_bf16x2(o[d][0] * inv0, o[d][1] * inv0);
  }
  if (pos1 < p.nq) {
    __nv_bfloat16* dst = p.out + (long long)pos1 * p.out_row + (long long)(h * G + g1) * p.out_head + 2 * qt;
#pragma unroll
    for (int d = 0; d < 16; ++d)
      *reinterpret_cast<uint32_t*>(dst + d * 8) = pack_bf16x2(o[d][2] * inv1, o[d][3] * inv1);
  }
}

}  // namespace nkv

using namespace nkv;

namespace nkv {
// Selected blocks of one prefill call copied into a device bf16 staging store
// [n_sel][hkv][B][D] (staging block i = history block ids[i]), dequantised on
// the way with int8_chunk's rounding.  Grid (n_sel, hkv): one CTA per
// (block, head) tile, every thread's loads issued before its stores.
constexpr int GD_THREADS = 256;
__global__ void __launch_bounds__(GD_THREADS) gather_blocks_kernel(const PrefillParams p, __nv_bfloat16* sk,
                                                                   __nv_bfloat16* sv) {
  const int i = blockIdx.x, h = blockIdx.y;
  const int nchunks = p.B * (NKV_D / 8);
  const long long dst = ((long long)i * p.hkv + h) * p.B * NKV_D;
  constexpr int PER = 4;  // chunks per thread and pass (B <= 128: at most two passes)
  for (int base = threadIdx.x; base < nchunks; base += GD_THREADS * PER) {
    uint4 kw[PER], vw[PER];
#pragma unroll
    for (int u = 0; u < PER; ++u) {
      const int ch = base + u * GD_THREADS;
      if (ch >= nchunks) continue;
      const int row = ch >> 4, c = ch & 15;
      const int key = i * p.B + row;
      if (p.kind == NKV_STORE_BF16) {
        long long id = __ldg(p.ids + i);
        if (id < 0 || id >= p.max_blocks) {
          if (p.err) atomicExch(p.err, ERR_BAD_INDEX);
          id = 0;
        }
        const long long o = ((id * p.hkv + h) * p.B + row) * NKV_D + c * 8;
        kw[u] = __ldg(reinterpret_cast<const uint4*>(p.k_store + o));
        vw[u] = __ldg(reinterpret_cast<const uint4*>(p.v_store + o));
      } else {
        int8_chunk(p, h, key, c, &kw[u], &vw[u]);
      }
    }
#pragma unroll
    for (int u = 0; u < PER; ++u) {
      const int ch = base + u * GD_THREADS;
      if (ch >= nchunks) continue;
      *reinterpret_cast<uint4*>(sk + dst + (long long)ch * 8) = kw[u];
      *reinterpret_cast<uint4*>(sv + dst + (long long)ch * 8) = vw[u];
    }
  }
}
}  // namespace nkv

extern "C" int nkv_prefill_gather(nkv_stream_t stream, const nkv_attend_args* a, void* k_out, void* v_out) {
  NKV_REQUIRE(a && k_out && v_out, "prefill_gather: null arguments");
  NKV_SUPPORTED(a->head_dim == NKV_D, "prefill_gather: head_dim %d unsupported (128 only)", a->head_dim);
  NKV_REQUIRE(a->store_kind >= 0 && a->store_kind <= 2, "prefill_gather: bad store_kind");
  NKV_REQUIRE(a->n_sel >= 1 && a->block_ids && a->k_store && a->v_store && a->max_blocks > 0 && a->hkv >= 1,
              "prefill_gather: needs selected blocks, their ids and the block store");
  NKV_SUPPORTED((a->block_size & (a->block_size - 1)) == 0 && a->block_size >= 16 && a->block_size <= 128,
                "prefill_gather: block_size %d unsupported (16, 32, 64 or 128)", a->block_size);
  NKV_REQUIRE(a->store_kind != NKV_STORE_INT8_REF || (a->k_chan_scale && a->v_block_scale),
              "prefill_gather: int8 reference scheme needs its scales");
  NKV_REQUIRE(a->store_kind != NKV_STORE_INT8_TOKEN || (a->k_tok_scale && a->v_tok_scale),
              "prefill_gather: int8 token scheme needs its scales");
  NKV_REQUIRE(((uintptr_t)a->k_store & 15) == 0 && ((uintptr_t)a->v_store & 15) == 0 &&
                  ((uintptr_t)k_out & 15) == 0 && ((uintptr_t)v_out & 15) == 0,
              "prefill_gather: stores must be 16-byte aligned");
  NKV_REQUIRE(a->workspace && a->workspace_bytes >= 256, "prefill_gather: workspace (error word) missing");
  PrefillParams p;
  memset(&p, 0, sizeof(p));
  p.hkv = a->hkv;
  p.B = a->block_size;
  p.log2B = 0;
  while ((1 << p.log2B) < a->block_size) ++p.log2B;
  p.ids = (const long long*)a->block_ids;
  p.n_sel = a->n_sel;
  p.max_blocks = a->max_blocks;
  p.kind = a->store_kind;
  p.k_store = (const __nv_bfloat16*)a->k_store;
  p.v_store = (const __nv_bfloat16*)a->v_store;
  p.k_q = (const signed char*)a->k_store;
  p.v_q = (const signed char*)a->v_store;
  p.kcs = a->k_chan_scale;
  p.vbs = a->v_block_scale;
  p.kts = (const __nv_bfloat16*)a->k_tok_scale;
  p.vts = (const __nv_bfloat16*)a->v_tok_scale;
  p.err = (int*)a->workspace;
  gather_blocks_kernel<<<dim3(a->n_sel, a->hkv), GD_THREADS, 0, (cudaStream_t)stream>>>(
      p, (__nv_bfloat16*)k_out, (__nv_bfloat16*)v_out);
  return check_launch("prefill_gather");
}

extern "C" size_t nkv_prefill_workspace_bytes(int hkv, int hq, int nq, int max_tokens) {
  (void)hkv;
  (void)hq;
  (void)nq;
  (void)max_tokens;
  return 256;  // the error word
}

extern "C" int nkv_prefill(nkv_stream_t stream, const nkv_attend_args* a) {
  NKV_REQUIRE(a, "prefill: null args");
  NKV_SUPPORTED(a->head_dim == NKV_D, "prefill: head_dim %d unsupported (128 only)", a->head_dim);
  NKV_REQUIRE(a->hkv >= 1 && a->hq % a->hkv == 0, "prefill: hq %d not a multiple of hkv %d", a->hq, a->hkv);
  const int G = a->hq / a->hkv;
  NKV_SUPPORTED(G == 1 || G == 2 || G == 4 || G == 8, "prefill: G=%d unsupported", G);
  NKV_REQUIRE(a->nq >= 1 && a->n_cur == a->nq, "prefill: n_cur (%d) must equal nq (%d)", a->n_cur, a->nq);
  NKV_REQUIRE(a->store_kind >= 0 && a->store_kind <= 2, "prefill: bad store_kind");
  NKV_REQUIRE(a->store_kind != NKV_STORE_INT8_REF || a->n_sel == 0 || (a->k_chan_scale && a->v_block_scale),
              "prefill: int8 reference scheme needs its scales");
  NKV_REQUIRE(a->store_kind != NKV_STORE_INT8_TOKEN || a->n_sel == 0 || (a->k_tok_scale && a->v_tok_scale),
              "prefill: int8 token scheme needs its scales");
  NKV_SUPPORTED(a->allowed == nullptr, "prefill: per-query allowed mask unsupported");
  NKV_REQUIRE(a->block_size >= 1 && a->n_sel >= 0 && a->sink_len >= 0 && a->ring_len >= 0,
              "prefill: negative segment length");
  NKV_SUPPORTED((a->block_size & (a->block_size - 1)) == 0 && a->block_size >= 16 && a->block_size <= 128,
                "prefill: block_size %d unsupported (16, 32, 64 or 128)", a->block_size);
  NKV_REQUIRE(a->n_sel == 0 || (a->block_ids && a->k_store && a->v_store && a->max_blocks > 0),
              "prefill: selected segment needs block_ids and the block store");
  NKV_REQUIRE(a->sink_len == 0 || (a->sink_k && a->sink_v && a->sink_len <= a->sink_cap), "prefill: bad sink");
  NKV_REQUIRE(a->ring_len == 0 || (a->ring_k && a->ring_v && a->ring_len <= a->ring_cap && a->ring_start >= 0 &&
                                   a->ring_start < a->ring_cap),
              "prefill: bad ring slice");
  NKV_REQUIRE(a->q && a->out && a->cur_k && a->cur_v && a->workspace && a->workspace_bytes >= 256,
              "prefill: null pointer or workspace too small");
  NKV_REQUIRE(((uintptr_t)a->q & 15) == 0 && ((uintptr_t)a->cur_k & 15) == 0 && ((uintptr_t)a->cur_v & 15) == 0 &&
                  ((uintptr_t)a->k_store & 15) == 0 && ((uintptr_t)a->v_store & 15) == 0 &&
                  ((uintptr_t)a->sink_k & 15) == 0 && ((uintptr_t)a->sink_v & 15) == 0 &&
                  ((uintptr_t)a->ring_k & 15) == 0 && ((uintptr_t)a->ring_v & 15) == 0 &&
                  a->q_row_stride % 8 == 0 && a->q_head_stride % 8 == 0 && a->cur_row_stride % 8 == 0 &&
                  a->cur_head_stride % 8 == 0,
              "prefill: inputs must be 16-byte aligned with strides multiple of 8 elements");
  NKV_REQUIRE(((uintptr_t)a->out & 3) == 0 && a->out_row_stride % 2 == 0 && a->out_head_stride % 2 == 0,
              "prefill: out must be 4-byte aligned with even strides");
  const long long ntok = (long long)a->n_sel * a->block_size + a->sink_len + a->ring_len + a->n_cur;
  NKV_REQUIRE(ntok < (1ll << 30), "prefill: key count %lld out of range", ntok);

  PrefillParams p;
  p.q = (const __nv_bfloat16*)a->q;
  p.q_row = a->q_row_stride;
  p.q_head = a->q_head_stride;
  p.nq = a->nq;
  p.hkv = a->hkv;
  p.B = a->block_size;
  p.log2B = 0;
  while ((1 << p.log2B) < a->block_size) ++p.log2B;
  p.sl2 = a->scale * 1.4426950408889634f;
  p.ids = (const long long*)a->block_ids;
  p.n_sel = a->n_sel;
  p.max_blocks = a->max_blocks;
  p.kind = a->store_kind;
  p.k_store = (const __nv_bfloat16*)a->k_store;
  p.v_store = (const __nv_bfloat16*)a->v_store;
  p.k_q = (const signed char*)a->k_store;
  p.v_q = (const signed char*)a->v_store;
  p.kcs = a->k_chan_scale;
  p.vbs = a->v_block_scale;
  p.kts = (const __nv_bfloat16*)a->k_tok_scale;
  p.vts = (const __nv_bfloat16*)a->v_tok_scale;
  p.sink_k = (const __nv_bfloat16*)a->sink_k;
  p.sink_v = (const __nv_bfloat16*)a->sink_v;
  p.sink_cap = a->sink_cap;
  p.sink_len = a->sink_len;
  p.ring_k = (const __nv_bfloat16*)a->ring_k;
  p.ring_v = (const __nv_bfloat16*)a->ring_v;
  p.ring_cap = a->ring_cap;
  p.ring_start = a->ring_start;
  p.ring_len = a->ring_len;
  p.cur_k = (const __nv_bfloat16*)a->cur_k;
  p.cur_v = (const __nv_bfloat16*)a->cur_v;
  p.cur_row = a->cur_row_stride;
  p.cur_head = a->cur_head_stride;
  p.n_cur = a->n_cur;
  p.out = (__nv_bfloat16*)a->out;
  p.out_row = a->out_row_stride;
  p.out_head = a->out_head_stride;
  p.err = (int*)a->workspace;

  cudaStream_t st = (cudaStream_t)stream;
  // the tcgen05/TMEM kernel takes every call it supports (NKV_PREFILL_TC=0: never)
  if (knob("NKV_PREFILL_TC", 1) != 0) {
    const int rc = prefill_tc(st, a);
    if (rc != NKV_ERR_UNSUPPORTED) return rc;
  }
  const int P = PF_ROWS / G;
  dim3 grid((a->nq + P - 1) / P, a->hkv);
  switch (G) {
#define NKV_PF_CASE(GG)                                                            \
  case GG:                                                                         \
    if (ensure_smem(prefill_kernel<GG>, PF_SMEM, "prefill")) return NKV_ERR_CUDA; \
    prefill_kernel<GG><<<grid, PF_THREADS, PF_SMEM, st>>>(p);                      \
    break;
    NKV_PF_CASE(1)
    NKV_PF_CASE(2)
    NKV_PF_CASE(4)
    NKV_PF_CASE(8)
#undef NKV_PF_CASE
    default:
      return NKV_ERR_UNSUPPORTED;
  }
  return check_launch("prefill");
}
