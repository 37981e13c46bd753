// Kernels (2)+(3): fused gather-and-attend GQA attention over the sparse key set.
//
// Logical keys of one KV head, in the reference's packed order
// (m12_runtime.py:1240-1308 decode, :716-749 verify):
//   [ selected blocks (block_ids order) | sink | recent ring slice | current ]
// They are never packed.  The grid is (splits, hkv); CTA (s, h) owns logical
// keys [s*tps, (s+1)*tps) of head h.  Two kernels share that structure:
//
//  decode_kernel (nq == 1, the hot path): the CTA's keys are fetched by 2D TMA
//  (64- and 8-row boxes, 128-byte swizzle) into shared memory, one mbarrier per
//  contiguous piece; int8, host-resident and current-token rows are loaded by
//  the threads into the same layout.  Q.K and P.V run on the tensor cores
//  (mma.sync m16n8k16, bf16 in, fp32 accumulate), one slice of <= 48 keys per
//  warp.  The splits of a head form one thread-block cluster (<= 16 CTAs) and
//  merge through DSMEM, or go through the workspace.
//
//  attend_kernel (nq > 1, verify): one cp.async.bulk per contiguous piece for
//  bf16 data or 128-bit loads + in-register dequant for an int8 store; scores
//  all keys for the nq*G query rows (causal for current tokens, the per-row
//  allowed mask for selected blocks), fp32 softmax and P.V, the same merges.
//
// Merges use the log-sum-exp rule and write bf16.  Without a cluster, the last
// CTA of a head (atomic ticket, no spinning) merges the workspace partials.
#include <cooperative_groups.h>
#include <cuda.h>  // CUtensorMap (encoded through the runtime's driver entry point)
#include <stdlib.h>
#include <string.h>

#include <mutex>

#include "nkv_common.cuh"
#include "nkv_host.h"

namespace cg = cooperative_groups;

namespace nkv {

constexpr int AT_THREADS = 256;
constexpr int AT_WARPS = AT_THREADS / 32;
// single-query decode kernel: 16 warps hide the Q.K latency chains; G = 8 needs
// the registers of a 256-thread launch
#ifndef NKV_DECODE_WARPS
#define NKV_DECODE_WARPS 8
#endif
template <int G> struct DK { static constexpr int WARPS = NKV_DECODE_WARPS, THREADS = WARPS * 32; };
constexpr int AT_TPS_MAX = 256;  // keys per CTA (K+V tiles: 128 KiB)
constexpr int AT_MIN_TPS = 16;
constexpr int AT_CLUSTER_MAX = 16;        // splits of one head merged through DSMEM
constexpr int AT_TPS_MAX_CLUSTER = 384;   // keys per CTA in cluster mode (K+V: 192 KiB)
constexpr int AT_MAX_SLOTS = 32;          // block slots one CTA can touch (tps / B + 2)
constexpr int AT_MAX_PIECES = AT_MAX_SLOTS + 8;  // + sink, two ring pieces, current tokens
// Bound of a wait on another GPU's words (~1 s of SM clock): the peers run
// their own launches, so their host-side skew is part of what is waited for.
constexpr long long PEER_WAIT_CYCLES = 2000000000ll;

struct AttendParams {
  const __nv_bfloat16* q;
  long long q_row, q_head;
  int nq, hkv, B;
  float scale;
  const long long* ids;
  int n_sel, max_blocks, kind;
  const void* k_store;
  const void* v_store;
  const float* kcs;
  const float* vbs;
  const __nv_bfloat16* kts;
  const __nv_bfloat16* vts;
  const unsigned char* allowed;
  int allowed_stride;
  const __nv_bfloat16* sink_k;
  const __nv_bfloat16* sink_v;
  int sink_cap, sink_len;
  __nv_bfloat16* ring_k;
  __nv_bfloat16* ring_v;
  int ring_cap, ring_start, ring_len;
  const __nv_bfloat16* cur_k;
  const __nv_bfloat16* cur_v;
  long long cur_row, cur_head;
  int n_cur, ring_write_pos;
  __nv_bfloat16* out;
  long long out_row, out_head;
  float* part_o;       // [hkv][splits][nr][D]
  float* part_ml;      // [hkv][splits][nr][2]
  unsigned* counters;  // [hkv]
  int* err;
  int splits, tps, ntok, nr, nr_pad;
  // buffer extents in elements (checked builds)
  long long ext_store, ext_sink, ext_ring, ext_cur, ext_q, ext_out, ext_part_o, ext_part_ml;
  int* trace;  // checked builds: per-CTA record of parameters and pieces (or null)
  int overlap;  // 1: wait for the preceding (select) grid before touching ids
  int cluster;  // 1: the splits of a head form one thread-block cluster (DSMEM merge)
  int log2B;    // block_size is a power of two
  // decode kernel: tile rows per K (or V) tile, bytes of the K-tile region,
  // segments TMA may read (1 selected blocks, 2 sink, 4 ring: bf16 in device memory)
  int tile_rows, region_k, tma_mask;
  // decode kernel, ranked mode: the CTAs rank these block scores (written by
  // the preceding scoring grid) themselves instead of reading ids
  const float* rank_scores;
  // decode kernel, device-resident ring head (graph replay): ring_dyn[0] is
  // the ring slot of logical recent slot 0 (the slot the current token is
  // written to), ring_dyn[1] counts arriving CTAs; the last CTA to arrive
  // advances the head.  Null: ring_start / ring_write_pos as given.
  int* ring_dyn;
  int sel_thr_every;  // decode kernel: 0, or every n-th selected piece loaded by the threads
  int rank_n;
  long long* rank_out;     // the ranked ids, written by CTA (0, 0)
  float* rank_out_scores;  // their scores (optional)
  // decode kernel, one-launch step (fs_keys set, rank_scores null): the CTAs
  // also score the blocks (CTA c of the grid owns blocks [c * fs_bpc, ...) for
  // every KV head), publish each block's masked score as a key tagged with
  // this launch's epoch, and select the top n_sel of the rank_n keys
  // themselves once every key carries the tag
  const __nv_bfloat16* fs_reps;  // [hkv][fs_reps_blocks][fs_r][D]
  int fs_r, fs_reps_blocks, fs_bpc, fs_nprot;
  int fs_prefetch;  // 1: each CTA starts an L2 prefetch of its representatives at launch
  const int* fs_prot;
  unsigned long long* fs_keys;  // [rank_n]: (tag << 32) | orderable score
  unsigned* fs_sync;            // [0] epoch, [1] CTAs done with this launch's keys
  // KV-head sharding over peer memory (xp_P > 0, ranked decode): the ranking
  // CTAs take every rank's block scores from this rank's exchange buffer
  // (polling their step tags; the score is the max over ranks), the merges
  // push this rank's output rows to every other rank, and each head's merging
  // CTA pulls the other ranks' rows of the same local head index into the
  // full-width output; the last merging CTA advances the epoch
  const u64* xp_scores;           // this rank's xs area
  u64* xp_out[NKV_MAX_PEERS];     // every rank's xo area
  uint32_t* xp_sync;              // this rank's [epoch, ticket]
  __nv_bfloat16* xp_full;         // this rank's full-width output [xp_hq][D]
  int xp_P, xp_rank, xp_cap, xp_hq;
};

// 2D tensor maps of the decode kernel over [rows][128] bf16 sources with
// 64-column boxes and 128-byte swizzle: m[source][K|V][box], source 0 = block
// store, 1 = sink, 2 = recent ring; box 0 = 8 rows, 1 = 64 rows.
struct DecodeMaps {
  CUtensorMap m[3][2][2];
  // whole 64-row tiles in one box: dims (64 columns, rows, 2 halves), the
  // halves 128 bytes apart, so one box lands as the [2][64][128 B] tile
  CUtensorMap t3[3][2];
};

__device__ __forceinline__ long long clamp_id(const AttendParams& p, int slot, bool* bad) {
  long long id = __ldg(p.ids + slot);
  if (id < 0 || id >= p.max_blocks) {
    *bad = true;
    if (p.err) atomicExch(p.err, ERR_BAD_INDEX);
    return 0;
  }
  *bad = false;
  return id;
}

// Walk the contiguous pieces of logical keys [t0, t1) of head h and issue one
// bulk copy per piece for K (which==0) or V (which==1).  Selected blocks are
// skipped when the store is int8 (those are loaded by the threads).
// With count_only, nothing is issued and the byte total is returned.
// part: 0 = every piece, 1 = pieces outside the selected segment, 2 = selected only.
__device__ uint32_t issue_bulk(const AttendParams& p, int h, int t0, int t1, __nv_bfloat16* dst,
                               int which, uint64_t* bar, bool count_only, int part = 0) {
  uint32_t total = 0;
  const int B = p.B;
  const int selEnd = p.n_sel * B, sinkEnd = selEnd + p.sink_len, ringEnd = sinkEnd + p.ring_len;
  int pos = t0;
  if (part == 1 && pos < selEnd) pos = min(selEnd, t1);
  while (pos < t1) {
    const __nv_bfloat16* src;
    int len;
    if (part == 2 && pos >= selEnd) break;
    if (pos < selEnd) {
      const int slot = pos / B, off = pos % B;
      len = min(B - off, t1 - pos);
      if (p.kind != NKV_STORE_BF16) { pos += len; continue; }
      bool bad;
      const long long id = clamp_id(p, slot, &bad);
      const __nv_bfloat16* base = reinterpret_cast<const __nv_bfloat16*>(which ? p.v_store : p.k_store);
      src = base + ((id * p.hkv + h) * B + off) * NKV_D;
    } else if (pos < sinkEnd) {
      const int off = pos - selEnd;
      len = min(sinkEnd - pos, t1 - pos);
      src = (which ? p.sink_v : p.sink_k) + ((long long)h * p.sink_cap + off) * NKV_D;
    } else if (pos < ringEnd) {
      const int i = pos - sinkEnd;
      int phys = p.ring_start + i;            // ring_start < cap, i < ring_len <= cap
      if (phys >= p.ring_cap) phys -= p.ring_cap;
      const int room = p.ring_cap - phys;     // slots before the physical end
      len = ringEnd - pos;
      if (t1 - pos < len) len = t1 - pos;
      if (room < len) len = room;
      if (len < 1 || phys < 0 || phys + len > p.ring_cap) {  // never taken for valid arguments
        if (p.err) atomicExch(p.err, ERR_BOUNDS);
        len = 1;
        phys = 0;
      }
      src = (which ? p.ring_v : p.ring_k) + ((long long)h * p.ring_cap + phys) * NKV_D;
    } else {
      const int j = pos - ringEnd;
      len = 1;
      src = (which ? p.cur_v : p.cur_k) + j * p.cur_row + h * p.cur_head;
    }
#ifdef NKV_CHECKED
    {
      long long ext, base_off;
      if (pos < selEnd) {
        ext = p.ext_store;
        base_off = src - reinterpret_cast<const __nv_bfloat16*>(which ? p.v_store : p.k_store);
      } else if (pos < sinkEnd) {
        ext = p.ext_sink;
        base_off = src - (which ? p.sink_v : p.sink_k);
      } else if (pos < ringEnd) {
        ext = p.ext_ring;
        base_off = src - (which ? p.ring_v : p.ring_k);
      } else {
        ext = p.ext_cur;
        base_off = src - (which ? p.cur_v : p.cur_k);
      }
      const int site = (pos < selEnd ? 10 : pos < sinkEnd ? 11 : pos < ringEnd ? 12 : 13) + 10 * which;
      if (!NKV_INB(p.err, site, base_off, (long long)len * NKV_D, ext) ||
          !NKV_INB(p.err, 30, (long long)(pos - t0) * NKV_D, (long long)len * NKV_D, (long long)p.tps * NKV_D)) {
        pos += len;  // skipped: not counted, not issued
        continue;
      }
    }
#endif
#ifdef NKV_CHECKED
    if (p.trace && count_only && which == 0) {
      int* tr = p.trace + (blockIdx.y * gridDim.x + blockIdx.x) * 64;
      const int k = tr[15];
      if (k < 12) {
        tr[16 + 4 * k] = pos;
        tr[17 + 4 * k] = len;
        tr[18 + 4 * k] = (int)((src - (pos < selEnd ? reinterpret_cast<const __nv_bfloat16*>(p.k_store)
                                   : pos < sinkEnd ? p.sink_k : pos < ringEnd ? p.ring_k : p.cur_k)) / NKV_D);
        tr[19 + 4 * k] = pos < selEnd ? 0 : pos < sinkEnd ? 1 : pos < ringEnd ? 2 : 3;
        tr[15] = k + 1;
      }
    }
#endif
    total += (uint32_t)len * NKV_D * 2;
    if (!count_only) bulk_g2s(dst + (long long)(pos - t0) * NKV_D, src, (uint32_t)len * NKV_D * 2, bar);
    pos += len;
  }
  return total;
}

// int8 selected keys of [t0, t1): 128-bit loads (16 values), dequant to bf16.
__device__ void load_int8(const AttendParams& p, int h, int t0, int t1, __nv_bfloat16* ks,
                          __nv_bfloat16* vs) {
  const int B = p.B;
  const int selEnd = min(p.n_sel * B, t1);
  if (t0 >= selEnd) return;
  const int nt = selEnd - t0;
  const signed char* kst = reinterpret_cast<const signed char*>(p.k_store);
  const signed char* vst = reinterpret_cast<const signed char*>(p.v_store);
  constexpr int U = 4;
  for (int base = threadIdx.x; base < nt * 8; base += AT_THREADS * U) {
    uint4 kr[U], vr[U];
    long long ids[U];
    int rows[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = base + u * AT_THREADS;
      rows[u] = -1;
      if (i < nt * 8) {
        const int t = i >> 3, c = i & 7;
        const int pos = t0 + t, slot = pos / B, off = pos % B;
        bool bad;
        const long long id = clamp_id(p, slot, &bad);
        ids[u] = id;
        rows[u] = t * 8 + c;
        const long long o = ((id * p.hkv + h) * B + off) * NKV_D + c * 16;
        kr[u] = ldg_nc_v4(kst + o);
        vr[u] = ldg_nc_v4(vst + o);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (rows[u] < 0) continue;
      const int t = rows[u] >> 3, c = rows[u] & 7;
      const int pos = t0 + t, off = pos % B;
      const signed char* kb = reinterpret_cast<const signed char*>(&kr[u]);
      const signed char* vb = reinterpret_cast<const signed char*>(&vr[u]);
      uint32_t kw[8], vw[8];
      if (p.kind == NKV_STORE_INT8_REF) {
        const float vsc = __ldg(p.vbs + ids[u] * p.hkv + h);
#pragma unroll
        for (int e = 0; e < 16; e += 2) {
          const int d = c * 16 + e;
          const float k0 = (float)kb[e] * __ldg(p.kcs + h * NKV_D + d);
          const float k1 = (float)kb[e + 1] * __ldg(p.kcs + h * NKV_D + d + 1);
          kw[e / 2] = (uint32_t)f2bf(k0) | ((uint32_t)f2bf(k1) << 16);
          vw[e / 2] = (uint32_t)f2bf((float)vb[e] * vsc) | ((uint32_t)f2bf((float)vb[e + 1] * vsc) << 16);
        }
      } else {
        const long long so = (ids[u] * p.hkv + h) * B + off;
        const float ksc = __bfloat162float(p.kts[so]);
        const float vsc = __bfloat162float(p.vts[so]);
#pragma unroll
        for (int e = 0; e < 16; e += 2) {
          kw[e / 2] = (uint32_t)f2bf((float)kb[e] * ksc) | ((uint32_t)f2bf((float)kb[e + 1] * ksc) << 16);
          vw[e / 2] = (uint32_t)f2bf((float)vb[e] * vsc) | ((uint32_t)f2bf((float)vb[e + 1] * vsc) << 16);
        }
      }
      uint4* kd = reinterpret_cast<uint4*>(ks + (long long)t * NKV_D + c * 16);
      uint4* vd = reinterpret_cast<uint4*>(vs + (long long)t * NKV_D + c * 16);
      kd[0] = make_uint4(kw[0], kw[1], kw[2], kw[3]);
      kd[1] = make_uint4(kw[4], kw[5], kw[6], kw[7]);
      vd[0] = make_uint4(vw[0], vw[1], vw[2], vw[3]);
      vd[1] = make_uint4(vw[4], vw[5], vw[6], vw[7]);
    }
  }
}

// Sum of G per-head partials over the 8 lanes of a token group, transposed:
// each step keeps half of the remaining heads and ships the other half to the
// partner lane, so G=4 costs 4 shuffles instead of 12.  Lane c (= lane & 7)
// ends with the total of head head_of<G>(c); lanes with c < G hold distinct heads.
template <int G>
__device__ __forceinline__ int head_of(int c) {
  int g = 0;
#pragma unroll
  for (int s = 0, w = G >> 1; w > 0; ++s, w >>= 1) g += ((c >> s) & 1) * w;
  return g;
}
template <int G>
__device__ __forceinline__ float reduce8_transposed(float (&v)[G], int c) {
  float cur[G];
#pragma unroll
  for (int i = 0; i < G; ++i) cur[i] = v[i];
  int len = G;
#pragma unroll
  for (int s = 0; s < 3; ++s) {
    const int m = 1 << s;
    if (len > 1) {
      const int half = len >> 1;
      const bool upper = (c >> s) & 1;
#pragma unroll
      for (int i = 0; i < G / 2; ++i) {
        if (i < half) {
          const float keep = upper ? cur[half + i] : cur[i];
          const float give = upper ? cur[i] : cur[half + i];
          cur[i] = keep + __shfl_xor_sync(FULL, give, m);
        }
      }
      len = half;
    } else {
      cur[0] += __shfl_xor_sync(FULL, cur[0], m);
    }
  }
  return cur[0];
}

// Logical key T visible to query row n?  ids_s: this CTA's block ids (-1 = bad).
__device__ __forceinline__ bool visible(const AttendParams& p, int T, int n, int selEnd, int ringEnd,
                                        const long long* ids_s, int slot0) {
  if (T < selEnd) {
    const int slot = T >> p.log2B;
    if (ids_s[slot - slot0] < 0) return false;
    if (p.allowed && !p.allowed[(long long)n * p.allowed_stride + slot]) return false;
    return true;
  }
  if (T >= ringEnd) return (T - ringEnd) <= n + (p.n_cur - p.nq);
  return true;
}

// acc[a][e] = sum over keys t = slice, slice+step, ... of p[t][rg*4+a] * V[t][lane*4+e]
__device__ __forceinline__ void pv_accumulate(const float* sc, const __nv_bfloat16* vs, int nrp, int rg,
                                              int slice, int step, int n, int lane, float (&acc)[4][4]) {
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b) acc[a][b] = 0.f;
#pragma unroll 4
  for (int t = slice; t < n; t += step) {
    const float4 pr = *reinterpret_cast<const float4*>(sc + t * nrp + rg * 4);
    const uint2 vw = *reinterpret_cast<const uint2*>(vs + (long long)t * NKV_D + lane * 4);
    const float v0 = bf_lo(vw.x), v1 = bf_hi(vw.x), v2 = bf_lo(vw.y), v3 = bf_hi(vw.y);
    const float pp[4] = {pr.x, pr.y, pr.z, pr.w};
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      acc[a][0] = fmaf(pp[a], v0, acc[a][0]);
      acc[a][1] = fmaf(pp[a], v1, acc[a][1]);
      acc[a][2] = fmaf(pp[a], v2, acc[a][2]);
      acc[a][3] = fmaf(pp[a], v3, acc[a][3]);
    }
  }
}

template <int G>
__device__ void combine_splits(const AttendParams& p, int h, float* wbuf, uint32_t xp_ep = 0u);
template <int G>
__device__ void combine_cluster(const AttendParams& p, int h, float* pm, float* pl, float* po, uint32_t xp_ep = 0u);

template <int G, bool Q1>
__global__ void __launch_bounds__(AT_THREADS) attend_kernel(AttendParams p) {
  extern __shared__ __align__(128) unsigned char sm[];
  __shared__ __align__(8) uint64_t bar[2];
  __shared__ unsigned s_ticket;
  __shared__ float s_m[64], s_l[64];
  __shared__ long long s_ids[AT_MAX_SLOTS];

  const int split = blockIdx.x, h = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int t0 = split * p.tps, t1 = min(p.ntok, t0 + p.tps), n = t1 - t0;
  const int nr = p.nr, nrp = p.nr_pad;
  const int B = p.B;
  const int selEnd = p.n_sel * B, sinkEnd = selEnd + p.sink_len, ringEnd = sinkEnd + p.ring_len;
  const int slot0 = t0 / B;
  const int nslots = t0 < selEnd ? (min(t1, selEnd) - 1) / B - slot0 + 1 : 0;

  __nv_bfloat16* ks = reinterpret_cast<__nv_bfloat16*>(sm);
  __nv_bfloat16* vs = ks + (long long)p.tps * NKV_D;
  float* sc = reinterpret_cast<float*>(vs + (long long)p.tps * NKV_D);  // [tps][nrp]
  float* red = sc + (long long)p.tps * nrp;                              // [8][4][D]
  float* qs = red + AT_WARPS * 4 * NKV_D;                                // [nr][D] (Q1 == false)
  float* pm = qs + (Q1 ? 0 : nr * NKV_D);                                // [nr]   (cluster merge)
  float* pl = pm + 64;                                                   // [nr]
  float* po = pl + 64;                                                   // [nr][D]

#ifdef NKV_CHECKED
  int* trc = p.trace ? p.trace + (blockIdx.y * gridDim.x + blockIdx.x) * 64 : nullptr;
#else
  int* trc = nullptr;
#endif
  NKV_STAMP(trc, 48);

  // ---- 1. data movement ---------------------------------------------------------
  const int n_int8 = (p.kind != NKV_STORE_BF16) ? max(0, min(selEnd, t1) - t0) : 0;
  if (tid == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    fence_mbar_init();
#ifdef NKV_CHECKED
    if (p.overlap) pdl_wait();  // the checked count pass reads ids
    if (p.trace) {
      trc[0] = t0; trc[1] = t1; trc[2] = p.ring_cap; trc[3] = p.ring_start; trc[4] = p.ring_len;
      trc[5] = p.sink_len; trc[6] = p.n_sel; trc[7] = p.B; trc[8] = p.tps; trc[9] = p.ntok;
      unsigned smid;
      asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
      trc[10] = h; trc[11] = p.sink_cap; trc[12] = p.splits; trc[13] = p.n_cur; trc[14] = (int)smid;
      trc[15] = 0;
    }
    mbar_expect_tx(&bar[0], issue_bulk(p, h, t0, t1, ks, 0, &bar[0], true));
    mbar_expect_tx(&bar[1], issue_bulk(p, h, t0, t1, vs, 1, &bar[1], true));
#else
    const uint32_t bytes = (uint32_t)(n - n_int8) * NKV_D * 2;
    mbar_expect_tx(&bar[0], bytes);
    mbar_expect_tx(&bar[1], bytes);
#endif
    // pieces that do not depend on the selection first
    issue_bulk(p, h, t0, t1, ks, 0, &bar[0], false, 1);
    issue_bulk(p, h, t0, t1, vs, 1, &bar[1], false, 1);
  }
  // decode: append the current token to the recent ring (a slot no CTA reads)
  if (split == 0 && p.ring_write_pos >= 0 && tid >= 32 && tid < 64 &&
      NKV_INB(p.err, 40, ((long long)h * p.ring_cap + p.ring_write_pos) * NKV_D, NKV_D, p.ext_ring) &&
      NKV_INB(p.err, 41, h * p.cur_head, NKV_D, p.ext_cur)) {
    const int c = tid & 15;
    const bool isv = (tid & 16) != 0;
    const __nv_bfloat16* src = (isv ? p.cur_v : p.cur_k) + h * p.cur_head + c * 8;
    __nv_bfloat16* dst = (isv ? p.ring_v : p.ring_k) + ((long long)h * p.ring_cap + p.ring_write_pos) * NKV_D + c * 8;
    *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
  }
  // queries for this head's G heads
  float qr[Q1 ? G : 1][16];
  const int c = lane & 7, t4 = lane >> 3;
  if (Q1) {
#pragma unroll
    for (int g = 0; g < (Q1 ? G : 1); ++g) {
      const __nv_bfloat16* qsrc = p.q + (long long)(h * G + g) * p.q_head;
      unpack8(__ldg(reinterpret_cast<const uint4*>(qsrc + c * 8)), qr[g]);
      unpack8(__ldg(reinterpret_cast<const uint4*>(qsrc + 64 + c * 8)), qr[g] + 8);
    }
  } else {
    for (int i = tid; i < nr * (NKV_D / 8); i += blockDim.x) {
      const int row = i / (NKV_D / 8), cc = i % (NKV_D / 8);
      const int qn = row / G, g = row % G;
      float f[8];
      unpack8(__ldg(reinterpret_cast<const uint4*>(p.q + qn * p.q_row + (long long)(h * G + g) * p.q_head + cc * 8)), f);
#pragma unroll
      for (int e = 0; e < 8; ++e) qs[row * NKV_D + cc * 8 + e] = f[e];
    }
  }
  NKV_STAMP(trc, 49);
  if (p.overlap) pdl_wait();  // block ids are complete past this point
  // selected blocks: lane i of warp 0 owns block slot slot0 + i
  if (warp == 0) {
    __syncwarp();
    if (lane < nslots) {
      const int slot = slot0 + lane;
      bool bad;
      const long long id = clamp_id(p, slot, &bad);
      s_ids[lane] = bad ? -1 : id;
      if (p.kind == NKV_STORE_BF16) {
        const int a0 = max(t0, slot * B), a1 = min(min(t1, selEnd), slot * B + B);
        const int off = a0 - slot * B, len = a1 - a0;
        const long long src = ((id * p.hkv + h) * B + off) * NKV_D;
        if (NKV_INB(p.err, 15, src, (long long)len * NKV_D, p.ext_store)) {
          bulk_g2s(ks + (long long)(a0 - t0) * NKV_D, reinterpret_cast<const __nv_bfloat16*>(p.k_store) + src,
                   (uint32_t)len * NKV_D * 2, &bar[0]);
          bulk_g2s(vs + (long long)(a0 - t0) * NKV_D, reinterpret_cast<const __nv_bfloat16*>(p.v_store) + src,
                   (uint32_t)len * NKV_D * 2, &bar[1]);
        }
      }
    }
  }
  if (n_int8 > 0) load_int8(p, h, t0, t1, ks, vs);
  __syncthreads();  // barrier init, ids, int8 tiles and qs visible
  NKV_STAMP(trc, 50);
  mbar_wait_bounded(&bar[0], 0, p.err);
  NKV_STAMP(trc, 51);

  // ---- 2. scores: lanes (t4, c) = (token of a group of 4, 16-dim slice); two groups
  //         per iteration for ILP; every lane keeps the running max of its row ----------
  float mloc = -INFINITY;
  if (Q1) {
    const int gh = head_of<G>(c);
    for (int tg = warp; tg * 4 < n; tg += 2 * AT_WARPS) {
      float kf[2][16];
      int tt[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        tt[u] = (tg + u * AT_WARPS) * 4 + t4;
        if (tt[u] < n) {
          unpack8(*reinterpret_cast<const uint4*>(ks + (long long)tt[u] * NKV_D + c * 8), kf[u]);
          unpack8(*reinterpret_cast<const uint4*>(ks + (long long)tt[u] * NKV_D + 64 + c * 8), kf[u] + 8);
        } else {
#pragma unroll
          for (int e = 0; e < 16; ++e) kf[u][e] = 0.f;
        }
      }
      float part[2][Q1 ? G : 1];
#pragma unroll
      for (int u = 0; u < 2; ++u)
#pragma unroll
        for (int g = 0; g < (Q1 ? G : 1); ++g) {
          float s0 = 0.f, s1 = 0.f;
#pragma unroll
          for (int e = 0; e < 16; e += 2) {
            s0 = fmaf(qr[g][e], kf[u][e], s0);
            s1 = fmaf(qr[g][e + 1], kf[u][e + 1], s1);
          }
          part[u][g] = s0 + s1;
        }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const float tot = reduce8_transposed<Q1 ? G : 1>(part[u], c);
        if (tt[u] < n && c < G) {
          const bool vis = visible(p, t0 + tt[u], 0, selEnd, ringEnd, s_ids, slot0);
          const float sv = vis ? tot * p.scale : -INFINITY;
          sc[tt[u] * nrp + gh] = sv;
          mloc = fmaxf(mloc, sv);
        }
      }
    }
    // row max: combine lanes holding the same head (other c bits, t4), then warps
#pragma unroll
    for (int m = G; m < 32; m <<= 1) mloc = fmaxf(mloc, __shfl_xor_sync(FULL, mloc, m));
    if (lane < G) red[warp * 64 + gh] = mloc;
  } else {
    for (int tg = warp; tg * 4 < n; tg += AT_WARPS) {
      const int t = tg * 4 + t4;
      const bool valid = t < n;
      float kf[16];
      if (valid) {
        unpack8(*reinterpret_cast<const uint4*>(ks + (long long)t * NKV_D + c * 8), kf);
        unpack8(*reinterpret_cast<const uint4*>(ks + (long long)t * NKV_D + 64 + c * 8), kf + 8);
      } else {
#pragma unroll
        for (int e = 0; e < 16; ++e) kf[e] = 0.f;
      }
      for (int qn = 0; qn < p.nq; ++qn) {
        float part[G];
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float* qrow = qs + (qn * G + g) * NKV_D;
          float s0 = 0.f, s1 = 0.f;
#pragma unroll
          for (int e = 0; e < 8; ++e) s0 = fmaf(qrow[c * 8 + e], kf[e], s0);
#pragma unroll
          for (int e = 0; e < 8; ++e) s1 = fmaf(qrow[64 + c * 8 + e], kf[8 + e], s1);
          part[g] = s0 + s1;
        }
        const float tot = reduce8_transposed<G>(part, c);
        if (valid && c < G) {
          const bool vis = visible(p, t0 + t, qn, selEnd, ringEnd, s_ids, slot0);
          sc[t * nrp + qn * G + head_of<G>(c)] = vis ? tot * p.scale : -INFINITY;
        }
      }
    }
  }
  if (tid < 64) s_l[tid] = 0.f;
  __syncthreads();
  NKV_STAMP(trc, 52);

  // ---- 3. split softmax: row max, exponentials and row sums over all threads ----------
  if (Q1) {
    if (tid < nr) {
      float m = -INFINITY;
      for (int w = 0; w < AT_WARPS; ++w) m = fmaxf(m, red[w * 64 + tid]);
      s_m[tid] = m;
    }
  } else {
    for (int row = warp; row < nr; row += AT_WARPS) {
      float m = -INFINITY;
      for (int t = lane; t < n; t += 32) m = fmaxf(m, sc[t * nrp + row]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(FULL, m, o));
      if (lane == 0) s_m[row] = m;
    }
  }
  __syncthreads();
  {
    // consecutive threads walk consecutive (token, row) entries; each thread's
    // entries share one row when nrp divides the thread count
    float lsum = 0.f;
    int lrow = -1;
    for (int i = tid; i < n * nrp; i += blockDim.x) {
      const int row = i % nrp;
      float e = 0.f;
      if (row < nr) {
        const float m = s_m[row];
        e = (m == -INFINITY) ? 0.f : __expf(sc[i] - m);
      }
      sc[i] = e;
      if (row != lrow) {
        if (lrow >= 0 && lrow < nr) atomicAdd(&s_l[lrow], lsum);
        lsum = 0.f;
        lrow = row;
      }
      lsum += e;
    }
    if (lrow >= 0 && lrow < nr) atomicAdd(&s_l[lrow], lsum);
  }
  __syncthreads();
  NKV_STAMP(trc, 53);
  mbar_wait_bounded(&bar[1], 0, p.err);
  NKV_STAMP(trc, 54);

  // ---- 4. P.V: lane owns 4 dims; a warp owns a group of 4 rows over a token slice --
  const int nrg = nrp / 4;
  float* dst_o = p.cluster ? po : p.part_o + (((long long)h * p.splits + split) * nr) * NKV_D;
  if (!p.cluster &&
      !NKV_INB(p.err, 44, (((long long)h * p.splits + split) * nr) * NKV_D, (long long)nr * NKV_D, p.ext_part_o))
    return;
  if (nrg >= AT_WARPS) {
    for (int rg = warp; rg < nrg; rg += AT_WARPS) {
      float acc[4][4];
      pv_accumulate(sc, vs, nrp, rg, 0, 1, n, lane, acc);
#pragma unroll
      for (int a = 0; a < 4; ++a)
        if (rg * 4 + a < nr)
          *reinterpret_cast<float4*>(dst_o + (rg * 4 + a) * NKV_D + lane * 4) =
              make_float4(acc[a][0], acc[a][1], acc[a][2], acc[a][3]);
    }
  } else {
    const int ts = AT_WARPS / nrg;  // token slices per row group
    if (warp < nrg * ts) {
      float acc[4][4];
      pv_accumulate(sc, vs, nrp, warp / ts, warp % ts, ts, n, lane, acc);
#pragma unroll
      for (int a = 0; a < 4; ++a)
        *reinterpret_cast<float4*>(red + (warp * 4 + a) * NKV_D + lane * 4) =
            make_float4(acc[a][0], acc[a][1], acc[a][2], acc[a][3]);
    }
    __syncthreads();
    for (int i = tid; i < nr * NKV_D; i += blockDim.x) {
      const int row = i / NKV_D, d = i % NKV_D;
      const int rg = row / 4, a = row % 4;
      float s = 0.f;
      for (int sl = 0; sl < ts; ++sl) s += red[((rg * ts + sl) * 4 + a) * NKV_D + d];
      dst_o[row * NKV_D + d] = s;
    }
  }
  if (p.cluster) {
    if (tid < nr) {
      pm[tid] = s_m[tid];
      pl[tid] = s_l[tid];
    }
    NKV_STAMP(trc, 55);
    combine_cluster<G>(p, h, pm, pl, po);
    NKV_STAMP(trc, 57);
    return;
  }
  if (tid < nr && NKV_INB(p.err, 42, (((long long)h * p.splits + split) * nr + tid) * 2, 2, p.ext_part_ml)) {
    float* ml = p.part_ml + (((long long)h * p.splits + split) * nr + tid) * 2;
    ml[0] = s_m[tid];
    ml[1] = s_l[tid];
  }

  // ---- 5. last CTA of the head merges the splits -----------------------------------
  NKV_STAMP(trc, 55);
  __threadfence();
  __syncthreads();
  if (tid == 0) s_ticket = atomicAdd(p.counters + h, 1u);
  __syncthreads();
  NKV_STAMP(trc, 56);
  if (s_ticket != (unsigned)p.splits - 1) return;
  __threadfence();
  if (tid == 0) p.counters[h] = 0u;
  combine_splits<G>(p, h, reinterpret_cast<float*>(ks));
  __syncthreads();
  NKV_STAMP(trc, 57);
}


// ---------------------------------------------------------------------------
// Peer exchange of the outputs (KV-head sharding).
// ---------------------------------------------------------------------------
// One tagged word (two bf16 of the full output, word index wi of the xo area)
// to every other rank.
__device__ __forceinline__ void peer_push(const AttendParams& p, uint32_t ep, long long wi, uint32_t payload) {
  const u64 w = ((u64)step_tag(ep) << 32) | payload;
  const long long at = (long long)(ep & 1u) * p.xp_hq * (NKV_D / 2) + wi;
  for (int r = 0; r < p.xp_P; ++r)
    if (r != p.xp_rank) st_peer_u64(p.xp_out[r] + at, w);
}
// Run by the merging CTA of local head h after its own rows are written and
// pushed: pulls the rows of local head h of every other rank (global head
// r * heads + h) from this rank's xo area into the full output (four words in
// flight per thread, each polled until it carries this step's tag; bounded),
// then arrives on the epoch ticket; the last of the grid's heads to arrive
// advances the epoch (every CTA of the grid has read it by then).
template <int G>
__device__ void peer_pull_arrive(const AttendParams& p, int h, uint32_t ep) {
  const int tid = threadIdx.x, bs = (int)blockDim.x, Hl = (int)gridDim.y;
  const uint32_t tag = step_tag(ep);
  constexpr int WPH = G * (NKV_D / 2);  // words per head
  const u64* xo = p.xp_out[p.xp_rank] + (long long)(ep & 1u) * p.xp_hq * (NKV_D / 2);
  const int n = (p.xp_P - 1) * WPH;
  bool late = false;
  for (int base = tid; base < n; base += 4 * bs) {
    long long wi[4];
    u64 w[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = base + u * bs;
      wi[u] = -1;
      if (i < n) {
        const int rr = i / WPH;
        const int r = rr < p.xp_rank ? rr : rr + 1;
        wi[u] = (long long)(r * Hl + h) * WPH + i % WPH;
        w[u] = ld_peer_u64(xo + wi[u]);
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (wi[u] < 0) continue;
      if ((uint32_t)(w[u] >> 32) != tag) {
        const long long t0 = clock64();
        while ((uint32_t)((w[u] = ld_peer_u64(xo + wi[u])) >> 32) != tag)
          if (clock64() - t0 > PEER_WAIT_CYCLES) {
            late = true;
            break;
          }
      }
      *reinterpret_cast<uint32_t*>(p.xp_full + wi[u] * 2) = (uint32_t)w[u];
    }
  }
  if (late && p.err) atomicExch(p.err, ERR_WAIT_TIMEOUT);
  __syncthreads();
  if (tid == 0 && atomicAdd(p.xp_sync + 1, 1u) == (unsigned)Hl - 1u) {
    p.xp_sync[1] = 0u;
    atomicAdd(p.xp_sync, 1u);
  }
}

// ---------------------------------------------------------------------------
// Decode tiles.  The K and V keys of a CTA sit in shared memory as
// [2][rows][128 B] (the two 64-column halves of a key row) in the 128-byte
// swizzle that TMA writes: 16-byte chunk c of row r is stored at chunk
// c ^ (r & 7).  The tile base is 1024-byte aligned and every piece starts at a
// multiple of 8 rows, so rows loaded by TMA and rows loaded by threads share one
// pattern, and the 8 rows of one ldmatrix matrix fall in 8 different bank groups.
// ---------------------------------------------------------------------------
constexpr int DT_PAD_ROWS = 32;  // tile rows beyond tps: padding of <= 4 pieces of ragged length
enum : int { PT_SEL = 0, PT_SINK = 1, PT_RING = 2, PT_THREADS = 3, PT_SKIP = 4, PT_EMPTY = 5 };

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
// One 64-row tile (both 64-column halves) of a [rows][128] bf16 tensor in one
// box of a DecodeMaps::t3 map.
__device__ __forceinline__ void tma_tile3(void* dst, const CUtensorMap* map, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(0), "r"(y), "r"(0), "r"(smem_u32(bar))
      : "memory");
}
// One box (8 or 64 rows x 64 columns) of a [rows][128] bf16 tensor into swizzled shared memory.
__device__ __forceinline__ void tma_box(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// TMA boxes of one piece: `len` rows of source `src` from row y0, into tile
// rows row0...: 64-row boxes while 64 rows remain, then 8-row boxes; the
// (box, half, K|V) jobs are spread over the lanes of the calling warp.
__device__ __forceinline__ void issue_piece(const DecodeMaps& tm, int src, int y0, int len, int row0,
                                            unsigned char* kt, unsigned char* vt, int NR, uint64_t* kb,
                                            uint64_t* vb, int lane) {
  const int nbig = len >> 6, nsmall = ((len & 63) + 7) >> 3;
  const int jobs = (nbig + nsmall) * 4;
  for (int j = lane; j < jobs; j += 32) {
    const int b = j >> 2, half = (j >> 1) & 1, isv = j & 1;
    const bool big = b < nbig;
    const int r = big ? b * 64 : nbig * 64 + (b - nbig) * 8;
    unsigned char* dst = (isv ? vt : kt) + ((size_t)half * NR + row0 + r) * 128;
    tma_box(dst, &tm.m[src][isv][big ? 1 : 0], half * 64, y0 + r, isv ? vb : kb);
  }
}


// ---------------------------------------------------------------------------
// One-launch decode step: scoring and selection inside the attention grid.
// ---------------------------------------------------------------------------
constexpr int FS_BPC_MAX = 64;  // blocks one CTA scores (for every KV head)
constexpr int FS_MAXE = 8;      // keys per thread in the selection (nblocks <= 8 x threads)

__device__ __forceinline__ void st_relaxed_u64(unsigned long long* a, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(a), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long* a) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(a) : "memory");
  return v;
}
__device__ __forceinline__ int ld_relaxed_s32(const int* a) {
  int v;
  asm volatile("ld.relaxed.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(a) : "memory");
  return v;
}
__device__ __forceinline__ unsigned ld_relaxed_u32(const unsigned* a) {
  unsigned v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(a) : "memory");
  return v;
}
// Bulk prefetch of `bytes` (a multiple of 16, 16-byte aligned) into L2, no completion tracking.
__device__ __forceinline__ void prefetch_l2_bulk(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
// Tag of a launch's keys: never 0, so a zeroed key array holds no valid key.
__device__ __forceinline__ uint32_t fs_tag(uint32_t epoch) { return epoch % 0xfffffffeu + 1u; }

// Scores of this CTA's blocks on the tensor cores: warp w scores KV heads
// w, w + NW, ...; for one head the CTA's representative rows (nb blocks x r,
// contiguous in [hkv][reps_blocks][r][D]) are the N columns and the head's G
// query rows the M rows (rows >= G zero) of mma.sync m16n8k16, K = D.  The K
// order inside the MMA is a permutation of the head dims, the same for both
// operands: at k-steps 2i and 2i + 1 lane quad t holds dims 32i + 8t ... + 7
// (one 16-byte load per operand row), so the products are the full dot
// products.  Per representative row the max over query rows (xor 4, 8, 16),
// then over the r rows of a block (r in {1, 2, 4}: the rows of a block sit in
// adjacent lanes), kept per (warp, block) in shared memory (orderable bits,
// no atomics); the block score is the max over the warps' entries, and
// protected blocks publish -inf.  Scores are fp32 sums of exact bf16
// products, in the tensor core's summation order.
// s_prot (optional): shared flags of the CTA's blocks that are protected
// (block b0 + i at index i), in place of a scan of the protected list per block.
template <int G, int NW>
__device__ void fs_score_publish(const AttendParams& p, int cta, uint32_t tag, unsigned (*s_part)[FS_BPC_MAX],
                                 [[maybe_unused]] int* trc, const unsigned char* s_prot = nullptr) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int b0 = cta * p.fs_bpc, nb = min(p.fs_bpc, p.rank_n - b0);
  if (nb <= 0) return;  // CTA-uniform
  const int g = lane >> 2, t = lane & 3;
  const int rows = nb * p.fs_r;
  for (int hh = warp; hh < p.hkv; hh += NW) {
    uint4 qf[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      qf[i] = g < G ? __ldg(reinterpret_cast<const uint4*>(p.q + (long long)(hh * G + g) * p.q_head + i * 32 + t * 8))
                    : make_uint4(0u, 0u, 0u, 0u);
    const __nv_bfloat16* rbase = p.fs_reps + ((long long)hh * p.fs_reps_blocks + b0) * p.fs_r * NKV_D;
    for (int row0 = 0; row0 < rows; row0 += 32) {
      uint4 rf[4][4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int rr = row0 + j * 8 + g;
#pragma unroll
        for (int i = 0; i < 4; ++i)
          rf[j][i] = rr < rows ? __ldg(reinterpret_cast<const uint4*>(rbase + (long long)rr * NKV_D + i * 32 + t * 8))
                               : make_uint4(0u, 0u, 0u, 0u);
      }
      float c[4][4];
#pragma unroll
      for (int j = 0; j < 4; ++j) c[j][0] = c[j][1] = c[j][2] = c[j][3] = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
#pragma unroll
        for (int j = 0; j < 4; ++j) mma_bf16(c[j], qf[i].x, 0u, qf[i].y, 0u, rf[j][i].x, rf[j][i].y);
#pragma unroll
        for (int j = 0; j < 4; ++j) mma_bf16(c[j], qf[i].z, 0u, qf[i].w, 0u, rf[j][i].z, rf[j][i].w);
      }
      if (row0 == 0) NKV_STAMP(trc, 45);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        // c[j][0..1]: query row g x representative rows row0 + 8j + 2t, + 1
        float v0 = g < G ? c[j][0] : -INFINITY, v1 = g < G ? c[j][1] : -INFINITY;
#pragma unroll
        for (int x = 4; x < 32; x <<= 1) {
          v0 = fmaxf(v0, __shfl_xor_sync(FULL, v0, x));
          v1 = fmaxf(v1, __shfl_xor_sync(FULL, v1, x));
        }
        const int rr = row0 + j * 8 + 2 * t;
        if (p.fs_r == 1) {
          if (g == 0 && rr < rows) s_part[warp][rr] = max(s_part[warp][rr], f32_order(v0));
          if (g == 0 && rr + 1 < rows) s_part[warp][rr + 1] = max(s_part[warp][rr + 1], f32_order(v1));
        } else {
          float m = fmaxf(v0, v1);  // rows rr, rr + 1: one block
          if (p.fs_r == 4) m = fmaxf(m, __shfl_xor_sync(FULL, m, 1));
          if (g == 0 && rr < rows && (rr % p.fs_r) == 0) {
            const int bl = rr / p.fs_r;
            s_part[warp][bl] = max(s_part[warp][bl], f32_order(m));
          }
        }
      }
    }
  }
  NKV_STAMP(trc, 44);
  __syncthreads();
  if (tid < nb) {
    const int b = b0 + tid;
    uint32_t u = 0u;
#pragma unroll
    for (int w = 0; w < NW; ++w) u = max(u, s_part[w][tid]);
    if (s_prot) {
      if (s_prot[tid]) u = f32_order(-INFINITY);
    } else {
      for (int i = 0; i < p.fs_nprot; ++i)
        if (__ldg(p.fs_prot + i) == b) u = f32_order(-INFINITY);
    }
    st_relaxed_u64(p.fs_keys + b, ((unsigned long long)tag << 32) | u);
  }
}

constexpr int FS_CAND_MAX = 256;  // candidates ranked by counting (more: extraction rounds)

// Top k (<= 32) of n orderable 32-bit scores (f32_order) held in registers,
// in rank order (score descending, then block id ascending: nkv_select's
// order), into s_sel[0, k) as make_key keys.  Thread t holds the scores of
// blocks t, t + NT, ... in u[0], u[1], ... (bit e of `live`: u[e] is a block).
//  1. threshold: every warp finds its 4th largest distinct score (4 warp max
//     reductions); theta = the smallest over the warps, so at least 4 x NW
//     keys score >= theta and the top k (<= 32) are among them (theta = 0,
//     every key, when fewer than k keys can be guaranteed that way);
//  2. the keys >= theta are compacted into shared memory (warp ballots);
//  3. each candidate's rank = the number of larger candidate keys; ranks below
//     k land in s_sel[rank].
// With more than FS_CAND_MAX candidates (flat or tied scores) the top k are
// extracted one per round (block-wide max of the remaining keys) instead.
// All threads of the CTA must call; s_sel is valid after the call.
template <int NW>
__device__ void topk_threshold(const uint32_t (&u)[FS_MAXE], unsigned live, int n, int k, u64* s_sel,
                               u64* s_cand, unsigned* s_misc, [[maybe_unused]] int* trc) {
  constexpr int NT = NW * 32;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int E = (n + NT - 1) / NT;
  // 1. per-warp 4th largest distinct score
  uint32_t prev = 0xffffffffu, th = 0u;
  bool more = true;
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    uint32_t m = 0u;
    bool any = false;
#pragma unroll
    for (int e = 0; e < FS_MAXE; ++e)
      if (((live >> e) & 1u) && (r == 0 || u[e] < prev)) {
        m = max(m, u[e]);
        any = true;
      }
    more = __any_sync(FULL, any) && more;
    m = __reduce_max_sync(FULL, m);
    prev = m;
    th = m;
  }
  const bool warp_live = __any_sync(FULL, live != 0u);
  if (lane == 0) s_misc[warp] = !warp_live ? 0xffffffffu : more ? th : 0u;
  __syncthreads();
  NKV_STAMP(trc, 36);
  uint32_t theta = 0xffffffffu;
  int nlive = 0;
#pragma unroll
  for (int w = 0; w < NW; ++w) {
    theta = min(theta, s_misc[w]);
    nlive += s_misc[w] != 0xffffffffu ? 1 : 0;
  }
  if (nlive * 4 < k) theta = 0u;
  // 2. candidates: per-warp counts, then each warp writes at its prefix
  unsigned cmask = 0u, wcount = 0u;
#pragma unroll
  for (int e = 0; e < FS_MAXE; ++e) {
    if (e >= E) break;  // CTA-uniform
    const bool cand = ((live >> e) & 1u) && u[e] >= theta;
    cmask |= cand ? 1u << e : 0u;
    wcount += (unsigned)__popc(__ballot_sync(FULL, cand));
  }
  if (lane == 0) s_misc[NW + warp] = wcount;
  __syncthreads();
  unsigned off = 0u, C = 0u;
#pragma unroll
  for (int w = 0; w < NW; ++w) {
    const unsigned c = s_misc[NW + w];
    off += w < warp ? c : 0u;
    C += c;
  }
#pragma unroll
  for (int e = 0; e < FS_MAXE; ++e) {
    if (e >= E) break;  // CTA-uniform
    const bool cand = (cmask >> e) & 1u;
    const unsigned bal = __ballot_sync(FULL, cand);
    const unsigned at = off + __popc(bal & ((1u << lane) - 1u));
    if (cand && at < FS_CAND_MAX) s_cand[at] = ((u64)u[e] << 32) | (u64)(0xffffffffu - (uint32_t)(tid + e * NT));
    off += __popc(bal);
  }
  __syncthreads();
  NKV_STAMP(trc, 37);
#ifdef NKV_CHECKED
  if (trc && tid == 0) trc[39] = (int)C;
#endif
  if (C <= FS_CAND_MAX) {
    // 3. rank by counting: 4 adjacent lanes per candidate, each over a quarter
    for (unsigned base = 0; base < C; base += NT / 4) {
      const unsigned c = base + (unsigned)(tid >> 2);
      const u64 key = c < C ? s_cand[c] : ~0ull;
      unsigned rank = 0u;
      for (unsigned d = (unsigned)(tid & 3); d < C; d += 4) rank += s_cand[d] > key ? 1u : 0u;
      rank += __shfl_xor_sync(FULL, rank, 1);
      rank += __shfl_xor_sync(FULL, rank, 2);
      if (c < C && (tid & 3) == 0 && rank < (unsigned)k) s_sel[rank] = key;
    }
  } else {
    // flat scores: k extraction rounds, each a block-wide max of the remaining keys
    u64 mine[FS_MAXE];
#pragma unroll
    for (int e = 0; e < FS_MAXE; ++e)
      mine[e] = ((live >> e) & 1u) ? ((u64)u[e] << 32) | (u64)(0xffffffffu - (uint32_t)(tid + e * NT)) : 0ull;
    u64* s_red = s_cand;  // NW partial maxima
    for (int r = 0; r < k; ++r) {
      u64 best = 0ull;
#pragma unroll
      for (int e = 0; e < FS_MAXE; ++e) best = umax64(best, mine[e]);
#pragma unroll
      for (int x = 1; x < 32; x <<= 1) best = umax64(best, shfl_xor64(best, x));
      __syncthreads();  // the previous round's reads of s_red are done
      if (lane == 0) s_red[warp] = best;
      __syncthreads();
      u64 top = 0ull;
#pragma unroll
      for (int w = 0; w < NW; ++w) top = umax64(top, s_red[w]);
      if (tid == 0) s_sel[r] = top;
#pragma unroll
      for (int e = 0; e < FS_MAXE; ++e)
        if (mine[e] == top) mine[e] = 0ull;
    }
  }
  NKV_STAMP(trc, 41);
  __syncthreads();
}

// Top n_sel of the rank_n published keys, in rank order, into s_sel
// (topk_threshold).  Thread t holds keys t, t + NT, ...: it polls them until
// they carry `tag` (bounded: ~0.2 s of SM clock, then ERR_WAIT_TIMEOUT).
// All threads of the CTA must call.
template <int NW>
__device__ void fs_select(const AttendParams& p, uint32_t tag, u64* s_sel, u64* s_cand, unsigned* s_misc,
                          [[maybe_unused]] int* trc) {
  constexpr int NT = NW * 32;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n = p.rank_n, k = p.n_sel;
  const int E = (n + NT - 1) / NT;
  uint32_t u[FS_MAXE];
  unsigned live = 0;
#pragma unroll
  for (int e = 0; e < FS_MAXE; ++e) {
    u[e] = 0u;
    if (e < E && tid + e * NT < n) live |= 1u << e;
  }
  unsigned pending = live;
  const long long t_start = clock64();
  while (pending) {
#pragma unroll
    for (int e = 0; e < FS_MAXE; ++e) {
      if ((pending >> e) & 1u) {
        const unsigned long long v = ld_relaxed_u64(p.fs_keys + tid + e * NT);
        if ((uint32_t)(v >> 32) == tag) {
          u[e] = (uint32_t)v;
          pending &= ~(1u << e);
        }
      }
    }
    if (pending && clock64() - t_start > 400000000ll) {
      if (p.err) atomicExch(p.err, ERR_WAIT_TIMEOUT);
      break;
    }
    if (pending) __nanosleep(64);  // keep the polls from crowding the publishers' traffic
  }
  NKV_STAMP(trc, 40);
  topk_threshold<NW>(u, live, n, k, s_sel, s_cand, s_misc, trc);
}

// Ranked decode: the top k (<= 32) of the n fp32 block scores written by the
// scoring grid, into s_sel (topk_threshold).  All threads of the CTA must call.
template <int NW>
__device__ void rank_topk(const float* __restrict__ scores, int n, int k, u64* s_sel, u64* s_cand,
                          unsigned* s_misc, int* trc) {
  constexpr int NT = NW * 32;
  const int tid = threadIdx.x;
  uint32_t u[FS_MAXE];
  unsigned live = 0u;
#pragma unroll
  for (int e = 0; e < FS_MAXE; ++e) {
    const int i = tid + e * NT;
    u[e] = 0u;
    if (i < n) {
      u[e] = f32_order(__ldcg(scores + i));
      live |= 1u << e;
    }
  }
  topk_threshold<NW>(u, live, n, k, s_sel, s_cand, s_misc, trc);
}
// rank_topk over the max across ranks of the tagged scores in this rank's
// exchange buffer: every (rank, block) word of the thread is loaded in one
// pass (all ranks' loads in flight together, one round trip), then only the
// words not yet carrying this step's tag are polled again (bounded, then
// ERR_WAIT_TIMEOUT and the stale value).
template <int NW>
__device__ void rank_topk_peer(const AttendParams& p, uint32_t ep, u64* s_sel, u64* s_cand, unsigned* s_misc,
                               int* trc) {
  constexpr int NT = NW * 32;
  static_assert(NKV_MAX_PEERS * FS_MAXE <= 64, "one pending bit per (rank, key) word");
  const int tid = threadIdx.x;
  const uint32_t tag = step_tag(ep);
  const u64* xs = p.xp_scores + (long long)(ep & 1u) * p.xp_P * p.xp_cap;
  float v[FS_MAXE];
  unsigned live = 0u;
#pragma unroll
  for (int e = 0; e < FS_MAXE; ++e) {
    v[e] = -INFINITY;
    if (tid + e * NT < p.rank_n) live |= 1u << e;
  }
  u64 pending = 0ull;  // bit r * FS_MAXE + e: word (rank r, key e) still without the tag
  for (int r = 0; r < p.xp_P; ++r) {
#pragma unroll
    for (int e = 0; e < FS_MAXE; ++e) {
      if (!((live >> e) & 1u)) continue;
      const u64 w = ld_peer_u64(xs + (long long)r * p.xp_cap + tid + e * NT);
      if ((uint32_t)(w >> 32) == tag) v[e] = fmaxf(v[e], f32_unorder((uint32_t)w));
      else pending |= 1ull << (r * FS_MAXE + e);
    }
  }
  const long long t0 = clock64();
  while (pending) {
    u64 left = pending;
    while (left) {
      const int b = __ffsll((long long)left) - 1;
      left &= left - 1ull;
      const int r = b / FS_MAXE, e = b % FS_MAXE;
      const u64 w = ld_peer_u64(xs + (long long)r * p.xp_cap + tid + e * NT);
      if ((uint32_t)(w >> 32) == tag) {
#pragma unroll
        for (int x = 0; x < FS_MAXE; ++x)  // v[e] with e known only at run time: keep v in registers
          if (x == e) v[x] = fmaxf(v[x], f32_unorder((uint32_t)w));
        pending &= ~(1ull << b);
      }
    }
    if (pending && clock64() - t0 > PEER_WAIT_CYCLES) {
      if (p.err) atomicExch(p.err, ERR_WAIT_TIMEOUT);
      break;
    }
  }
  uint32_t u[FS_MAXE];
#pragma unroll
  for (int e = 0; e < FS_MAXE; ++e) u[e] = ((live >> e) & 1u) ? f32_order(v[e]) : 0u;
  topk_threshold<NW>(u, live, p.rank_n, p.n_sel, s_sel, s_cand, s_misc, trc);
}

// The launch is done with its keys once every CTA has arrived here: the last
// CTA resets the arrival count and advances the epoch (read by the next launch).
__device__ __forceinline__ void fs_arrive(const AttendParams& p) {
  const unsigned total = gridDim.x * gridDim.y;
  if (atomicAdd(p.fs_sync + 1, 1u) == total - 1u) {
    p.fs_sync[1] = 0u;
    atomicAdd(p.fs_sync, 1u);
  }
}

// Rows [pos0, pos0 + len) of the logical keys, loaded by the threads of the
// CTA into tile rows row0... : 16-byte copies for bf16 sources (the current
// tokens, a host-resident store, any segment TMA cannot address), in-register
// dequant for an int8 store (reference scheme: per-channel K scale, per-block
// V scale; token scheme: per-token bf16 scales).
__device__ void thread_rows(const AttendParams& p, int h, int pos0, int len, int row0, unsigned char* kt,
                            unsigned char* vt, int NR, const long long* s_ids, int slot0, int selEnd, int sinkEnd,
                            int ringEnd, int ring_start) {
  const int B = p.B;
  if (pos0 < selEnd && p.kind != NKV_STORE_BF16) {
    const signed char* kst = reinterpret_cast<const signed char*>(p.k_store);
    const signed char* vst = reinterpret_cast<const signed char*>(p.v_store);
    for (int i = threadIdx.x; i < len * 8; i += blockDim.x) {
      const int r = i >> 3, c = i & 7, pos = pos0 + r, off = pos & (B - 1);
      long long id = s_ids[(pos >> p.log2B) - slot0];
      if (id < 0) id = 0;  // masked in the scores
      const long long o = ((id * p.hkv + h) * B + off) * NKV_D + c * 16;
      if (!NKV_INB(p.err, 14, o, 16, p.ext_store)) continue;
      const uint4 kr = ldg_nc_v4(kst + o), vr = ldg_nc_v4(vst + o);
      const signed char* kb = reinterpret_cast<const signed char*>(&kr);
      const signed char* vb = reinterpret_cast<const signed char*>(&vr);
      uint32_t kw[8], vw[8];
      if (p.kind == NKV_STORE_INT8_REF) {
        const float vsc = __ldg(p.vbs + id * p.hkv + h);
#pragma unroll
        for (int e = 0; e < 16; e += 2) {
          const int d = c * 16 + e;
          const float k0 = (float)kb[e] * __ldg(p.kcs + h * NKV_D + d);
          const float k1 = (float)kb[e + 1] * __ldg(p.kcs + h * NKV_D + d + 1);
          kw[e / 2] = (uint32_t)f2bf(k0) | ((uint32_t)f2bf(k1) << 16);
          vw[e / 2] = (uint32_t)f2bf((float)vb[e] * vsc) | ((uint32_t)f2bf((float)vb[e + 1] * vsc) << 16);
        }
      } else {
        const long long so = (id * p.hkv + h) * B + off;
        const float ksc = __bfloat162float(p.kts[so]);
        const float vsc = __bfloat162float(p.vts[so]);
#pragma unroll
        for (int e = 0; e < 16; e += 2) {
          kw[e / 2] = (uint32_t)f2bf((float)kb[e] * ksc) | ((uint32_t)f2bf((float)kb[e + 1] * ksc) << 16);
          vw[e / 2] = (uint32_t)f2bf((float)vb[e] * vsc) | ((uint32_t)f2bf((float)vb[e + 1] * vsc) << 16);
        }
      }
      const int row = row0 + r;
      *reinterpret_cast<uint4*>(kt + swz(NR, row, c * 16)) = make_uint4(kw[0], kw[1], kw[2], kw[3]);
      *reinterpret_cast<uint4*>(kt + swz(NR, row, c * 16 + 8)) = make_uint4(kw[4], kw[5], kw[6], kw[7]);
      *reinterpret_cast<uint4*>(vt + swz(NR, row, c * 16)) = make_uint4(vw[0], vw[1], vw[2], vw[3]);
      *reinterpret_cast<uint4*>(vt + swz(NR, row, c * 16 + 8)) = make_uint4(vw[4], vw[5], vw[6], vw[7]);
    }
    return;
  }
  for (int i = threadIdx.x; i < len * 16; i += blockDim.x) {
    const int r = i >> 4, c = i & 15, pos = pos0 + r;
    const __nv_bfloat16 *ksrc, *vsrc;
    long long o;
    [[maybe_unused]] long long ext;
    if (pos < selEnd) {
      long long id = s_ids[(pos >> p.log2B) - slot0];
      if (id < 0) id = 0;
      o = ((id * p.hkv + h) * B + (pos & (B - 1))) * NKV_D;
      ksrc = reinterpret_cast<const __nv_bfloat16*>(p.k_store);
      vsrc = reinterpret_cast<const __nv_bfloat16*>(p.v_store);
      ext = p.ext_store;
    } else if (pos < sinkEnd) {
      o = ((long long)h * p.sink_cap + (pos - selEnd)) * NKV_D;
      ksrc = p.sink_k;
      vsrc = p.sink_v;
      ext = p.ext_sink;
    } else if (pos < ringEnd) {
      int phys = ring_start + (pos - sinkEnd);
      if (phys >= p.ring_cap) phys -= p.ring_cap;
      o = ((long long)h * p.ring_cap + phys) * NKV_D;
      ksrc = p.ring_k;
      vsrc = p.ring_v;
      ext = p.ext_ring;
    } else {
      o = (long long)(pos - ringEnd) * p.cur_row + (long long)h * p.cur_head;
      ksrc = p.cur_k;
      vsrc = p.cur_v;
      ext = p.ext_cur;
    }
    if (!NKV_INB(p.err, 15, o + c * 8, 8, ext)) continue;
    const uint4 kv = ldg_nc_v4(ksrc + o + c * 8), vv = ldg_nc_v4(vsrc + o + c * 8);
    *reinterpret_cast<uint4*>(kt + swz(NR, row0 + r, c * 8)) = kv;
    *reinterpret_cast<uint4*>(vt + swz(NR, row0 + r, c * 8)) = vv;
  }
}

// Single-query decode (nq == 1) on the tensor cores.
//  data:   the CTA's keys are cut into pieces that are contiguous in one
//          source (a selected block, the sink, one or two runs of the recent
//          ring, the current token).  A piece in device memory is fetched by
//          2D TMA boxes of 8 rows x 64 columns into its own 8-row-aligned rows
//          of the swizzled tiles, with one mbarrier for its K and one for its
//          V; the rest (current tokens, int8 or host-resident blocks) is loaded
//          by the threads.  Copies that do not depend on the selection are
//          issued before the programmatic-dependent-launch wait, the selected
//          blocks right after it.
//  math:   a warp owns a slice of up to 48 keys and starts as soon as the
//          pieces of its slice have landed.  S = Q K^T with mma.sync m16n8k16
//          (A = the G query rows, rows >= G zero; B = K via ldmatrix), softmax
//          on the accumulator fragments, O += P V with P as the bf16 A operand
//          and V via ldmatrix.trans.
//  merge:  warp partials through shared memory (over the K tile, after every
//          warp is done with it), then the splits of a head through the
//          cluster (DSMEM) or the workspace.
template <int G, bool FS = false>
__global__ void __launch_bounds__(DK<G>::THREADS) decode_kernel(const AttendParams p,
                                                               const __grid_constant__ DecodeMaps tm) {
  extern __shared__ __align__(16) unsigned char sm_raw[];
  __shared__ __align__(8) uint64_t kbar[AT_MAX_PIECES], vbar[AT_MAX_PIECES];
  __shared__ int plo[AT_MAX_PIECES + 1], plen[AT_MAX_PIECES], prow[AT_MAX_PIECES], ptype[AT_MAX_PIECES];
  __shared__ unsigned s_thr[2];  // pieces the threads load (bit i of the 64-bit pair = piece i)
  __shared__ unsigned s_ticket;
  __shared__ long long s_ids[AT_MAX_SLOTS];
  __shared__ short srow[AT_TPS_MAX_CLUSTER];
  constexpr int NW = DK<G>::WARPS;
  // one-launch step: per-block score maxima, the selected keys, the radix
  // histogram and the scan's warp sums
  __shared__ unsigned s_part[NW][FS_BPC_MAX];
  __shared__ u64 s_sel[32];
  __shared__ u64 s_cand[FS_CAND_MAX];
  __shared__ unsigned s_misc[2 * NW];

  const int split = blockIdx.x, h = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int t0 = split * p.tps, t1 = min(p.ntok, t0 + p.tps), n = t1 - t0;
  const int B = p.B;
  const int selEnd = p.n_sel * B, sinkEnd = selEnd + p.sink_len, ringEnd = sinkEnd + p.ring_len;
  const int slot0 = t0 >> p.log2B;
  const int nslots = t0 < selEnd ? ((min(t1, selEnd) - 1) >> p.log2B) - slot0 + 1 : 0;
  const int NR = p.tile_rows;
  unsigned char* sm = sm_raw + ((1024u - (smem_u32(sm_raw) & 1023u)) & 1023u);
  unsigned char* kt = sm;                          // K tile, later the warp partials
  unsigned char* vt = sm + (size_t)p.region_k;     // V tile, later the CTA partial

#ifdef NKV_CHECKED
  int* trc = p.trace ? p.trace + (blockIdx.y * gridDim.x + blockIdx.x) * 64 : nullptr;
#else
  [[maybe_unused]] int* trc = nullptr;
#endif
  NKV_STAMP(trc, 48);
  // a kernel launched after this one with programmatic dependent launch (the
  // next layer's scoring grid) may become resident now; it waits for this
  // grid's completion before reading anything
  if (!FS) pdl_launch_dependents();
  // recent ring: explicit (arguments) or device-resident (graph replay).  With
  // a device head only the CTAs holding ring keys or the current token read
  // it (splits from sinkEnd / tps on: the others keep it off their prologue);
  // the last of those readers to arrive advances it, and the CTA holding the
  // current token writes it into the ring.
  int ring_start = p.ring_start, ring_wpos = p.ring_write_pos;
  const bool ring_writer = p.ring_dyn ? split == (int)gridDim.x - 1 : split == 0;
  if (p.ring_dyn) {
    ring_wpos = -1;
    const int first_reader = sinkEnd / p.tps;
    if (split >= first_reader) {
      // (the arrival that lets the last reader advance the head comes after
      // the prologue, once the head is in use: its round trip stays off the
      // CTA's first barrier)
      __shared__ int s_head;
      if (tid == 0) s_head = ld_relaxed_s32(p.ring_dyn);
      __syncthreads();
      ring_wpos = s_head;
      ring_start = s_head + p.ring_cap - p.ring_len;
      if (ring_start >= p.ring_cap) ring_start -= p.ring_cap;
    }
  }
  // peer exchange: this step's epoch (advanced only after every CTA read it)
  const uint32_t xp_ep = p.xp_P ? ld_peer_u32(p.xp_sync) : 0u;
  // one-launch step: this launch's tag (the epoch load overlaps the prologue)
  uint32_t fs_tg = 0u;
  if constexpr (FS) {
    fs_tg = fs_tag(ld_relaxed_u32(p.fs_sync));
    for (int i = tid; i < NW * FS_BPC_MAX; i += NW * 32) s_part[i / FS_BPC_MAX][i % FS_BPC_MAX] = 0u;
    // the representatives this CTA scores, one contiguous range per KV head
    const int b0 = (h * gridDim.x + split) * p.fs_bpc, nb = min(p.fs_bpc, p.rank_n - b0);
    if (p.fs_prefetch && tid < p.hkv && nb > 0)
      prefetch_l2_bulk(p.fs_reps + ((long long)tid * p.fs_reps_blocks + b0) * p.fs_r * NKV_D,
                       (uint32_t)(nb * p.fs_r * NKV_D * 2));
  }

  // ---- pieces ------------------------------------------------------------------------
  // Fixed table: pieces [0, nslots) are the selected blocks the range touches,
  // then the sink, the ring run up to the physical wrap, the run after it and
  // the current tokens (each possibly empty).  Piece i is computed by thread i
  // in O(1).  Selected pieces keep their key offset as tile row (their lengths
  // are multiples of 8 because tps and block_size are); the others follow,
  // each rounded up to 8 rows.
  const int np = nslots + 4;
  bool by_threads = false;
  if (tid < np) {
    auto clampk = [&](int x) { return min(max(x, t0), t1); };
    int a, b, row = 0, type;
    if (tid < nslots) {
      a = max(t0, (slot0 + tid) * B);
      b = min(min(t1, selEnd), (slot0 + tid + 1) * B);
      row = a - t0;
      type = (p.tma_mask & 1) ? PT_SEL : PT_THREADS;
      // every sel_thr_every-th selected piece by the threads (16-byte loads)
      // beside the TMA boxes of the others: two load paths into the SM
      if (p.sel_thr_every > 0 && tid % p.sel_thr_every == p.sel_thr_every - 1) type = PT_THREADS;
    } else {
      const int k = tid - nslots;  // 0 sink, 1 ring before the wrap, 2 ring after it, 3 current
      const int wrap = min(ringEnd, sinkEnd + (p.ring_cap - ring_start));
      const int e0 = clampk(selEnd), e1 = clampk(sinkEnd), e2 = clampk(wrap), e3 = clampk(ringEnd);
      row = e0 - t0;
      if (k >= 1) row += (e1 - e0 + 7) & ~7;
      if (k >= 2) row += (e2 - e1 + 7) & ~7;
      if (k >= 3) row += (e3 - e2 + 7) & ~7;
      a = k == 0 ? e0 : k == 1 ? e1 : k == 2 ? e2 : e3;
      b = k == 0 ? e1 : k == 1 ? e2 : k == 2 ? e3 : t1;
      type = k == 0 ? ((p.tma_mask & 2) ? PT_SINK : PT_THREADS)
                    : k == 3 ? PT_THREADS : ((p.tma_mask & 4) ? PT_RING : PT_THREADS);
    }
    const int len = b - a;
    if (len <= 0) {
      type = PT_EMPTY;
    } else if (row + ((len + 7) & ~7) > NR) {  // never taken: tps + 32 rows hold every table
      if (p.err) atomicExch(p.err, ERR_BOUNDS);
      type = PT_SKIP;
      row = 0;
    }
    by_threads = type == PT_THREADS;
    plo[tid] = a - t0;
    plen[tid] = len > 0 ? len : 0;
    prow[tid] = row;
    ptype[tid] = type;
    if (tid == np - 1) plo[np] = n;
    if (type <= PT_RING) {
      const uint32_t bytes = (uint32_t)((len + 7) & ~7) * 256u;  // K (or V): rows x 2 halves x 128 B
      mbar_init(&kbar[tid], 1);
      mbar_init(&vbar[tid], 1);
      fence_mbar_init();
      mbar_expect_tx(&kbar[tid], bytes);
      mbar_expect_tx(&vbar[tid], bytes);
    }
  }
  // (after the barrier initialisation: its fence would wait for these loads)
  if (tid >= 64 && tid < 76 && ((p.tma_mask >> ((tid - 64) >> 2)) & 1)) {
    const int m = tid - 64;
    prefetch_tmap(&tm.m[m >> 2][(m >> 1) & 1][m & 1]);
  }
  // block ids: read now unless they come from the grid this one overlaps
  long long id_early = 0;
  if (!FS && !p.overlap && !p.rank_scores && !p.xp_P && tid < nslots) id_early = __ldg(p.ids + slot0 + tid);
  if (warp < 2) {  // np <= AT_MAX_SLOTS + 4 pieces live in warps 0 and 1
    const unsigned bits = __ballot_sync(FULL, by_threads);
    if (lane == 0) s_thr[warp] = bits;
  }
  // Q as the A operand (rows >= G are zero), loaded while the table is built
  const int qg = lane >> 2, qt = lane & 3;
  uint32_t qa[8][2];
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    if (qg < G) {
      const __nv_bfloat16* qrow = p.q + (long long)(h * G + qg) * p.q_head + kk * 16 + 2 * qt;
      qa[kk][0] = __ldg(reinterpret_cast<const uint32_t*>(qrow));
      qa[kk][1] = __ldg(reinterpret_cast<const uint32_t*>(qrow + 8));
    } else {
      qa[kk][0] = qa[kk][1] = 0u;
    }
  }
  __syncthreads();
  NKV_STAMP(trc, 61);
  const unsigned long long thr_pieces = ((unsigned long long)s_thr[1] << 32) | s_thr[0];
  // token -> tile row, written by the warp that owns the piece (i % NW)
  for (int i = warp; i < np; i += NW)
    for (int r = lane; r < plen[i]; r += 32) srow[plo[i] + r] = (short)(ptype[i] == PT_SKIP ? 0 : prow[i] + r);
  // sink and ring pieces: TMA boxes, piece i issued by warp i % NW
  for (int i = warp; i < np; i += NW) {
    const int type = ptype[i];
    if (type != PT_SINK && type != PT_RING) continue;
    const int pos0 = t0 + plo[i];
    int y0;
    if (type == PT_SINK) {
      y0 = h * p.sink_cap + (pos0 - selEnd);
    } else {
      int phys = ring_start + (pos0 - sinkEnd);
      if (phys >= p.ring_cap) phys -= p.ring_cap;
      y0 = h * p.ring_cap + phys;
    }
    issue_piece(tm, type, y0, plen[i], prow[i], kt, vt, NR, &kbar[i], &vbar[i], lane);
  }
  // decode: append the current token to the recent ring (a slot no CTA reads)
  if (ring_writer && ring_wpos >= 0 && tid >= 64 && tid < 96 &&
      NKV_INB(p.err, 40, ((long long)h * p.ring_cap + ring_wpos) * NKV_D, NKV_D, p.ext_ring) &&
      NKV_INB(p.err, 41, h * p.cur_head, NKV_D, p.ext_cur)) {
    const int c = tid & 15;
    const bool isv = (tid & 16) != 0;
    const __nv_bfloat16* src = (isv ? p.cur_v : p.cur_k) + h * p.cur_head + c * 8;
    __nv_bfloat16* dst = (isv ? p.ring_v : p.ring_k) + ((long long)h * p.ring_cap + ring_wpos) * NKV_D + c * 8;
    *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
  }
  // thread-loaded pieces outside the selected segment
  for (unsigned long long m = thr_pieces; m; m &= m - 1) {
    const int i = __ffsll((long long)m) - 1;
    if (t0 + plo[i] >= selEnd)
      thread_rows(p, h, t0 + plo[i], plen[i], prow[i], kt, vt, NR, s_ids, slot0, selEnd, sinkEnd, ringEnd,
                  ring_start);
  }
  if (p.ring_dyn && tid == 0 && split >= sinkEnd / p.tps) {
    // device ring head: this CTA has read it (ring_wpos holds it); the last of
    // the readers to arrive advances it for the next step
    const unsigned readers = (gridDim.x - (unsigned)(sinkEnd / p.tps)) * gridDim.y;
    if (atomicAdd(reinterpret_cast<unsigned*>(p.ring_dyn + 1), 1u) == readers - 1u) {
      p.ring_dyn[1] = 0;
      p.ring_dyn[0] = ring_wpos + 1 == p.ring_cap ? 0 : ring_wpos + 1;
    }
  }
  NKV_STAMP(trc, 62);
  if (p.overlap) pdl_wait();  // block ids (or scores) are complete past this point
  if constexpr (FS) {
    // one-launch step: score this CTA's blocks, then (CTAs that hold selected
    // blocks, and CTA (0, 0), which publishes the ids) select from every
    // CTA's published keys; slots take the selected blocks in rank order
    fs_score_publish<G, NW>(p, h * gridDim.x + split, fs_tg, s_part, trc);
    NKV_STAMP(trc, 46);
    if (nslots > 0 || (split == 0 && h == 0)) {
      fs_select<NW>(p, fs_tg, s_sel, s_cand, s_misc, trc);
      NKV_STAMP(trc, 47);
      if (tid < nslots) {
        const long long id = (long long)key_id(s_sel[slot0 + tid]);
        const bool bad = id >= p.rank_n;  // only after a timed-out wait
        if (bad && p.err) atomicExch(p.err, ERR_BAD_INDEX);
        s_ids[tid] = bad ? -1 : id;
      }
    }
    if (tid == 0) fs_arrive(p);
  } else if (p.rank_scores || p.xp_P) {
    // ranked mode: the CTAs that hold selected blocks (and CTA (0, 0), which
    // publishes the ids) rank the block scores themselves (with a peer
    // exchange: the max over ranks of the scores in the exchange buffer)
    if (nslots > 0 || (split == 0 && h == 0)) {
      if (p.xp_P)
        rank_topk_peer<NW>(p, xp_ep, s_sel, s_cand, s_misc, trc);
      else
        rank_topk<NW>(p.rank_scores, p.rank_n, p.n_sel, s_sel, s_cand, s_misc, trc);
      if (tid < nslots) s_ids[tid] = (long long)key_id(s_sel[slot0 + tid]);
      if (split == 0 && h == 0 && tid < p.n_sel) {
        p.rank_out[tid] = (long long)key_id(s_sel[tid]);
        if (p.rank_out_scores) p.rank_out_scores[tid] = key_score(s_sel[tid]);
      }
    }
  } else if (tid < nslots) {
    const long long id = p.overlap ? __ldg(p.ids + slot0 + tid) : id_early;
    const bool bad = id < 0 || id >= p.max_blocks;
    if (bad && p.err) atomicExch(p.err, ERR_BAD_INDEX);
    s_ids[tid] = bad ? -1 : id;
  }
  __syncthreads();
  NKV_STAMP(trc, 49);
  NKV_STAMP(trc, 30);
  // selected blocks: TMA boxes (piece i issued by warp i % NW), or the threads
  // (int8, host-resident)
  for (int i = warp; i < np; i += NW) {
    if (ptype[i] != PT_SEL) continue;
    const int pos0 = t0 + plo[i];
    long long id = s_ids[(pos0 >> p.log2B) - slot0];
    if (id < 0) id = 0;  // masked in the scores
    const int y0 = (int)((id * p.hkv + h) * B + (pos0 & (B - 1)));
    if (i == 0) NKV_STAMP(trc, 31);
    issue_piece(tm, PT_SEL, y0, plen[i], prow[i], kt, vt, NR, &kbar[i], &vbar[i], lane);
    if (i == 0) NKV_STAMP(trc, 42);
  }
  NKV_STAMP(trc, 43);
  if (FS && split == 0 && h == 0 && warp == NW - 1 && lane < p.n_sel) {
    // the selected ids in rank order
    p.rank_out[lane] = (long long)key_id(s_sel[lane]);
    if (p.rank_out_scores) p.rank_out_scores[lane] = key_score(s_sel[lane]);
  }
  NKV_STAMP(trc, 63);
  for (unsigned long long m = thr_pieces; m; m &= m - 1) {
    const int i = __ffsll((long long)m) - 1;
    if (t0 + plo[i] < selEnd)
      thread_rows(p, h, t0 + plo[i], plen[i], prow[i], kt, vt, NR, s_ids, slot0, selEnd, sinkEnd, ringEnd,
                  ring_start);
  }
  __syncthreads();  // thread-loaded rows visible
  NKV_STAMP(trc, 50);

  // ---- this warp's slice [lo, hi), 8-aligned -----------------------------------------
  const int tpw = ((n + NW - 1) / NW + 7) / 8 * 8;
  const int lo = min(n, warp * tpw), hi = min(n, lo + tpw);
  int pa = 0, pb = -1;
  if (lo < hi) {
    while (pa + 1 < np && plo[pa + 1] <= lo) ++pa;
    pb = pa;
    while (pb + 1 < np && plo[pb + 1] < hi) ++pb;
  }
  for (int i = pa; i <= pb; ++i)
    if (ptype[i] <= PT_RING) mbar_wait_poll(&kbar[i], 0, p.err);
  NKV_STAMP(trc, 51);

  // slices hold at most 48 keys (tps <= 384 over 8 warps, rounded to 8)
  constexpr int MAXT = AT_TPS_MAX_CLUSTER / (8 * NW);  // n-tiles of 8 keys per warp slice
  float sfr[MAXT][4], sfr2[MAXT][4];
  const int ntile = (hi - lo + 7) / 8;
  // ldmatrix row address pattern: lane i feeds row (i & 7) of matrix (i >> 3)
  const int mrow = lane & 7, msel = lane >> 3;
  int rowj[MAXT];
#pragma unroll
  for (int j = 0; j < MAXT; ++j) {
    sfr[j][0] = sfr[j][1] = sfr[j][2] = sfr[j][3] = 0.f;
    sfr2[j][0] = sfr2[j][1] = sfr2[j][2] = sfr2[j][3] = 0.f;
    int t = lo + j * 8 + mrow;
    if (t >= hi) t = lo;  // only this slice's rows are known to have landed; masked below
    rowj[j] = j < ntile ? srow[t] : 0;
  }
  // k-steps outermost, the ldmatrix of every n-tile issued before the mma
  // that use them, and two accumulators per n-tile (even / odd k-steps): the
  // asm statements keep their order, so the order written here is the
  // schedule; consecutive mma.sync are independent.
#pragma unroll
  for (int kk = 0; kk < 8; kk += 2) {
    // matrices: (kk, lo 8 dims), (kk, hi 8 dims), (kk+1, lo), (kk+1, hi)
    uint32_t b[MAXT][4];
#pragma unroll
    for (int j = 0; j < MAXT; ++j)
      if (j < ntile) ldsm_x4(b[j], kt + swz(NR, rowj[j], (kk + (msel >> 1)) * 16 + (msel & 1) * 8));
#pragma unroll
    for (int j = 0; j < MAXT; ++j)
      if (j < ntile) mma_bf16(sfr[j], qa[kk][0], 0u, qa[kk][1], 0u, b[j][0], b[j][1]);
#pragma unroll
    for (int j = 0; j < MAXT; ++j)
      if (j < ntile) mma_bf16(sfr2[j], qa[kk + 1][0], 0u, qa[kk + 1][1], 0u, b[j][2], b[j][3]);
  }
#pragma unroll
  for (int j = 0; j < MAXT; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) sfr[j][e] += sfr2[j][e];
  NKV_STAMP(trc, 58);
  // mask + scale; lane holds row qg keys lo + 8j + 2qt + {0, 1}.  Bit i of
  // vis = key lo + i of the slice is visible (two keys per lane, one ballot each).
  const unsigned long long vis =
      (unsigned long long)__ballot_sync(FULL, lo + lane < hi &&
                                                  visible(p, t0 + lo + lane, 0, selEnd, ringEnd, s_ids, slot0)) |
      ((unsigned long long)__ballot_sync(FULL, lo + 32 + lane < hi &&
                                                   visible(p, t0 + lo + 32 + lane, 0, selEnd, ringEnd, s_ids, slot0))
       << 32);
  const unsigned long long visq = qg < G ? vis >> (2 * qt) : 0ull;
  float mloc = -INFINITY;
#pragma unroll
  for (int j = 0; j < MAXT; ++j) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float sv = ((visq >> (j * 8 + e)) & 1ull) ? sfr[j][e] * p.scale : -INFINITY;
      sfr[j][e] = sv;
      mloc = fmaxf(mloc, sv);
    }
  }
  mloc = fmaxf(mloc, __shfl_xor_sync(FULL, mloc, 1));
  mloc = fmaxf(mloc, __shfl_xor_sync(FULL, mloc, 2));
  float lloc = 0.f;
#pragma unroll
  for (int j = 0; j < MAXT; ++j)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float pe = (mloc == -INFINITY || sfr[j][e] == -INFINITY) ? 0.f : __expf(sfr[j][e] - mloc);
      sfr[j][e] = pe;
      lloc += pe;
    }
  lloc += __shfl_xor_sync(FULL, lloc, 1);
  lloc += __shfl_xor_sync(FULL, lloc, 2);
  NKV_STAMP(trc, 52);
  for (int i = pa; i <= pb; ++i)
    if (ptype[i] <= PT_RING) mbar_wait_poll(&vbar[i], 0, p.err);
  NKV_STAMP(trc, 53);

  // O += P V: k-steps of 16 keys (two n-tiles of scores), 16 n-tiles of 8 dims
  float ofr[16][4];
#pragma unroll
  for (int d = 0; d < 16; ++d) ofr[d][0] = ofr[d][1] = ofr[d][2] = ofr[d][3] = 0.f;
#pragma unroll
  for (int ksx = 0; ksx < (MAXT + 1) / 2; ++ksx) {
    if (2 * ksx < ntile) {
      const uint32_t pa0 = pack_bf16x2(sfr[2 * ksx][0], sfr[2 * ksx][1]);
      const uint32_t pa2 = 2 * ksx + 1 < MAXT ? pack_bf16x2(sfr[2 * ksx + 1][0], sfr[2 * ksx + 1][1]) : 0u;
      // ldmatrix.trans rows: keys lo + 16 ksx + (msel & 1) * 8 + mrow, dims + (msel >> 1) * 8
      int t = lo + ksx * 16 + (msel & 1) * 8 + mrow;
      if (t >= hi) t = lo;  // landed, finite values times p = 0
      const int row = srow[t];
      // the eight ldmatrix of the k-step first, then its sixteen mma
      uint32_t b[8][4];
#pragma unroll
      for (int dn = 0; dn < 16; dn += 2) ldsm_x4_t(b[dn / 2], vt + swz(NR, row, dn * 8 + (msel >> 1) * 8));
#pragma unroll
      for (int dn = 0; dn < 16; dn += 2) {
        mma_bf16(ofr[dn], pa0, 0u, pa2, 0u, b[dn / 2][0], b[dn / 2][1]);
        mma_bf16(ofr[dn + 1], pa0, 0u, pa2, 0u, b[dn / 2][2], b[dn / 2][3]);
      }
    }
  }
  float* wpo = reinterpret_cast<float*>(kt);  // [NW][G][D] over the K tile
  float* wml = wpo + NW * G * NKV_D;          // [NW][G][2]
  float* pm = reinterpret_cast<float*>(vt);   // [G] CTA partial over the V tile
  float* pl = pm + 64;
  float* po = pl + 64;                        // [G][D]
  __syncthreads();  // every warp is done with the K tile
  // warp partial: rows qg < G hold o[qg][8 dn + 2 qt + {0,1}]
  if (qg < G) {
#pragma unroll
    for (int dn = 0; dn < 16; ++dn)
      *reinterpret_cast<float2*>(wpo + (warp * G + qg) * NKV_D + dn * 8 + 2 * qt) = make_float2(ofr[dn][0], ofr[dn][1]);
    if (qt == 0) {
      wml[(warp * G + qg) * 2] = lo < hi ? mloc : -INFINITY;
      wml[(warp * G + qg) * 2 + 1] = lo < hi ? lloc : 0.f;
    }
  }
  __syncthreads();  // warp partials complete; every warp is done with the V tile
  NKV_STAMP(trc, 54);

  // ---- merge the warp slices into the CTA partial -----------------------------------
  float* dst_o = p.cluster ? po : p.part_o + (((long long)h * p.splits + split) * G) * NKV_D;
  for (int it = tid; it < G * (NKV_D / 4); it += DK<G>::THREADS) {
    const int g = it / (NKV_D / 4), d4 = it % (NKV_D / 4);
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < NW; ++w) M = fmaxf(M, wml[(w * G + g) * 2]);
    float L = 0.f;
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      const float m = wml[(w * G + g) * 2];
      if (m == -INFINITY) continue;
      const float sw = __expf(m - M);
      L += sw * wml[(w * G + g) * 2 + 1];
      const float4 v = *reinterpret_cast<const float4*>(wpo + (w * G + g) * NKV_D + d4 * 4);
      o.x = fmaf(sw, v.x, o.x);
      o.y = fmaf(sw, v.y, o.y);
      o.z = fmaf(sw, v.z, o.z);
      o.w = fmaf(sw, v.w, o.w);
    }
    *reinterpret_cast<float4*>(dst_o + g * NKV_D + d4 * 4) = o;
    if (d4 == 0) {
      if (p.cluster) {
        pm[g] = M;
        pl[g] = L;
      } else {
        float* ml = p.part_ml + (((long long)h * p.splits + split) * G + g) * 2;
        ml[0] = M;
        ml[1] = L;
      }
    }
  }
  NKV_STAMP(trc, 55);
  if (p.cluster) {
    combine_cluster<G>(p, h, pm, pl, po, xp_ep);  // begins and ends with a cluster barrier
    if (p.xp_P && split == 0) peer_pull_arrive<G>(p, h, xp_ep);
    NKV_STAMP(trc, 57);
    return;
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) s_ticket = atomicAdd(p.counters + h, 1u);
  __syncthreads();
  if (s_ticket != (unsigned)p.splits - 1) return;
  __threadfence();
  if (tid == 0) p.counters[h] = 0u;
  combine_splits<G>(p, h, reinterpret_cast<float*>(kt), xp_ep);
  if (p.xp_P) peer_pull_arrive<G>(p, h, xp_ep);
}

// Cluster merge: the CTAs of one cluster are the splits of one KV head.  After
// a cluster barrier, the output is cut into tasks of 32 dims of one query row;
// task t is done by warp (t / C) % warps of CTA t % C in one DSMEM round trip:
// lane q < C reads split q's (m, l), every lane reads its dim of all C partial
// outputs, then the weights exp(m_q - M) travel by shuffle.  A second barrier
// keeps every CTA's shared memory alive until its peers are done reading.
template <int G>
__device__ void combine_cluster(const AttendParams& p, int h, float* pm, float* pl, float* po, uint32_t xp_ep) {
  cg::cluster_group cluster = cg::this_cluster();
  const int C = (int)cluster.num_blocks();
  const int rank = (int)cluster.block_rank();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (int)blockDim.x >> 5;
  const int tasks = p.nr * (NKV_D / 32);
  cluster.sync();
#ifdef NKV_CHECKED
  int* trc = p.trace ? p.trace + (blockIdx.y * gridDim.x + blockIdx.x) * 64 : nullptr;
  NKV_STAMP(trc, 59);
#endif
  for (int task = rank + C * warp; task < tasks; task += C * nw) {
    const int row = task >> 2, d = (task & 3) * 32 + lane;
    float mq = -INFINITY, lq = 0.f;
    if (lane < C) {
      mq = *cluster.map_shared_rank(pm + row, lane);
      lq = *cluster.map_shared_rank(pl + row, lane);
    }
    float v[AT_CLUSTER_MAX];
#pragma unroll
    for (int q = 0; q < AT_CLUSTER_MAX; ++q) v[q] = q < C ? *cluster.map_shared_rank(po + row * NKV_D + d, q) : 0.f;
    float M = mq;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(FULL, M, o));
    const float w = mq == -INFINITY ? 0.f : __expf(mq - M);
    float L = w * lq;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(FULL, L, o);
    float acc = 0.f;
#pragma unroll
    for (int q = 0; q < AT_CLUSTER_MAX; ++q) acc = fmaf(__shfl_sync(FULL, w, q), v[q], acc);
    const int qn = row / G, g = row % G;
    const long long oo = qn * p.out_row + (long long)(h * G + g) * p.out_head + d;
    const float val = acc * (1.f / L);
    if (NKV_INB(p.err, 43, oo, 1, p.ext_out)) p.out[oo] = __float2bfloat16(val);
    if (p.xp_P) {  // peer exchange: dims (d, d + 1) of this row to every other rank
      const float nxt = __shfl_down_sync(FULL, val, 1);
      if (!(lane & 1))
        peer_push(p, xp_ep, ((long long)(p.xp_rank * gridDim.y + h) * G + g) * (NKV_D / 2) + d / 2,
                  pack_bf16x2(val, nxt));
    }
  }
#ifdef NKV_CHECKED
  NKV_STAMP(trc, 60);
#endif
  cluster.sync();
}

// ---------------------------------------------------------------------------
// Tile-split decode kernel (ranked decode, bf16 block store in device memory,
// block size 64, one query).  The grid is one cluster of CL CTAs per KV head;
// the head's keys are cut into 64-key tiles, each one TMA box (two 64-column
// halves) for K and one for V:
//   early tiles  the sink, then the recent ring slice as its run before and
//                after the physical wrap (each run cut into 64-key tiles, the
//                last one partial): they do not depend on the selection, so
//                they are loaded and attended while the scores are produced;
//   selected     one tile per selected block, in rank order;
//   current      the decode token itself (one key, from registers).
// CTA s of a head owns early tiles s, s + CL, ... and selected ranks s,
// s + CL, ... (two ranks and at most one early tile at CL = 16, k = 32: about
// 170 keys per CTA on 128 SMs).  Every CTA ranks the scoring grid's block
// scores itself (topk_threshold), so no id crosses the grid.  Within a CTA a
// warp attends 16-key chunks (warps 0-3 the four chunks of a first tile,
// warps 4-7 those of a second) with its own online softmax state: S = Q K^T
// and O += P V on mma.sync m16n8k16, with P split into a bf16 head and a bf16
// remainder (two P.V products) so that P enters the sum with ~16 significant
// bits, as the reference's fp32 P.V does.  The warp states merge in shared
// memory; each CTA of the head merges D / CL output dims, and every CTA
// pushes the matching parts of its partial into the others with asynchronous
// remote stores (st.async) that complete their merge barriers (no cluster
// barrier on the way out, no remote loads).
// ---------------------------------------------------------------------------
constexpr int DS_WARPS = 8;
constexpr int DS_TILE_BYTES = 64 * 256;  // one K (or V) tile: [2 halves][64 rows][128 B]

// Cluster helpers: split arrive / wait barrier, the shared::cluster address of
// a variable in another CTA's shared memory, and an asynchronous remote store
// that completes `bytes` of the remote mbarrier's transaction count.
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
__device__ __forceinline__ uint32_t cluster_addr(const void* local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(local)), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_async_v4(uint32_t raddr, float4 v, uint32_t rbar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(raddr),
               "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w), "r"(rbar)
               : "memory");
}
__device__ __forceinline__ void st_async_v2(uint32_t raddr, float a, float b, uint32_t rbar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f32 [%0], {%1, %2}, [%3];" ::"r"(raddr), "f"(a),
               "f"(b), "r"(rbar)
               : "memory");
}

template <int CL>
struct DS {
  static constexpr int MAX_EARLY = CL >= 16 ? 1 : 2;       // early tiles per CTA (<= 10 early tiles per head)
  static constexpr int MAX_SEL = 32 / CL;                    // selected tiles per CTA (k <= 32)
  static constexpr int MAX_TILES = MAX_EARLY + MAX_SEL;
  // output dims each CTA of the cluster merges, and the bytes one CTA pushes
  // into another: its partial o for those dims of the 4 query rows, and (m, l)
  static constexpr int SW = NKV_D / CL;
  static constexpr int PUSH_BYTES = 4 * SW * 4 + 4 * 2 * 4;
  // tiles, then the receive area: o [CL][4][SW], (m, l) [CL][4][2]
  static constexpr size_t SMEM = 1024 + (size_t)MAX_TILES * 2 * DS_TILE_BYTES + (size_t)CL * PUSH_BYTES;
};

// Early tiles: the sink (one tile of sink_len rows), then the ring in its
// physical order, 64 slots per tile (softmax is order-independent, so the
// tiles do not depend on the ring head: they are issued before the head is
// read, and the head only decides which of their rows are attended).
// Early tile e of head h: (source, first row in its 2D map).
__device__ __forceinline__ void ds_early_tile(const AttendParams& p, int h, int e, int* src, int* y) {
  if (p.sink_len > 0) {
    if (e == 0) {
      *src = 1;
      *y = h * p.sink_cap;
      return;
    }
    --e;
  }
  *src = 2;
  *y = h * p.ring_cap + e * 64;
}

__device__ __forceinline__ int ds_early_count(const AttendParams& p) {
  return (p.sink_len > 0 ? 1 : 0) + (p.ring_len > 0 ? (p.ring_cap + 63) >> 6 : 0);
}

// The K and V tiles of 64 rows of source src from row y: one whole-tile box
// each where the source has the 3D maps (tma_mask bit 3 + src), else two
// 64-column boxes each.
__device__ __forceinline__ void ds_issue_tile(const DecodeMaps& tm, int tma_mask, int src, int y, unsigned char* kd,
                                              uint64_t* bar) {
  mbar_expect_tx(bar, 2 * DS_TILE_BYTES);
  if ((tma_mask >> (3 + src)) & 1) {
    tma_tile3(kd, &tm.t3[src][0], y, bar);
    tma_tile3(kd + DS_TILE_BYTES, &tm.t3[src][1], y, bar);
  } else {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      tma_box(kd + half * (64 * 128), &tm.m[src][0][1], half * 64, y, bar);
      tma_box(kd + DS_TILE_BYTES + half * (64 * 128), &tm.m[src][1][1], half * 64, y, bar);
    }
  }
}

// Rows of a tile that are attended: row r is a key iff r < rows and
// (r + off) mod cap < len.  Selected and sink tiles use the first rows; a
// ring tile starting at slot b attends the slots of the window
// [ring_start, ring_start + ring_len) mod ring_cap.
struct DsMask {
  int rows, off, cap, len;
};
__device__ __forceinline__ DsMask ds_mask_rows(int rows) { return DsMask{rows, 0, 1 << 30, 1 << 30}; }
__device__ __forceinline__ DsMask ds_early_mask(const AttendParams& p, int e, int ring_start) {
  if (p.sink_len > 0) {
    if (e == 0) return ds_mask_rows(p.sink_len);
    --e;
  }
  const int b = e * 64;
  int off = b - ring_start;
  if (off < 0) off += p.ring_cap;
  return DsMask{min(64, p.ring_cap - b), off, p.ring_cap, p.ring_len};
}
__device__ __forceinline__ bool ds_key(const DsMask& m, int r) {
  int u = r + m.off;
  if (u >= m.cap) u -= m.cap;  // r < cap and off < cap
  return r < m.rows && u < m.len;
}

// The G query rows as bf16 pairs in shared memory, row stride DS_QW words
// (lanes of a row quad and the 4 rows hit 16 distinct banks); read per chunk
// instead of held in registers.
constexpr int DS_QW = 68;
__device__ __forceinline__ uint32_t ds_q(const uint32_t* sq, int g, int word) {
  return g < 4 ? sq[g * DS_QW + word] : 0u;
}

// Transpose of an 8 x 8 b16 matrix held in mma fragment layout (lane l: row
// l / 4, columns 2 (l % 4), + 1).
__device__ __forceinline__ uint32_t movm_t(uint32_t a) {
  uint32_t d;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
  return d;
}

// One warp's 16-key chunk at tile rows [r0, r0 + 16), all in the transposed
// orientation, whose N = 8 columns are the query rows (4 real, G = 4):
//   S^T = K Q^T   (A = 16 key rows by ldmatrix, B = Q^T from shared memory;
//                  8 mma for 16 keys x 128 dims),
//   O^T += V^T P^T (A = V^T by ldmatrix.trans, B = P^T: the S^T accumulator
//                  as bf16, transposed in registers by movmatrix).
// Lane (g, t) = (lane / 4, lane % 4) holds S^T[key g | g + 8][query 2t | 2t + 1]
// and the online softmax state (m, l) of queries 2t and 2t + 1 (real for
// t < 2); ofr is O^T in mma layout: ofr[mt] = O[query 2t | 2t + 1][dim 16 mt +
// g (+ 8)].  P enters P.V split into a bf16 head and a bf16 remainder (two
// products), so that it carries ~16 significant bits, as an fp32 P.V does.
__device__ __forceinline__ void ds_chunk(const unsigned char* kt, unsigned char* vt, int r0, const DsMask& mk,
                                         const uint32_t* sq, float scale, float (&m_run)[2], float (&l_run)[2],
                                         float (&ofr)[8][4], int lane) {
  const int mrow = lane & 7, msel = lane >> 3, g = lane >> 2, t = lane & 3;
  // rows of the chunk that are not keys: their V rows are zeroed, so that
  // whatever the tile holds there (a slot outside the window, a slot being
  // rewritten in this call) contributes exactly nothing (p = 0 times a
  // finite value)
  const unsigned dead = __ballot_sync(FULL, !ds_key(mk, r0 + (lane & 15))) & 0xffffu;
  // S^T, k-steps of 16 dims alternating between two accumulators
  float c[2][4];
#pragma unroll
  for (int e = 0; e < 4; ++e) c[0][e] = c[1][e] = 0.f;
  const int krow = r0 + (msel & 1) * 8 + mrow;
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    uint32_t a[4];
    ldsm_x4(a, kt + swz(64, krow, ks * 16 + (msel >> 1) * 8));
    mma_bf16(c[ks & 1], a[0], a[1], a[2], a[3], ds_q(sq, g, ks * 8 + t), ds_q(sq, g, ks * 8 + 4 + t));
  }
  const bool dlo = (dead >> g) & 1u, dhi = (dead >> (g + 8)) & 1u;
  float v[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) v[e] = (e < 2 ? dlo : dhi) ? -INFINITY : (c[0][e] + c[1][e]) * scale;
  // per query: max over the 16 keys (the 8 lanes of a column)
  float mq[2] = {fmaxf(v[0], v[2]), fmaxf(v[1], v[3])};
#pragma unroll
  for (int x = 4; x < 32; x <<= 1) {
    mq[0] = fmaxf(mq[0], __shfl_xor_sync(FULL, mq[0], x));
    mq[1] = fmaxf(mq[1], __shfl_xor_sync(FULL, mq[1], x));
  }
  const float mn[2] = {fmaxf(m_run[0], mq[0]), fmaxf(m_run[1], mq[1])};
  // nothing visible yet: the mask does not depend on the query, so this holds
  // for every lane or none (the mma below are warp-collective)
  if (__all_sync(FULL, mn[0] == -INFINITY && mn[1] == -INFINITY)) return;
  float al[2], pe[4], ls[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) al[i] = m_run[i] == -INFINITY ? 0.f : __expf(m_run[i] - mn[i]);
#pragma unroll
  for (int e = 0; e < 4; ++e) pe[e] = v[e] == -INFINITY ? 0.f : __expf(v[e] - mn[e & 1]);
  ls[0] = pe[0] + pe[2];
  ls[1] = pe[1] + pe[3];
#pragma unroll
  for (int x = 4; x < 32; x <<= 1) {
    ls[0] += __shfl_xor_sync(FULL, ls[0], x);
    ls[1] += __shfl_xor_sync(FULL, ls[1], x);
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    l_run[i] = l_run[i] * al[i] + ls[i];
    m_run[i] = mn[i];
  }
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) {
    ofr[mt][0] *= al[0];
    ofr[mt][1] *= al[1];
    ofr[mt][2] *= al[0];
    ofr[mt][3] *= al[1];
  }
  // P^T fragments: [key g | g + 8][queries 2t, 2t + 1] packed, then transposed
  // to [query g][keys 2t, 2t + 1 (+ 8)] = the B operand of O^T += V^T P^T
  const uint32_t h0 = pack_bf16x2(pe[0], pe[1]), h1 = pack_bf16x2(pe[2], pe[3]);
  const uint32_t l0 = pack_bf16x2(pe[0] - bf_lo(h0), pe[1] - __uint_as_float(h0 & 0xffff0000u));
  const uint32_t l1 = pack_bf16x2(pe[2] - bf_lo(h1), pe[3] - __uint_as_float(h1 & 0xffff0000u));
  const uint32_t ph0 = movm_t(h0), ph1 = movm_t(h1), pl0 = movm_t(l0), pl1 = movm_t(l1);
  if (dead) {  // warp-uniform
#pragma unroll
    for (int rr = lane >> 4; rr < 16; rr += 2)
      if ((dead >> rr) & 1u) *reinterpret_cast<uint4*>(vt + swz(64, r0 + rr, (lane & 15) * 8)) = make_uint4(0u, 0u, 0u, 0u);
    __syncwarp();
  }
  // O^T += V^T P^T: A = V^T (16 dims x 16 keys) by ldmatrix.trans of the key
  // rows (matrix q: keys r0 + (q >> 1) * 8 + row, dims 16 mt + (q & 1) * 8)
  const int vrow = r0 + (msel >> 1) * 8 + mrow;
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) {
    uint32_t a[4];
    ldsm_x4_t(a, vt + swz(64, vrow, mt * 16 + (msel & 1) * 8));
    mma_bf16(ofr[mt], a[0], a[1], a[2], a[3], ph0, ph1);
    mma_bf16(ofr[mt], a[0], a[1], a[2], a[3], pl0, pl1);
  }
}

template <int CL, bool FUSED>
__global__ void __launch_bounds__(DS_WARPS * 32, 2) decode_split_kernel(const AttendParams p,
                                                                     const __grid_constant__ DecodeMaps tm) {
  constexpr int G = 4, NW = DS_WARPS, NT = NW * 32;
  constexpr int MT = DS<CL>::MAX_TILES;
  extern __shared__ __align__(16) unsigned char sm_raw[];
  __shared__ __align__(8) uint64_t bar[MT];
  __shared__ u64 s_sel[32];
  __shared__ u64 s_cand[FS_CAND_MAX];
  __shared__ unsigned s_misc[2 * NW];
  __shared__ int s_head;
  __shared__ __align__(8) uint64_t merge_bar;  // the other CTAs' partials for this CTA's dims have landed
  __shared__ __align__(16) uint32_t s_q[G * DS_QW];  // this head's G query rows (bf16 pairs)
  __shared__ unsigned s_part[FUSED ? NW : 1][FS_BPC_MAX];  // fused scoring: per-warp block maxima
  __shared__ unsigned char s_pflag[FUSED ? FS_BPC_MAX : 1];   // fused scoring: protected flags of this CTA's blocks
  const int split = blockIdx.x, h = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  unsigned char* sm = sm_raw + ((1024u - (smem_u32(sm_raw) & 1023u)) & 1023u);
  unsigned char* tiles = sm;  // [MT][K | V]
  // every CTA of the cluster merges SW output dims: it receives each CTA's
  // partial for them, o [CL][G][SW], and (m, l) [CL][G][2]
  constexpr int SW = DS<CL>::SW;
  float* recv = reinterpret_cast<float*>(sm + (size_t)MT * 2 * DS_TILE_BYTES);
  float* recv_ml = recv + CL * G * SW;

  // fused scoring (FUSED): this launch's key tag, and an L2 prefetch of the
  // representatives this CTA scores (a prefetch reads nothing into the SM, so
  // it may run before the wait below; every load waits)
  uint32_t fs_tg = 0u;
  if constexpr (FUSED) {
    fs_tg = fs_tag(ld_relaxed_u32(p.fs_sync));
    for (int i = tid; i < NW * FS_BPC_MAX; i += NT) (&s_part[0][0])[i] = 0u;
    if (tid < FS_BPC_MAX) s_pflag[tid] = 0;
    const int b0 = (h * CL + split) * p.fs_bpc, nb = min(p.fs_bpc, p.rank_n - b0);
    if (tid < p.hkv && nb > 0)
      prefetch_l2_bulk(p.fs_reps + ((long long)tid * p.fs_reps_blocks + b0) * p.fs_r * NKV_D,
                       (uint32_t)(nb * p.fs_r * NKV_D * 2));
  }
  // barriers, then the early tiles' loads, before anything else: they do
  // not depend on the scores, on q or on the ring head
  const int n_early = ds_early_count(p);
  int n_my_early = 0;
  for (int e = split; e < n_early && n_my_early < DS<CL>::MAX_EARLY; e += CL) ++n_my_early;
  int n_my_sel = 0;
  for (int r = split; r < p.n_sel && n_my_sel < DS<CL>::MAX_SEL; r += CL) ++n_my_sel;
  const int ntiles = n_my_early + n_my_sel;
  if (tid < MT) mbar_init(&bar[tid], 1);
  if (tid == MT) {
    mbar_init(&merge_bar, 1);
    mbar_expect_tx(&merge_bar, (CL - 1) * DS<CL>::PUSH_BYTES);  // the one arrival; the rest are st.async bytes
  }
  if (tid <= MT) fence_mbar_init();
  // early tile i: thread i (which initialised its barrier) issues its four boxes
  auto issue_early = [&]() {
    if (tid < n_my_early) {
      int src, y;
      ds_early_tile(p, h, split + tid * CL, &src, &y);
      ds_issue_tile(tm, p.tma_mask, src, y, tiles + (size_t)tid * 2 * DS_TILE_BYTES, &bar[tid]);
    }
  };
  // With fused scoring the preceding kernel may produce q, the current token,
  // the representatives or the sink / ring: everything waits for it.
  // Otherwise the preceding kernel is the scoring grid, which itself waited
  // for its predecessor before releasing this grid: only the scores wait.
  if (!FUSED) issue_early();
  // every CTA's merge barrier is initialised before any CTA of the cluster
  // stores into it: each CTA arrives here and waits before its pushes (the
  // init fence above orders the inits; a relaxed arrival does not wait for
  // this thread's loads in flight)
  cluster_arrive_relaxed();
  // the descriptors of the maps used later, by threads off the early path
  if (tid >= NT - 6) {
    const int src = (tid - (NT - 6)) >> 1;
    prefetch_tmap((p.tma_mask >> (3 + src)) & 1 ? &tm.t3[src][tid & 1] : &tm.m[src][tid & 1][1]);
  }
  pdl_launch_dependents();
  if (FUSED) pdl_wait();
  // device-resident ring head (graph replay)
  int head_v = 0;
  if (p.ring_dyn && tid == 0) head_v = ld_relaxed_s32(p.ring_dyn);
  // Q into shared memory: one 32-bit word (two dims of one row) per thread
  const int qg = lane >> 2, qt = lane & 3;
  static_assert(G * (NKV_D / 2) == NT, "one Q word per thread");
  s_q[(tid >> 6) * DS_QW + (tid & 63)] =
      __ldg(reinterpret_cast<const uint32_t*>(p.q + (long long)(h * G + (tid >> 6)) * p.q_head) + (tid & 63));
  if constexpr (FUSED) {
    issue_early();
    __syncthreads();  // the flags were cleared before the wait
    const int b0 = (h * CL + split) * p.fs_bpc;
    for (int i = tid; i < p.fs_nprot; i += NT) {
      const int b = __ldg(p.fs_prot + i) - b0;
      if (b >= 0 && b < p.fs_bpc) s_pflag[b] = 1;
    }
  }
  if (p.ring_dyn && tid == 0) s_head = head_v;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};  // queries 2t, 2t + 1
  float ofr[8][4];
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) ofr[mt][0] = ofr[mt][1] = ofr[mt][2] = ofr[mt][3] = 0.f;
  __syncthreads();  // barrier init and the ring head visible
  // The recent window: explicit, or from the device-resident head.  With a
  // device head every CTA arrives once it has read it; the last to arrive
  // advances it at its end.  The arrival is issued here and its result used
  // only at the end, so its round trip overlaps the CTA's work.  (An arrival
  // comes after the CTA's read of the head has returned its value, so the
  // advance cannot reach a read.)
  int ring_start = p.ring_start, ring_wpos = p.ring_write_pos;
  unsigned ring_ticket = 0u;
  if (p.ring_dyn) {
    ring_wpos = s_head;
    ring_start = s_head + p.ring_cap - p.ring_len;
    if (ring_start >= p.ring_cap) ring_start -= p.ring_cap;
    if (tid == 0) ring_ticket = atomicAdd(reinterpret_cast<unsigned*>(p.ring_dyn) + 1, 1u);
  }
  // fused scoring: this CTA's blocks are scored and published first, so that
  // the other CTAs' keys arrive while the early tiles are attended
  if constexpr (FUSED) fs_score_publish<G, NW>(p, h * CL + split, fs_tg, s_part, nullptr, s_pflag);
  // early tiles: warps 4t .. 4t + 3 take the four chunks of tile t
  for (int t = 0; t < n_my_early; ++t) {
    if ((warp >> 2) != (t & 1)) continue;
    mbar_wait_poll(&bar[t], 0, p.err);
    unsigned char* kt = tiles + (size_t)t * 2 * DS_TILE_BYTES;
    ds_chunk(kt, kt + DS_TILE_BYTES, (warp & 3) * 16, ds_early_mask(p, split + t * CL, ring_start), s_q, p.scale,
             m_run, l_run, ofr, lane);
  }

  // ---- selection: every CTA ranks the block scores itself -----------------------------
  if constexpr (FUSED) {
    // the top n_sel of every CTA's keys, once they all carry this launch's tag
    fs_select<NW>(p, fs_tg, s_sel, s_cand, s_misc, nullptr);
    if (tid == 0) fs_arrive(p);
  } else {
    pdl_wait();  // the scoring grid's scores are complete past this point
    rank_topk<NW>(p.rank_scores, p.rank_n, p.n_sel, s_sel, s_cand, s_misc, nullptr);
  }
  if (split == 0 && h == 0 && tid < p.n_sel) {
    p.rank_out[tid] = (long long)key_id(s_sel[tid]);
    if (p.rank_out_scores) p.rank_out_scores[tid] = key_score(s_sel[tid]);
  }
  if (tid < n_my_sel) {
    const int slot = n_my_early + tid;
    long long id = (long long)key_id(s_sel[split + tid * CL]);
    if (id < 0 || id >= p.max_blocks) {  // only after a bad score array
      if (p.err) atomicExch(p.err, ERR_BAD_INDEX);
      id = 0;
    }
    ds_issue_tile(tm, p.tma_mask, 0, (int)((id * p.hkv + h) * 64), tiles + (size_t)slot * 2 * DS_TILE_BYTES,
                  &bar[slot]);
  }
  // selected tiles: tile n_my_early + j goes to warps 4 * ((n_my_early + j) & 1) ...
  for (int t = n_my_early; t < ntiles; ++t) {
    if ((warp >> 2) != (t & 1)) continue;
    mbar_wait_poll(&bar[t], 0, p.err);
    unsigned char* kt = tiles + (size_t)t * 2 * DS_TILE_BYTES;
    ds_chunk(kt, kt + DS_TILE_BYTES, (warp & 3) * 16, ds_mask_rows(64), s_q, p.scale, m_run, l_run, ofr, lane);
  }
  // the current token: one key, attended by warp NW - 1 of the head's last CTA
  const bool cur_owner = split == CL - 1 && p.n_cur > 0;
  if (cur_owner && warp == NW - 1) {
    const __nv_bfloat16* kc = p.cur_k + (long long)h * p.cur_head;
    const __nv_bfloat16* vc = p.cur_v + (long long)h * p.cur_head;
    // s = q_g . k (lane qt of row quad g takes dims 16 kk + 2 qt + {0, 1}
    // and 16 kk + 8 + 2 qt + {0, 1} for every k-step kk)
    float part = 0.f;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const uint32_t k0 = __ldg(reinterpret_cast<const uint32_t*>(kc + kk * 16 + 2 * qt));
      const uint32_t k1 = __ldg(reinterpret_cast<const uint32_t*>(kc + kk * 16 + 8 + 2 * qt));
      const uint32_t q0 = ds_q(s_q, qg, kk * 8 + qt), q1 = ds_q(s_q, qg, kk * 8 + 4 + qt);
      part = fmaf(bf_lo(q0), bf_lo(k0), part);
      part = fmaf(__uint_as_float(q0 & 0xffff0000u), __uint_as_float(k0 & 0xffff0000u), part);
      part = fmaf(bf_lo(q1), bf_lo(k1), part);
      part = fmaf(__uint_as_float(q1 & 0xffff0000u), __uint_as_float(k1 & 0xffff0000u), part);
    }
    part += __shfl_xor_sync(FULL, part, 1);
    part += __shfl_xor_sync(FULL, part, 2);
    // this lane's queries 2 qt, 2 qt + 1 (their sums sit in row quads 2 qt, 2 qt + 1)
    const float sc[2] = {__shfl_sync(FULL, part, (2 * qt) * 4) * p.scale,
                         __shfl_sync(FULL, part, (2 * qt + 1) * 4) * p.scale};
    float al[2], pe[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const float m_new = fmaxf(m_run[i], sc[i]);
      al[i] = m_run[i] == -INFINITY ? 0.f : __expf(m_run[i] - m_new);
      pe[i] = __expf(sc[i] - m_new);
      l_run[i] = l_run[i] * al[i] + pe[i];
      m_run[i] = m_new;
    }
    // lane (g, qt) holds O[2 qt | 2 qt + 1][16 mt + g (+ 8)]
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
      const float v0 = __bfloat162float(vc[mt * 16 + qg]), v1 = __bfloat162float(vc[mt * 16 + qg + 8]);
      ofr[mt][0] = fmaf(pe[0], v0, ofr[mt][0] * al[0]);
      ofr[mt][1] = fmaf(pe[1], v0, ofr[mt][1] * al[1]);
      ofr[mt][2] = fmaf(pe[0], v1, ofr[mt][2] * al[0]);
      ofr[mt][3] = fmaf(pe[1], v1, ofr[mt][3] * al[1]);
    }
  }

  // ---- warp states -> CTA partial -> cluster merge -----------------------------------
  __syncthreads();  // every warp is done with the tiles
  float* wpo = reinterpret_cast<float*>(tiles);  // [NW][G][D]
  float* wml = wpo + NW * G * NKV_D;              // [NW][G][2]
  if (qt < 2) {  // query rows 2 qt, 2 qt + 1
    float* o0 = wpo + (warp * G + 2 * qt) * NKV_D;
    float* o1 = o0 + NKV_D;
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
      o0[mt * 16 + qg] = ofr[mt][0];
      o1[mt * 16 + qg] = ofr[mt][1];
      o0[mt * 16 + qg + 8] = ofr[mt][2];
      o1[mt * 16 + qg + 8] = ofr[mt][3];
    }
  }
  if (qg == 0 && qt < 2) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      wml[(warp * G + 2 * qt + i) * 2] = m_run[i];
      wml[(warp * G + 2 * qt + i) * 2 + 1] = l_run[i];
    }
  }
  __syncthreads();
  cluster_wait_acquire();
  {
    // (row g, 4 dims d4) per lane pair: lane hs of the pair sums warps
    // 4 hs .. 4 hs + 3, one shuffle adds the halves
    static_assert(G * (NKV_D / 4) * 2 == NT, "one lane pair per 4 output dims");
    const int it = tid >> 1, hs = tid & 1;
    const int g = it / (NKV_D / 4), d4 = it % (NKV_D / 4);
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < NW; ++w) M = fmaxf(M, wml[(w * G + g) * 2]);
    float L = 0.f;
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int w4 = 0; w4 < NW / 2; ++w4) {
      const int w = hs * (NW / 2) + w4;
      const float m = wml[(w * G + g) * 2];
      if (m == -INFINITY) continue;
      const float sw = __expf(m - M);
      L = fmaf(sw, wml[(w * G + g) * 2 + 1], L);
      const float4 v = *reinterpret_cast<const float4*>(wpo + (w * G + g) * NKV_D + d4 * 4);
      o.x = fmaf(sw, v.x, o.x);
      o.y = fmaf(sw, v.y, o.y);
      o.z = fmaf(sw, v.z, o.z);
      o.w = fmaf(sw, v.w, o.w);
    }
    L += __shfl_xor_sync(FULL, L, 1);
    o.x += __shfl_xor_sync(FULL, o.x, 1);
    o.y += __shfl_xor_sync(FULL, o.y, 1);
    o.z += __shfl_xor_sync(FULL, o.z, 1);
    o.w += __shfl_xor_sync(FULL, o.w, 1);
    // the CTA partial goes to the CTAs that merge its dims: to this CTA by a
    // plain store, to the others by asynchronous remote stores that complete
    // their merge barriers; (m, l) goes to every CTA of the cluster
    if (hs == 0) {
      const int r = (d4 * 4) / SW;
      float* dst_o = recv + ((size_t)split * G + g) * SW + (d4 * 4) % SW;
      if (r == split) *reinterpret_cast<float4*>(dst_o) = o;
      else st_async_v4(cluster_addr(dst_o, r), o, cluster_addr(&merge_bar, r));
    } else if (d4 < CL) {  // (m, l) of row g to CTA d4 (one remote store per lane)
      float* dst_ml = recv_ml + ((size_t)split * G + g) * 2;
      if (d4 == split) {
        dst_ml[0] = M;
        dst_ml[1] = L;
      } else {
        st_async_v2(cluster_addr(dst_ml, d4), M, L, cluster_addr(&merge_bar, d4));
      }
    }
  }
  // the decode token goes into the ring slot no CTA reads in this call
  if (cur_owner && ring_wpos >= 0 && tid >= NT - 32) {
    const int i = tid - (NT - 32);  // 16-byte chunks: 16 of K, 16 of V
    const __nv_bfloat16* src = (i < 16 ? p.cur_k : p.cur_v) + (long long)h * p.cur_head + (i & 15) * 8;
    __nv_bfloat16* dst = (i < 16 ? p.ring_k : p.ring_v) + ((long long)h * p.ring_cap + ring_wpos) * NKV_D + (i & 15) * 8;
    *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
  }
  // this CTA's dims: wait for every CTA's partial, merge, write the output
  __syncthreads();  // this CTA's own stores into the receive area
  mbar_wait_poll(&merge_bar, 0, p.err);
  {
    // LPO adjacent lanes per output, each taking SPL of the CL partials, then
    // a shuffle tree (short dependency chains instead of CL serial steps)
    constexpr int NOUT = G * SW, LPO = NT / NOUT, SPL = CL / LPO;
    static_assert(NOUT * LPO == NT && SPL * LPO == CL && 32 % LPO == 0, "merge lanes");
    const int oi = tid / LPO, j = tid % LPO;
    const int g = oi / SW, d = oi % SW;
    float mv[SPL];
    float M = -INFINITY;
#pragma unroll
    for (int c = 0; c < SPL; ++c) {
      mv[c] = recv_ml[((j * SPL + c) * G + g) * 2];
      M = fmaxf(M, mv[c]);
    }
#pragma unroll
    for (int x = 1; x < LPO; x <<= 1) M = fmaxf(M, __shfl_xor_sync(FULL, M, x));
    float L = 0.f, o = 0.f;
#pragma unroll
    for (int c = 0; c < SPL; ++c) {
      if (mv[c] == -INFINITY) continue;
      const int sc = j * SPL + c;
      const float sw = __expf(mv[c] - M);
      L = fmaf(sw, recv_ml[(sc * G + g) * 2 + 1], L);
      o = fmaf(sw, recv[(sc * G + g) * SW + d], o);
    }
#pragma unroll
    for (int x = 1; x < LPO; x <<= 1) {
      L += __shfl_xor_sync(FULL, L, x);
      o += __shfl_xor_sync(FULL, o, x);
    }
    if (j == 0) p.out[(long long)(h * G + g) * p.out_head + split * SW + d] = __float2bfloat16(o / L);
  }
  // device-resident ring head: the last CTA of the grid to arrive (every CTA
  // had read the head before its arrival) advances it past the slot written above
  if (p.ring_dyn && tid == 0 && ring_ticket == gridDim.x * gridDim.y - 1u) {
    p.ring_dyn[1] = 0;
    int nh = s_head + 1;
    if (nh >= p.ring_cap) nh = 0;
    p.ring_dyn[0] = nh;
  }
}

// Log-sum-exp merge of the splits of head h, run by the head's last CTA.
// wbuf (shared, >= 2 * nr * splits floats) first receives every split's (m, l)
// in one parallel load, then the per-(row, split) weights exp(m - M) / L; the
// outputs are weighted sums of float4 partial rows, with the splits divided
// between two threads per output when there are few rows.
template <int G>
__device__ void combine_splits(const AttendParams& p, int h, float* wbuf, uint32_t xp_ep) {
  const int tid = threadIdx.x;
  const int nr = p.nr, S = p.splits;
  float* wm = wbuf;            // [nr][S]
  float* wl = wbuf + nr * S;   // [nr][S]
  const float* ml = p.part_ml + (long long)h * S * nr * 2;
  for (int i = tid; i < nr * S; i += blockDim.x) {
    const int row = i / S, sp = i % S;
    const float2 v = __ldcg(reinterpret_cast<const float2*>(ml + ((long long)sp * nr + row) * 2));
    wm[i] = v.x;
    wl[i] = v.y;
  }
  __syncthreads();
  for (int row = tid >> 5; row < nr; row += (int)(blockDim.x >> 5)) {
    const int lane = tid & 31;
    float M = -INFINITY;
    for (int sp = lane; sp < S; sp += 32) M = fmaxf(M, wm[row * S + sp]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(FULL, M, o));
    float L = 0.f;
    for (int sp = lane; sp < S; sp += 32) {
      const float m = wm[row * S + sp];
      L += (m == -INFINITY) ? 0.f : wl[row * S + sp] * __expf(m - M);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(FULL, L, o);
    __syncwarp();
    for (int sp = lane; sp < S; sp += 32) {
      const float m = wm[row * S + sp];
      wm[row * S + sp] = (m == -INFINITY) ? 0.f : __expf(m - M) / L;
    }
  }
  __syncthreads();
  const int items = nr * (NKV_D / 4);          // (row, 4-dim group)
  const int tpi = items >= (int)blockDim.x ? 1 : 2;  // threads per item
  const float* po = p.part_o + (long long)h * S * nr * NKV_D;
  for (int base = 0; base < items * tpi; base += blockDim.x) {
    const int idx = base + tid;
    const int item = idx / tpi, half = idx % tpi;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if (item < items) {
      const int row = item / (NKV_D / 4), d4 = item % (NKV_D / 4);
#pragma unroll 4
      for (int sp = half; sp < S; sp += tpi) {
        const float w = wm[row * S + sp];
        const float4 v = __ldcg(reinterpret_cast<const float4*>(po + ((long long)sp * nr + row) * NKV_D) + d4);
        acc.x = fmaf(w, v.x, acc.x);
        acc.y = fmaf(w, v.y, acc.y);
        acc.z = fmaf(w, v.z, acc.z);
        acc.w = fmaf(w, v.w, acc.w);
      }
    }
    if (tpi == 2) {
      acc.x += __shfl_xor_sync(FULL, acc.x, 1);
      acc.y += __shfl_xor_sync(FULL, acc.y, 1);
      acc.z += __shfl_xor_sync(FULL, acc.z, 1);
      acc.w += __shfl_xor_sync(FULL, acc.w, 1);
    }
    if (item < items && half == 0) {
      const int row = item / (NKV_D / 4), d4 = item % (NKV_D / 4);
      const int qn = row / G, g = row % G;
      const long long oo = qn * p.out_row + (long long)(h * G + g) * p.out_head + d4 * 4;
      if (NKV_INB(p.err, 43, oo, 4, p.ext_out)) {
        uint2 w;
        w.x = (uint32_t)f2bf(acc.x) | ((uint32_t)f2bf(acc.y) << 16);
        w.y = (uint32_t)f2bf(acc.z) | ((uint32_t)f2bf(acc.w) << 16);
        *reinterpret_cast<uint2*>(p.out + oo) = w;
        if (p.xp_P) {  // peer exchange: the four dims to every other rank
          const long long wi = ((long long)(p.xp_rank * gridDim.y + h) * G + g) * (NKV_D / 2) + d4 * 2;
          peer_push(p, xp_ep, wi, w.x);
          peer_push(p, xp_ep, wi + 1, w.y);
        }
      }
    }
  }
}

// Launch shape of the most recent nkv_attend call on this thread.
static thread_local int g_last_cluster = -1, g_last_splits = 0, g_last_tps = 0;

static int env_int(const char* name, int dflt) { return knob(name, dflt); }

static int splits_for(int ntok, int hkv, int sms) {
  int s_mem = (ntok + AT_TPS_MAX - 1) / AT_TPS_MAX;
  int s_par = sms / hkv;
  int s_cap = (ntok + AT_MIN_TPS - 1) / AT_MIN_TPS;
  int s = s_par < s_cap ? s_par : s_cap;
  if (s < s_mem) s = s_mem;
  if (s < 1) s = 1;
  return s;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// dependency on libcuda).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
static EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = []() -> EncodeTiledFn {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      f = nullptr;
    cudaGetLastError();
    return reinterpret_cast<EncodeTiledFn>(f);
  }();
  return fn;
}

// Tensor map over `rows` rows of 128 bf16 at `base` (boxes of `box_rows` x 64
// columns, 128-byte swizzle, zero fill outside), or false when TMA must not
// read it: memory that is not device memory (mapped host memory, managed
// memory), a base that is not 16-byte aligned, or more rows than a coordinate
// holds.  Maps are cached per thread in a small hash table keyed by
// (base, rows, box_rows); encoding touches no device state.
// box_rows = -64: the whole-tile 3D form of DecodeMaps::t3.
static bool tma_rows_map(CUtensorMap* out, const void* base, long long rows, int box_rows) {
  struct Entry { const void* base; long long rows; int box; bool ok; CUtensorMap map; };
  constexpr int N = 512;
  static thread_local Entry* cache = nullptr;
  if (!base || rows < 1 || rows >= (1ll << 31) || ((uintptr_t)base & 15)) return false;
  if (!cache) cache = static_cast<Entry*>(calloc(N, sizeof(Entry)));
  if (!cache) return false;
  uint64_t key = (uint64_t)(uintptr_t)base ^ ((uint64_t)rows * 0x9e3779b97f4a7c15ull) ^ (uint64_t)box_rows;
  key ^= key >> 29;
  Entry& e = cache[(key * 0xbf58476d1ce4e5b9ull) >> 55];  // 9 bits: N = 512
  if (e.base == base && e.rows == rows && e.box == box_rows) {
    if (e.ok) *out = e.map;
    return e.ok;
  }
  e.base = base;
  e.rows = rows;
  e.box = box_rows;
  e.ok = false;
  cudaPointerAttributes pa;
  const bool dev = cudaPointerGetAttributes(&pa, base) == cudaSuccess && pa.type == cudaMemoryTypeDevice;
  cudaGetLastError();
  EncodeTiledFn fn = encode_tiled();
  if (dev && fn && box_rows < 0 && -box_rows <= rows) {
    const cuuint64_t dims[3] = {64, (cuuint64_t)rows, 2};
    const cuuint64_t strides[2] = {(cuuint64_t)NKV_D * 2, 128};
    const cuuint32_t box[3] = {64, (cuuint32_t)(-box_rows), 2};
    const cuuint32_t es[3] = {1, 1, 1};
    e.ok = fn(&e.map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
  } else if (dev && fn && box_rows > 0 && box_rows <= rows) {
    const cuuint64_t dims[2] = {(cuuint64_t)NKV_D, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)NKV_D * 2};
    const cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
    const cuuint32_t es[2] = {1, 1};
    e.ok = fn(&e.map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
  }
  if (e.ok) *out = e.map;
  return e.ok;
}

// The four maps of one source (K and V, 8- and 64-row boxes); a source of
// fewer than 64 rows never has a piece of 64 rows and gets no 64-row maps.
// *tile3: the source also has whole-tile maps (t3).
static bool source_maps(DecodeMaps* m, int src, const void* k, const void* v, long long rows, bool* tile3) {
  *tile3 = false;
  if (!tma_rows_map(&m->m[src][0][0], k, rows, 8) || !tma_rows_map(&m->m[src][1][0], v, rows, 8)) return false;
  if (rows < 64) return true;
  if (!tma_rows_map(&m->m[src][0][1], k, rows, 64) || !tma_rows_map(&m->m[src][1][1], v, rows, 64)) return false;
  *tile3 = env_int("NKV_TMA_TILE3", 1) && tma_rows_map(&m->t3[src][0], k, rows, -64) &&
           tma_rows_map(&m->t3[src][1], v, rows, -64);
  return true;
}

// The decode kernel's tensor maps for one combination of sources (block
// store, sink, recent ring; a null pointer = source absent), with the mask of
// the sources TMA may read.  Cached per thread, least recently used out of 64
// combinations: a layer's buffers stay put, so a decode step finds its maps
// with one lookup instead of twelve.
static const DecodeMaps& decode_maps(const void* ks, const void* vs, long long krows, const void* sk, const void* sv,
                                     long long srows, const void* rk, const void* rv, long long rrows, int* mask) {
  struct Entry { const void* ptr[6]; long long rows[3]; int mask; unsigned long long stamp; DecodeMaps maps; };
  constexpr int N = 64;
  static thread_local Entry* cache = nullptr;
  static thread_local unsigned long long clock = 0;
  static thread_local DecodeMaps scratch;
  const void* ptr[6] = {ks, vs, sk, sv, rk, rv};
  const long long rows[3] = {ks ? krows : 0, sk ? srows : 0, rk ? rrows : 0};
  if (!cache) cache = static_cast<Entry*>(calloc(N, sizeof(Entry)));
  Entry* victim = nullptr;
  if (cache) {
    for (int i = 0; i < N; ++i) {
      Entry& e = cache[i];
      if (e.stamp && e.ptr[0] == ptr[0] && e.ptr[1] == ptr[1] && e.ptr[2] == ptr[2] && e.ptr[3] == ptr[3] &&
          e.ptr[4] == ptr[4] && e.ptr[5] == ptr[5] && e.rows[0] == rows[0] && e.rows[1] == rows[1] &&
          e.rows[2] == rows[2]) {
        e.stamp = ++clock;
        *mask = e.mask;
        return e.maps;
      }
      if (!victim || e.stamp < victim->stamp) victim = &e;
    }
  }
  DecodeMaps& m = victim ? victim->maps : scratch;
  memset(&m, 0, sizeof(m));
  // bit s: source s is TMA-readable; bit 3 + s: it also has whole-tile maps
  int mk = 0;
  bool t3 = false;
  if (ks && source_maps(&m, 0, ks, vs, krows, &t3)) mk |= 1 | (t3 ? 8 : 0);
  if (sk && source_maps(&m, 1, sk, sv, srows, &t3)) mk |= 2 | (t3 ? 16 : 0);
  if (rk && source_maps(&m, 2, rk, rv, rrows, &t3)) mk |= 4 | (t3 ? 32 : 0);
  if (victim) {
    for (int i = 0; i < 6; ++i) victim->ptr[i] = ptr[i];
    for (int i = 0; i < 3; ++i) victim->rows[i] = rows[i];
    victim->mask = mk;
    victim->stamp = ++clock;
  }
  *mask = mk;
  return m;
}

// cudaOccupancyMaxActiveClusters for a launch configuration, cached per
// thread by (kernel, device, cluster size, block count, shared memory): the
// query costs microseconds of host time and its answer never changes.
static bool cluster_occupancy(const void* kern, const cudaLaunchConfig_t& lc, int* nclusters) {
  struct Entry { const void* fn; int dev, cl, blocks; size_t smem; int n; };
  static thread_local Entry cache[32];
  static thread_local int used = 0, next = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  int cl = 1;
  for (unsigned i = 0; i < lc.numAttrs; ++i)
    if (lc.attrs[i].id == cudaLaunchAttributeClusterDimension) cl = (int)lc.attrs[i].val.clusterDim.x;
  const int blocks = (int)(lc.gridDim.x * lc.gridDim.y * lc.gridDim.z);
  for (int i = 0; i < used; ++i) {
    const Entry& e = cache[i];
    if (e.fn == kern && e.dev == dev && e.cl == cl && e.blocks == blocks && e.smem == lc.dynamicSmemBytes) {
      *nclusters = e.n;
      return true;
    }
  }
  int n = 0;
  const cudaError_t err = cudaOccupancyMaxActiveClusters(&n, kern, &lc);
  cudaGetLastError();
  if (err != cudaSuccess) return false;
  const int slot = used < 32 ? used++ : (next++ & 31);
  cache[slot] = Entry{kern, dev, cl, blocks, lc.dynamicSmemBytes, n};
  *nclusters = n;
  return true;
}

static size_t attend_ws(int hkv, int nr, int max_tokens) {
  const long long smax = (max_tokens + AT_MIN_TPS - 1) / AT_MIN_TPS + 1;
  size_t o = 256 + ((hkv * 4 + 255) / 256) * 256;
  o += (size_t)hkv * smax * nr * NKV_D * 4;
  o += (size_t)hkv * smax * nr * 2 * 4;
  return o + 256;
}

}  // namespace nkv

using namespace nkv;

extern "C" size_t nkv_attend_workspace_bytes(int hkv, int hq, int nq, int max_tokens) {
  if (hkv < 1) hkv = 1;
  if (nq < 1) nq = 1;
  if (max_tokens < 1) max_tokens = 1;
  return attend_ws(hkv, (hq / hkv) * nq, max_tokens);
}

struct RankArgs {
  const float* scores;  // ranked mode: block scores of a scoring grid; null: one-launch step or peer exchange
  int nblocks;
  int64_t* out_ids;
  float* out_scores;
  const PeerArgs* peer;  // KV-head sharding over peer memory (scores from the exchange)
  void* out_full;        // with peer: this rank's full-width output
  // one-launch step: the attention grid scores the blocks itself
  const void* reps;
  int r, reps_blocks;
  const int32_t* prot;
  int nprot;
  void* sel_ws;  // select workspace: epoch at +16, arrivals at +20, keys at +256
  int32_t* ring_head;  // device-resident recent-ring head [head, arrivals] (decode kernel) or null
  int split_only;      // one-launch step: the fused tile-split kernel only (FS_DECLINED otherwise)
};
static bool g_fs_unavailable = false;  // the cooperative cluster launch was refused once

static int attend_impl(nkv_stream_t stream, const nkv_attend_args* a, const RankArgs* rank);

extern "C" int nkv_attend(nkv_stream_t stream, const nkv_attend_args* a) {
  return attend_impl(stream, a, nullptr);
}

namespace nkv {
int attend_ranked(nkv_stream_t stream, const nkv_attend_args* a, const float* scores, int nblocks,
                  int64_t* out_ids, float* out_scores, const PeerArgs* peer, void* out_full, int32_t* ring_head) {
  NKV_REQUIRE(a && a->nq == 1 && (scores || peer) && out_ids, "attend_ranked: needs one query, scores and out_ids");
  if (peer) {
    NKV_REQUIRE(peer->P >= 1 && peer->P <= NKV_MAX_PEERS && peer->rank >= 0 && peer->rank < peer->P && peer->exch &&
                    nblocks <= peer->cap && peer->hq_all == a->hq * peer->P && out_full,
                "attend_ranked: bad peer exchange (P=%d, rank=%d, cap=%d, hq_all=%d)", peer->P, peer->rank, peer->cap,
                peer->hq_all);
    NKV_REQUIRE((const char*)a->out == (const char*)out_full + (size_t)peer->rank * a->hq * NKV_D * 2 &&
                    a->out_head_stride == NKV_D,
                "attend_ranked: args->out must be this rank's rows of out_full");
    for (int i = 0; i < peer->P; ++i)
      NKV_REQUIRE(peer->exch[i] && ((uintptr_t)peer->exch[i] & 15) == 0, "attend_ranked: exchange %d missing", i);
  }
  NKV_REQUIRE(a->n_sel >= 1 && a->n_sel <= 32 && a->n_sel <= nblocks, "attend_ranked: k=%d out of [1, 32]",
              a->n_sel);
  NKV_SUPPORTED(nblocks <= FS_MAXE * NKV_DECODE_WARPS * 32, "attend_ranked: %d blocks exceed the in-kernel ranking",
                nblocks);
  if (ring_head) {
    // graph replay: every replay appends one token at the device-resident head,
    // so the window length must already be at its fixed size
    NKV_REQUIRE(((uintptr_t)ring_head & 7) == 0 && a->n_cur == 1 && a->ring_cap >= 1 && a->ring_write_pos >= 0 &&
                    a->ring_len == a->ring_cap - 1 && a->ring_k && a->ring_v,
                "attend_ranked: a device ring head needs a full recent window (ring_len %d, cap %d) and one "
                "current token",
                a->ring_len, a->ring_cap);
  }
  RankArgs r{scores, nblocks, out_ids, out_scores, peer, out_full, nullptr, 0, 0, nullptr, 0, nullptr, ring_head, 0};
  return attend_impl(stream, a, &r);
}

// One-launch decode step: scoring, selection and attention in one cooperative
// cluster launch.  Returns FS_DECLINED (nothing launched) where it does not
// apply; the caller then runs the scoring grid and the ranked attention.
int attend_step(nkv_stream_t stream, const nkv_attend_args* a, const void* reps, int r, int reps_blocks,
                int nblocks, const int32_t* prot, int nprot, void* sel_ws, size_t sel_ws_bytes, int64_t* out_ids,
                float* out_scores, int32_t* ring_head, int split_only) {
  NKV_REQUIRE(a && a->nq == 1 && reps && out_ids && sel_ws, "decode step: null argument");
  NKV_REQUIRE(a->n_sel >= 1 && a->n_sel <= nblocks && nblocks <= reps_blocks, "decode step: k=%d, nblocks=%d",
              a->n_sel, nblocks);
  NKV_REQUIRE(nprot == 0 || prot, "decode step: protected ids missing");
  NKV_REQUIRE(((uintptr_t)reps & 15) == 0, "decode step: reps must be 16-byte aligned");
  NKV_REQUIRE(sel_ws_bytes >= nkv_select_workspace_bytes(reps_blocks, 1), "decode step: select workspace too small");
  if ((g_fs_unavailable && !split_only) || a->n_sel > 32 || r < 1 || r > 4 || r == 3 ||
      nblocks > FS_MAXE * NKV_DECODE_WARPS * 32)
    return FS_DECLINED;
  if (ring_head)
    NKV_REQUIRE(((uintptr_t)ring_head & 7) == 0 && a->n_cur == 1 && a->ring_cap >= 1 && a->ring_write_pos >= 0 &&
                    a->ring_len == a->ring_cap - 1 && a->ring_k && a->ring_v,
                "decode step: a device ring head needs a full recent window (ring_len %d, cap %d)", a->ring_len,
                a->ring_cap);
  RankArgs ra{nullptr, nblocks, out_ids, out_scores, nullptr, nullptr, reps, r, reps_blocks, prot, nprot, sel_ws,
              ring_head, split_only};
  return attend_impl(stream, a, &ra);
}
}  // namespace nkv

// The tile-split decode kernel for a ranked single-query step: one cluster of
// 16 CTAs per KV head where the SMs hold every head's cluster, else 8; returns
// FS_DECLINED (nothing launched) when neither shape fits the call or the
// device, so that the caller takes the general decode kernel.
template <bool FUSED>
static int launch_split(AttendParams p, const DecodeMaps& maps, const nkv_attend_args* a, cudaStream_t st) {
  const int early_max = (a->sink_len > 0 ? 1 : 0) + (a->ring_len > 0 ? (a->ring_cap + 63) / 64 : 0);
  const int cl_knob = env_int("NKV_SPLIT_CL", 16);  // 16: try 16 then 8; 8: 8 only
  for (int CL : {16, 8}) {
    if (CL > cl_knob) continue;
    const int max_early = CL >= 16 ? DS<16>::MAX_EARLY : DS<8>::MAX_EARLY;
    if (early_max > CL * max_early || a->n_sel > 32) continue;
    if (FUSED) {
      p.fs_bpc = (p.rank_n + CL * a->hkv - 1) / (CL * a->hkv);
      if (p.fs_bpc > FS_BPC_MAX) continue;
    }
    const void* kern =
        CL == 16 ? (const void*)decode_split_kernel<16, FUSED> : (const void*)decode_split_kernel<8, FUSED>;
    const size_t smem = CL == 16 ? DS<16>::SMEM : DS<8>::SMEM;
    if (ensure_smem(kern, smem, "attend split")) return NKV_ERR_CUDA;
    if (CL > 8 && ensure_nonportable_cluster(kern, "attend split")) {
      cudaGetLastError();
      continue;
    }
    cudaLaunchAttribute attr[2];
    cudaLaunchConfig_t lc = {};
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = p.overlap;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = CL;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    lc.gridDim = dim3(CL, a->hkv);
    lc.blockDim = dim3(DS_WARPS * 32);
    lc.dynamicSmemBytes = smem;
    lc.stream = st;
    lc.attrs = attr;
    lc.numAttrs = 2;
    int nclusters = 0;
    if (!cluster_occupancy(kern, lc, &nclusters) || nclusters < 1) continue;
    p.cluster = 1;
    p.splits = CL;
    p.tps = (int)((p.ntok + CL - 1) / CL);
    g_last_cluster = 2;
    g_last_splits = CL;
    g_last_tps = p.tps;
    const cudaError_t le = CL == 16 ? cudaLaunchKernelEx(&lc, decode_split_kernel<16, FUSED>, p, maps)
                                    : cudaLaunchKernelEx(&lc, decode_split_kernel<8, FUSED>, p, maps);
    if (le != cudaSuccess) return check_launch("attend split");
    return check_launch("attend split");
  }
  return FS_DECLINED;
}

static int attend_impl(nkv_stream_t stream, const nkv_attend_args* a, const RankArgs* rank) {
  NKV_REQUIRE(a, "attend: null args");
  NKV_SUPPORTED(a->head_dim == NKV_D, "attend: head_dim %d unsupported (128 only)", a->head_dim);
  NKV_REQUIRE(a->hkv >= 1 && a->hq % a->hkv == 0, "attend: hq %d not a multiple of hkv %d", a->hq,
              a->hkv);
  const int G = a->hq / a->hkv;
  NKV_SUPPORTED(G == 1 || G == 2 || G == 4 || G == 8, "attend: G=%d unsupported", G);
  NKV_SUPPORTED(a->nq >= 1 && a->nq <= 8 && a->nq * G <= 64, "attend: nq=%d unsupported", a->nq);
  NKV_REQUIRE(a->n_cur == a->nq || a->n_cur == 0, "attend: n_cur (%d) must be 0 or nq (%d)",
              a->n_cur, a->nq);
  NKV_REQUIRE(a->block_size >= 1 && a->n_sel >= 0 && a->sink_len >= 0 && a->ring_len >= 0,
              "attend: negative segment length");
  NKV_SUPPORTED((a->block_size & (a->block_size - 1)) == 0 && a->block_size >= 16 && a->block_size <= 128,
                "attend: block_size %d unsupported (16, 32, 64 or 128)", a->block_size);
  NKV_REQUIRE(a->n_sel == 0 || (a->block_ids && a->k_store && a->v_store && a->max_blocks > 0),
              "attend: selected segment needs block_ids and the block store");
  NKV_REQUIRE(a->store_kind >= 0 && a->store_kind <= 2, "attend: bad store_kind");
  NKV_REQUIRE(a->store_kind != NKV_STORE_INT8_REF || a->n_sel == 0 || (a->k_chan_scale && a->v_block_scale),
              "attend: int8 reference scheme needs its scales");
  NKV_REQUIRE(a->store_kind != NKV_STORE_INT8_TOKEN || a->n_sel == 0 || (a->k_tok_scale && a->v_tok_scale),
              "attend: int8 token scheme needs its scales");
  NKV_REQUIRE(a->sink_len <= a->sink_cap || a->sink_len == 0, "attend: sink_len > sink_cap");
  NKV_REQUIRE(a->sink_len == 0 || (a->sink_k && a->sink_v), "attend: sink missing");
  NKV_REQUIRE(a->ring_len == 0 || (a->ring_k && a->ring_v && a->ring_len <= a->ring_cap &&
                                   a->ring_start >= 0 && a->ring_start < a->ring_cap),
              "attend: bad ring slice");
  NKV_REQUIRE(a->ring_write_pos < a->ring_cap && (a->ring_write_pos < 0 || a->ring_k),
              "attend: bad ring_write_pos");
  NKV_REQUIRE(a->q && a->out && a->workspace, "attend: null pointer");
  NKV_REQUIRE(a->n_cur == 0 || (a->cur_k && a->cur_v), "attend: current tokens missing");
  NKV_REQUIRE(a->ring_write_pos < 0 || a->n_cur >= 1, "attend: ring write needs a current token");
  NKV_REQUIRE(a->allowed == nullptr || a->allowed_stride >= a->n_sel, "attend: allowed stride");
  NKV_REQUIRE(((uintptr_t)a->out & 7) == 0 && a->out_head_stride % 4 == 0 && a->out_row_stride % 4 == 0,
              "attend: out must be 8-byte aligned with strides multiple of 4 elements");
  NKV_REQUIRE(((uintptr_t)a->q & 15) == 0 && ((uintptr_t)a->cur_k & 15) == 0 &&
                  ((uintptr_t)a->cur_v & 15) == 0 && a->q_row_stride % 8 == 0 &&
                  a->q_head_stride % 8 == 0 && a->cur_row_stride % 8 == 0 &&
                  a->cur_head_stride % 8 == 0,
              "attend: q/cur must be 16-byte aligned with strides multiple of 8 elements");
  const long long ntok = (long long)a->n_sel * a->block_size + a->sink_len + a->ring_len + a->n_cur;
  NKV_REQUIRE(ntok >= 1 && ntok < (1ll << 30), "attend: key count %lld out of range", ntok);
  const int nr = a->nq * G;
  NKV_REQUIRE(a->workspace_bytes >= attend_ws(a->hkv, nr, (int)ntok),
              "attend: workspace too small (%zu < %zu)", a->workspace_bytes,
              attend_ws(a->hkv, nr, (int)ntok));

  AttendParams p;
  p.q = (const __nv_bfloat16*)a->q;
  p.q_row = a->q_row_stride;
  p.q_head = a->q_head_stride;
  p.nq = a->nq;
  p.hkv = a->hkv;
  p.B = a->block_size;
  p.log2B = 0;
  while ((1 << p.log2B) < a->block_size) ++p.log2B;
  p.scale = a->scale;
  p.ids = (const long long*)a->block_ids;
  p.n_sel = a->n_sel;
  p.max_blocks = a->max_blocks;
  p.kind = a->store_kind;
  p.k_store = a->k_store;
  p.v_store = a->v_store;
  p.kcs = a->k_chan_scale;
  p.vbs = a->v_block_scale;
  p.kts = (const __nv_bfloat16*)a->k_tok_scale;
  p.vts = (const __nv_bfloat16*)a->v_tok_scale;
  p.allowed = a->allowed;
  p.allowed_stride = a->allowed_stride;
  p.sink_k = (const __nv_bfloat16*)a->sink_k;
  p.sink_v = (const __nv_bfloat16*)a->sink_v;
  p.sink_cap = a->sink_cap;
  p.sink_len = a->sink_len;
  p.ring_k = (__nv_bfloat16*)a->ring_k;
  p.ring_v = (__nv_bfloat16*)a->ring_v;
  p.ring_cap = a->ring_cap;
  p.ring_start = a->ring_start;
  p.ring_len = a->ring_len;
  p.cur_k = (const __nv_bfloat16*)a->cur_k;
  p.cur_v = (const __nv_bfloat16*)a->cur_v;
  p.cur_row = a->cur_row_stride;
  p.cur_head = a->cur_head_stride;
  p.n_cur = a->n_cur;
  p.ring_write_pos = a->ring_write_pos;
  p.out = (__nv_bfloat16*)a->out;
  p.out_row = a->out_row_stride;
  p.out_head = a->out_head_stride;
  p.ntok = (int)ntok;
  p.nr = nr;
  p.nr_pad = (nr + 3) / 4 * 4;
  const int sms = sm_count();
  // cluster mode: one cluster of C <= 16 CTAs per head, enough heads x C to
  // cover the SMs, and every split's keys within the cluster tile limit.
  // NKV_ATTEND_CLUSTER (0 = never, N = cluster size) overrides the choice.
  const int cl_env = env_int("NKV_ATTEND_CLUSTER", -1);
  int C = 0;
  if (cl_env != 0 && (cl_env > 0 || a->hkv * AT_CLUSTER_MAX >= sms / 2 || a->hkv * 8 >= sms / 2)) {
    C = cl_env > 0 ? (cl_env > AT_CLUSTER_MAX ? AT_CLUSTER_MAX : cl_env) : AT_CLUSTER_MAX;
    while (cl_env <= 0 && C > 1 && a->hkv * C > sms + sms / 4) C >>= 1;
    if (cl_env <= 0 && a->nq == 1) {
      // single query: the fewest CTAs per head that keep <= 336 keys each
      // (the per-CTA prologue and merge dominate small CTAs)
      int c = 1;
      while (c < AT_CLUSTER_MAX && (p.ntok + c - 1) / c > 336) c <<= 1;
      if (c < C) C = c;
    }
    int tps = (p.ntok + C - 1) / C;
    if (tps < AT_MIN_TPS) {
      C = (p.ntok + AT_MIN_TPS - 1) / AT_MIN_TPS;
      tps = (p.ntok + C - 1) / C;
    }
    tps = (tps + 7) / 8 * 8;
    if (tps > AT_TPS_MAX_CLUSTER || (tps / a->block_size + 2) > AT_MAX_SLOTS) C = 0;
    else {
      p.tps = tps;
      p.splits = (p.ntok + tps - 1) / tps;
      C = p.splits;
    }
  }
  p.cluster = C > 0 ? 1 : 0;
  // NKV_ATTEND_MERGE: 0 = workspace merge, 1 = cluster merge where it fits
  if (env_int("NKV_ATTEND_MERGE", 1) == 0) p.cluster = 0;
  p.rank_scores = rank ? rank->scores : nullptr;
  p.rank_n = rank ? rank->nblocks : 0;
  p.rank_out = rank ? (long long*)rank->out_ids : nullptr;
  p.rank_out_scores = rank ? rank->out_scores : nullptr;
  p.ring_dyn = rank ? rank->ring_head : nullptr;
  p.sel_thr_every = env_int("NKV_SEL_THREADS", 0);
  const bool one_launch = rank && !rank->scores && !rank->peer;
  p.fs_reps = one_launch ? (const __nv_bfloat16*)rank->reps : nullptr;
  p.fs_r = one_launch ? rank->r : 0;
  p.fs_reps_blocks = one_launch ? rank->reps_blocks : 0;
  p.fs_prot = one_launch ? rank->prot : nullptr;
  p.fs_nprot = one_launch ? rank->nprot : 0;
  p.fs_keys = one_launch ? (unsigned long long*)((char*)rank->sel_ws + 256) : nullptr;
  p.fs_sync = one_launch ? (unsigned*)((char*)rank->sel_ws + 16) : nullptr;
  p.fs_bpc = 0;
  p.fs_prefetch = env_int("NKV_FS_PREFETCH", 1);
  p.xp_P = 0;
  p.xp_scores = nullptr;
  p.xp_sync = nullptr;
  p.xp_full = nullptr;
  p.xp_rank = p.xp_cap = p.xp_hq = 0;
  for (int i = 0; i < NKV_MAX_PEERS; ++i) p.xp_out[i] = nullptr;
  if (rank && rank->peer) {
    const PeerArgs& pa = *rank->peer;
    p.xp_P = pa.P;
    p.xp_rank = pa.rank;
    p.xp_cap = pa.cap;
    p.xp_hq = pa.hq_all;
    p.xp_scores = (const u64*)((const char*)pa.exch[pa.rank] + peer_xs_offset());
    p.xp_sync = (uint32_t*)pa.exch[pa.rank];
    p.xp_full = (__nv_bfloat16*)rank->out_full;
    for (int i = 0; i < pa.P; ++i) p.xp_out[i] = (u64*)((char*)pa.exch[i] + peer_xo_offset(pa.P, pa.cap));
  }
  AttendParams pg = p;  // workspace-merge configuration (fallback)
  pg.cluster = 0;
  {
    AttendParams& q = pg;
    q.splits = splits_for(q.ntok, a->hkv, sms);
    q.tps = (q.ntok + q.splits - 1) / q.splits;
    q.tps = (q.tps + 7) / 8 * 8;
    q.splits = (q.ntok + q.tps - 1) / q.tps;
    while (2 * nr * q.splits > q.tps * 64) {
      q.tps *= 2;
      q.splits = (q.ntok + q.tps - 1) / q.tps;
    }
  }
  if (!p.cluster) {
    p.splits = splits_for(p.ntok, a->hkv, sms);
    p.tps = (p.ntok + p.splits - 1) / p.splits;
    p.tps = (p.tps + 7) / 8 * 8;
    p.splits = (p.ntok + p.tps - 1) / p.tps;
    // the merge keeps 2 * nr * splits floats in the K tile region (tps * 64 floats)
    while (2 * nr * p.splits > p.tps * 64) {
      p.tps *= 2;
      p.splits = (p.ntok + p.tps - 1) / p.tps;
    }
    NKV_SUPPORTED(p.tps <= AT_TPS_MAX && p.tps / a->block_size + 2 <= AT_MAX_SLOTS,
                  "attend: %d keys per CTA exceed the tile limit", p.tps);
  }
  auto finish = [&](AttendParams& p) -> int {
    char* ws = (char*)a->workspace;
    p.err = (int*)ws;
    p.counters = (unsigned*)(ws + 256);
    size_t off = 256 + ((a->hkv * 4 + 255) / 256) * 256;
    p.part_o = (float*)(ws + off);
    off += (size_t)a->hkv * p.splits * nr * NKV_D * 4;
    p.part_ml = (float*)(ws + off);
    p.trace = nullptr;
#ifdef NKV_CHECKED
    {
      const size_t need = attend_ws(a->hkv, nr, (int)ntok);
      const size_t tb = (size_t)p.splits * a->hkv * 64 * 4;
      if (a->workspace_bytes >= need + tb + 256) p.trace = (int*)(ws + a->workspace_bytes - tb);
    }
#endif
    p.ext_part_o = (long long)a->hkv * p.splits * nr * NKV_D;
    p.ext_part_ml = (long long)a->hkv * p.splits * nr * 2;
    p.ext_store = (long long)a->max_blocks * a->hkv * a->block_size * NKV_D;
    p.ext_sink = (long long)a->hkv * a->sink_cap * NKV_D;
    p.ext_ring = (long long)a->hkv * a->ring_cap * NKV_D;
    p.ext_cur = a->n_cur ? (a->n_cur - 1) * a->cur_row_stride + (a->hkv - 1) * a->cur_head_stride + NKV_D : 0;
    p.ext_q = (a->nq - 1) * a->q_row_stride + (a->hq - 1) * a->q_head_stride + NKV_D;
    p.ext_out = (a->nq - 1) * a->out_row_stride + (a->hq - 1) * a->out_head_stride + NKV_D;

    return NKV_OK;
  };
  finish(p);
  finish(pg);
  const int dk_warps = NKV_DECODE_WARPS;  // DK<G>::WARPS
  // decode_kernel: 1 KiB alignment slack + K region (tile, then warp partials)
  // + V region (tile, then the CTA partial)
  auto decode_regions = [&](AttendParams& q) {
    q.tile_rows = q.tps + DT_PAD_ROWS;
    size_t rk = (size_t)q.tile_rows * 256, wp = (size_t)dk_warps * G * (NKV_D + 2) * 4;
    if (rk < wp) rk = wp;
    q.region_k = (int)((rk + 1023) / 1024 * 1024);
  };
  decode_regions(p);
  decode_regions(pg);
  auto smem_of = [&](const AttendParams& q) -> size_t {
    if (a->nq == 1) {
      size_t rv = (size_t)q.tile_rows * 256, cp = (size_t)(128 + G * NKV_D) * 4;
      return 1024 + (size_t)q.region_k + (rv > cp ? rv : cp);
    }
    return (size_t)q.tps * NKV_D * 2 * 2 + (size_t)q.tps * q.nr_pad * 4 + AT_WARPS * 4 * NKV_D * 4 +
           (size_t)nr * NKV_D * 4 + (q.cluster ? (size_t)(128 + nr * NKV_D) * 4 : 0);
  };

  NKV_SUPPORTED(smem_of(pg) <= 220 * 1024 && pg.tps / a->block_size + 2 <= AT_MAX_SLOTS &&
                    (a->nq != 1 || pg.tps <= AT_TPS_MAX_CLUSTER),
                "attend: %d keys per CTA exceed the tile limit", pg.tps);
  if (p.cluster && smem_of(p) > 220 * 1024) p = pg;
  cudaStream_t st = (cudaStream_t)stream;
  const bool q1 = a->nq == 1;
  p.overlap = pg.overlap = a->overlap_select ? 1 : 0;
  if (one_launch && !rank->split_only) {
    // every CTA of the grid waits for every other CTA's keys: cluster mode
    // only, as one cooperative launch (all CTAs co-resident), no overlap
    // with the preceding kernel
    if (!p.cluster || !q1) return FS_DECLINED;
    p.fs_bpc = (rank->nblocks + p.splits * a->hkv - 1) / (p.splits * a->hkv);
    if (p.fs_bpc > FS_BPC_MAX) return FS_DECLINED;
    p.overlap = 0;
  }
  cudaLaunchAttribute attr[3];
  cudaLaunchConfig_t lc = {};
  auto config = [&](const AttendParams& q) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = q.overlap;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = q.cluster ? q.splits : 1;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    lc.gridDim = dim3(q.splits, a->hkv);
    lc.blockDim = dim3(a->nq == 1 ? NKV_DECODE_WARPS * 32 : AT_THREADS);
    lc.dynamicSmemBytes = smem_of(q);
    lc.stream = st;
    lc.attrs = attr;
    lc.numAttrs = 2;
    if (q.fs_keys) {
      attr[2].id = cudaLaunchAttributeCooperative;
      attr[2].val.cooperative = 1;
      lc.numAttrs = 3;
    }
  };
  DecodeMaps maps;
  if (q1) {
    int mask = 0;
    const bool want_sel = a->n_sel > 0 && a->store_kind == NKV_STORE_BF16;
    const DecodeMaps& dm = decode_maps(want_sel ? a->k_store : nullptr, want_sel ? a->v_store : nullptr,
                                       (long long)a->max_blocks * a->hkv * a->block_size,
                                       a->sink_len > 0 ? a->sink_k : nullptr, a->sink_len > 0 ? a->sink_v : nullptr,
                                       (long long)a->hkv * a->sink_cap, a->ring_len > 0 ? a->ring_k : nullptr,
                                       a->ring_len > 0 ? a->ring_v : nullptr, (long long)a->hkv * a->ring_cap, &mask);
    maps = dm;
    p.tma_mask = pg.tma_mask = env_int("NKV_ATTEND_TMA", 1) ? mask : 0;
    NKV_REQUIRE(((uintptr_t)a->k_store & 15) == 0 && ((uintptr_t)a->v_store & 15) == 0 &&
                    ((uintptr_t)a->sink_k & 15) == 0 && ((uintptr_t)a->sink_v & 15) == 0 &&
                    ((uintptr_t)a->ring_k & 15) == 0 && ((uintptr_t)a->ring_v & 15) == 0,
                "attend: store, sink and ring must be 16-byte aligned");
  }
  if (q1 && rank && rank->scores && !rank->peer && G == 4 && a->store_kind == NKV_STORE_BF16 &&
      a->block_size == 64 && a->n_sel >= 1 && a->n_sel <= 32 && a->sink_len <= 64 && a->n_cur == 1 &&
      (p.tma_mask & 1) && (a->sink_len == 0 || (p.tma_mask & 2)) && (a->ring_len == 0 || (p.tma_mask & 4)) &&
      env_int("NKV_DECODE_SPLIT", 1)) {
    const int r = launch_split<false>(p, maps, a, st);
    if (r != FS_DECLINED) return r;
  }
  // one-launch step: the fused form of the same kernel where it applies
  if (q1 && one_launch && G == 4 && a->store_kind == NKV_STORE_BF16 && a->block_size == 64 && a->n_sel >= 1 &&
      a->n_sel <= 32 && a->sink_len <= 64 && a->n_cur == 1 && (p.tma_mask & 1) &&
      (a->sink_len == 0 || (p.tma_mask & 2)) && (a->ring_len == 0 || (p.tma_mask & 4)) &&
      env_int("NKV_DECODE_SPLIT", 1)) {
    const int r = launch_split<true>(p, maps, a, st);
    if (r != FS_DECLINED) return r;
  }
  if (one_launch && rank->split_only) return FS_DECLINED;
  switch (G * 2 + (q1 ? 1 : 0)) {
#define NKV_AT_CASE(GG, QQ)                                                                     \
  case GG * 2 + (QQ ? 1 : 0): {                                                                 \
    auto kern = !QQ ? (const void*)attend_kernel<GG, false>                                     \
                : one_launch ? (const void*)decode_kernel<GG, true> : (const void*)decode_kernel<GG>; \
    if (ensure_smem(kern, smem_of(p) > smem_of(pg) ? smem_of(p) : smem_of(pg), "attend"))       \
      return NKV_ERR_CUDA;                                                                      \
    if (p.cluster) {                                                                            \
      int ok = p.splits <= 8 || !ensure_nonportable_cluster(kern, "attend");                    \
      int nclusters = 0;                                                                        \
      config(p);                                                                                \
      lc.numAttrs = 2; /* occupancy of the cluster shape (without the cooperative flag) */     \
      if (ok && !cluster_occupancy(kern, lc, &nclusters)) ok = 0;                             \
      if (one_launch && (!ok || nclusters < a->hkv)) return FS_DECLINED;                        \
      if (!ok || nclusters < 1) p = pg;                                                         \
    }                                                                                           \
    config(p);                                                                                  \
    g_last_cluster = p.cluster;                                                                 \
    g_last_splits = p.splits;                                                                   \
    g_last_tps = p.tps;                                                                         \
    cudaError_t le = !QQ ? cudaLaunchKernelEx(&lc, attend_kernel<GG, false>, p)                 \
                     : one_launch ? cudaLaunchKernelEx(&lc, decode_kernel<GG, true>, p, maps)   \
                                  : cudaLaunchKernelEx(&lc, decode_kernel<GG>, p, maps);        \
    if (le != cudaSuccess && one_launch) {                                                      \
      /* a refused launch configuration (nothing ran): fall back from now on */                \
      cudaGetLastError();                                                                       \
      g_fs_unavailable = true;                                                                  \
      return FS_DECLINED;                                                                       \
    }                                                                                           \
    if (le != cudaSuccess) return check_launch("attend");                                       \
    break;                                                                                      \
  }
    NKV_AT_CASE(1, true)
    NKV_AT_CASE(1, false)
    NKV_AT_CASE(2, true)
    NKV_AT_CASE(2, false)
    NKV_AT_CASE(4, true)
    NKV_AT_CASE(4, false)
    NKV_AT_CASE(8, true)
    NKV_AT_CASE(8, false)
#undef NKV_AT_CASE
    default:
      return NKV_ERR_UNSUPPORTED;
  }
  return check_launch("attend");
}

extern "C" int nkv_attend_last_config(int* cluster, int* splits, int* keys_per_cta) {
  if (cluster) *cluster = g_last_cluster;
  if (splits) *splits = g_last_splits;
  if (keys_per_cta) *keys_per_cta = g_last_tps;
  return NKV_OK;
}

// ---------------------------------------------------------------------------
// nkv_attend_static: nkv_attend on a scratch buffer that lives inside this
// library, for callers that cannot allocate device memory at call time (a
// host framework owning the device memory pool, serving loops that forbid
// allocation after warm-up, code that must not synchronise the device, which
// cudaMalloc and cudaFree may do).
//
// The scratch is one file-scope device array (NKV_ATTEND_STATIC_SCRATCH_BYTES),
// created when the CUDA module is loaded on a device.  The first call with a
// device current looks its address up once with cudaGetSymbolAddress (which
// may load the module on that device); make that first call before capturing
// a stream.  Every call clears the error word and the per-head merge counters
// (the part of the workspace the kernels expect to start at zero) with
// cudaMemsetAsync on the caller's stream, then launches the unchanged
// nkv_attend path with the scratch as its workspace.  Because that memset sits
// between a preceding selection and the attention, overlap_select is ignored.
// All calls on one device share the scratch: calls that may run at the same
// time (other streams, other host threads) race on it.  The error word the
// kernels write stays readable through nkv_attend_static_check until the next
// call clears it.  The scratch address is cached per device ordinal for the
// life of the process.
// ---------------------------------------------------------------------------
static __device__ __align__(256) unsigned char g_attend_scratch[NKV_ATTEND_STATIC_SCRATCH_BYTES];
static std::mutex g_attend_scratch_mu;
static void* g_attend_scratch_ptr[64];  // per device ordinal, for the life of the process

// Device address of the scratch on the current device (looked up once per
// device, then cached).
static int attend_scratch(const char* who, void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    set_error("%s: no usable current device (%s)", who, cudaGetErrorString(e));
    return NKV_ERR_CUDA;
  }
  std::lock_guard<std::mutex> lock(g_attend_scratch_mu);
  void* ws = g_attend_scratch_ptr[dev];
  if (!ws) {
    e = cudaGetSymbolAddress(&ws, g_attend_scratch);
    if (e != cudaSuccess || !ws) {
      cudaGetLastError();
      set_error("%s: cudaGetSymbolAddress of the scratch failed on device %d: %s", who, dev,
                cudaGetErrorString(e));
      return NKV_ERR_CUDA;
    }
    g_attend_scratch_ptr[dev] = ws;
  }
  *out = ws;
  return NKV_OK;
}

extern "C" int nkv_attend_static(nkv_stream_t stream, const nkv_attend_args* a) {
  NKV_REQUIRE(a, "attend_static: null args");
  NKV_REQUIRE(a->hkv >= 1 && a->hq >= 1 && a->nq >= 1 && a->block_size >= 1 && a->n_sel >= 0 &&
                  a->sink_len >= 0 && a->ring_len >= 0 && a->n_cur >= 0,
              "attend_static: bad geometry");
  const long long ntok = (long long)a->n_sel * a->block_size + a->sink_len + a->ring_len + a->n_cur;
  NKV_REQUIRE(ntok >= 1 && ntok < (1ll << 30), "attend_static: key count %lld out of range", ntok);
  const size_t need = nkv_attend_workspace_bytes(a->hkv, a->hq, a->nq, (int)ntok);
  NKV_REQUIRE(need <= (size_t)NKV_ATTEND_STATIC_SCRATCH_BYTES,
              "attend_static: this call needs %zu bytes of workspace but the static scratch holds %zu "
              "(fewer keys, heads or queries per call, or nkv_attend with a caller workspace)",
              need, (size_t)NKV_ATTEND_STATIC_SCRATCH_BYTES);
  void* ws = nullptr;
  int rc = attend_scratch("attend_static", &ws);
  if (rc != NKV_OK) return rc;
  cudaError_t e;
  // error word (256 B) + per-head counters, as laid out by the attend workspace
  const size_t zero_bytes = 256 + ((size_t)(a->hkv * 4 + 255) / 256) * 256;
  e = cudaMemsetAsync(ws, 0, zero_bytes, (cudaStream_t)stream);
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error("attend_static: clearing the scratch header failed: %s", cudaGetErrorString(e));
    return NKV_ERR_CUDA;
  }
  nkv_attend_args b = *a;
  b.workspace = ws;
  b.workspace_bytes = NKV_ATTEND_STATIC_SCRATCH_BYTES;
  b.overlap_select = 0;
  return nkv_attend(stream, &b);
}

// The error word of the static scratch on the current device: the same
// contract as nkv_check on a caller workspace (synchronous on `stream`,
// NKV_ERR_DEVICE and cleared when a kernel recorded an error).
extern "C" int nkv_attend_static_check(nkv_stream_t stream) {
  void* ws = nullptr;
  int rc = attend_scratch("attend_static_check", &ws);
  if (rc != NKV_OK) return rc;
  return nkv_check(stream, ws);
}
