// Kernel (1): block-representative scoring + protection + exact Top-K.
//
// One launch.  Scoring CTAs each own a contiguous range of blocks for all KV
// heads; a warp scores one (kv head, block) unit at a time:
//   lanes 8j..8j+7 hold representative j, 16 dims each (one 1 KiB unit is read
//   by 2 x 128-bit loads per lane, fully coalesced), query rows for the head's
//   G query heads come from L1.  Per (row, head) the 16-dim partial dots are
//   summed over 8 lanes (3 shuffles), the max over reps takes 2 more.
// The block score (max over heads) goes to a workspace array; the last CTA to
// finish (atomic ticket, no spinning) ranks all blocks:
//   k <= 32 : every warp keeps a sorted top-32 of its chunks in registers
//             (bitonic sort + merge on 64-bit keys), chunks whose max cannot
//             enter the list are skipped, then a 3-level merge tree.
//   k > 32  : bitonic sort of all keys in shared memory.
// Keys order by (score desc, id asc), so the result is deterministic.
#include <stdlib.h>

#include "nkv_common.cuh"
#include "nkv_host.h"

namespace nkv {

constexpr int SEL_THREADS = 512;
constexpr int SEL_WARPS = SEL_THREADS / 32;
constexpr int SEL_MAX_SMEM_SORT = 16384;  // generic path: keys in shared memory

struct SelectParams {
  const __nv_bfloat16* q;
  long long q_row_stride, q_head_stride;
  int nq, hq, hkv, r;
  const __nv_bfloat16* reps;
  int max_blocks, nblocks;
  const int* protected_ids;
  int n_protected;
  int k;
  int per_query;  // 1: separate ranking per query row (lossless verify)
  int score_only; // 1: write the masked block scores and stop (the ranking happens in the consumer)
  long long* out_ids;
  float* out_topk_scores;
  float* out_block_scores;
  // per-query outputs
  long long* out_union;
  int* out_count;
  unsigned char* out_allowed;
  // workspace
  float* scores;       // [nq or 1][nblocks]
  unsigned* ticket;    // one counter
  int bpc;             // blocks per scoring CTA
  int* err;
  long long ext_reps, ext_q;
  int* trace;  // checked builds: per-CTA phase stamps (or null)
  // KV-head sharding over peer memory (xs_P > 0): every block score is also
  // pushed, tagged with this step's epoch, into each rank's exchange buffer at
  // xs_peer[r] + (parity * xs_P + xs_rank) * xs_cap + block
  u64* xs_peer[NKV_MAX_PEERS];
  int xs_P, xs_rank, xs_cap;
  const uint32_t* xs_epoch;  // this rank's exchange header (epoch word)
};

// Score of one (head, block) unit for query row n (or max over rows when n < 0).
template <int G>
__device__ __forceinline__ float unit_score(const SelectParams& p, int h, int b, int n_lo, int n_hi) {
  const int lane = threadIdx.x & 31;
  const int j = lane >> 3;       // representative handled by this lane group
  const int c = lane & 7;        // 16-dim column slice
  float best = -INFINITY;
  for (int j0 = 0; j0 < p.r; j0 += 4) {
    const int jj = j0 + j;
    const bool valid = jj < p.r;
    float rv[16];
    if (valid && NKV_INB(p.err, 50, (((long long)h * p.max_blocks + b) * p.r + jj) * NKV_D + c * 16, 16, p.ext_reps)) {
      const __nv_bfloat16* src = p.reps + (((long long)h * p.max_blocks + b) * p.r + jj) * NKV_D + c * 16;
      uint4 a = __ldg(reinterpret_cast<const uint4*>(src));
      uint4 bq = __ldg(reinterpret_cast<const uint4*>(src + 8));
      unpack8(a, rv);
      unpack8(bq, rv + 8);
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i) rv[i] = 0.f;
    }
    for (int n = n_lo; n < n_hi; ++n) {
      float part[G];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const __nv_bfloat16* qs = p.q + n * p.q_row_stride + (long long)(h * G + g) * p.q_head_stride + c * 16;
        float qv[16];
        if (!NKV_INB(p.err, 51, qs - p.q, 16, p.ext_q)) qs = p.q;
        unpack8(__ldg(reinterpret_cast<const uint4*>(qs)), qv);
        unpack8(__ldg(reinterpret_cast<const uint4*>(qs + 8)), qv + 8);
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < 16; ++i) s = fmaf(qv[i], rv[i], s);
        part[g] = s;
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float s = part[g];
        s += __shfl_xor_sync(FULL, s, 1);
        s += __shfl_xor_sync(FULL, s, 2);
        s += __shfl_xor_sync(FULL, s, 4);
        if (valid) best = fmaxf(best, s);
      }
    }
  }
  best = fmaxf(best, __shfl_xor_sync(FULL, best, 8));
  best = fmaxf(best, __shfl_xor_sync(FULL, best, 16));
  return best;
}

__device__ __forceinline__ bool is_protected(const SelectParams& p, int b) {
  for (int i = 0; i < p.n_protected; ++i)
    if (__ldg(p.protected_ids + i) == b) return true;
  return false;
}

// Top-k (k <= 32) of scores[0..n) by the warp-list method; result in lane order
// of warp 0 (descending).  All threads of the CTA must call.
__device__ u64 topk32(const float* scores, int n, u64* lists /* [SEL_WARPS][32] smem */) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  u64 run = 0;  // 0 is below every real key
  const int nchunks = (n + 31) / 32;
  for (int ch = warp; ch < nchunks; ch += SEL_WARPS) {
    const int i = ch * 32 + lane;
    u64 key = i < n ? make_key(scores[i], (uint32_t)i) : 0ull;
    // skip chunks that cannot improve the running list
    u64 run_min = shfl64(run, 31);
    uint32_t hi = (uint32_t)(key >> 32);
    uint32_t chunk_hi = __reduce_max_sync(FULL, hi);
    if (chunk_hi < (uint32_t)(run_min >> 32)) continue;
    key = warp_sort_desc(key);
    run = warp_merge_desc(run, key);
  }
  lists[warp * 32 + lane] = run;
  __syncthreads();
  for (int s = 1; s < SEL_WARPS; s <<= 1) {
    if ((warp % (2 * s)) == 0 && warp + s < SEL_WARPS) {
      u64 a = lists[warp * 32 + lane];
      u64 b = lists[(warp + s) * 32 + lane];
      lists[warp * 32 + lane] = warp_merge_desc(a, b);
    }
    __syncthreads();
  }
  return lists[lane];
}

// Top-k (k <= 32) with a threshold filter: every thread of the CTA holds the
// keys i = tid, tid + blockDim.x, ...; the maximum of each group of 16
// consecutive lanes is taken per round, and the smallest of those group maxima
// (over >= 32 groups) is a score that at least 32 blocks reach.  Only blocks
// scoring >= that threshold are compacted and ranked (bitonic sort + merge of
// warp lists); when too many survive the function falls back to topk32().
// Requires blockDim.x == SEL_THREADS and n <= 4 * SEL_THREADS.
__device__ u64 topk32_filtered(const float* scores, int n, u64* lists, u64* cand, int* s_cnt,
                               uint32_t* s_thr) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int tid = threadIdx.x;
  // threshold: min over (group of 16 lanes x round) maxima of the orderable score
  uint32_t gmin = 0xffffffffu;
  for (int base = 0; base < n; base += SEL_THREADS) {
    const int i = base + tid;
    const uint32_t o = i < n ? f32_order(scores[i]) : 0u;
    // max over 16 lanes (xor 1..8 stays within a half warp)
    uint32_t m = o;
#pragma unroll
    for (int x = 1; x < 16; x <<= 1) m = max(m, __shfl_xor_sync(FULL, m, x));
    // only groups that hold real keys take part
    const bool full = (base + (tid & ~15)) < n;
    if (full) gmin = min(gmin, m);
  }
  gmin = __reduce_min_sync(FULL, gmin);
  if (tid == 0) *s_cnt = 0;
  if (lane == 0) s_thr[warp] = gmin;
  __syncthreads();
  uint32_t thr = 0xffffffffu;
#pragma unroll
  for (int w = 0; w < SEL_WARPS; ++w) thr = min(thr, s_thr[w]);
  // compact survivors
  for (int base = 0; base < n; base += SEL_THREADS) {
    const int i = base + tid;
    const bool keep = i < n && f32_order(scores[i]) >= thr;
    const unsigned bal = __ballot_sync(FULL, keep);
    int off = 0;
    if (lane == 0 && bal) off = atomicAdd(s_cnt, __popc(bal));
    off = __shfl_sync(FULL, off, 0);
    if (keep) {
      const int slot = off + __popc(bal & ((1u << lane) - 1));
      if (slot < 4 * 32) cand[slot] = make_key(scores[i], (uint32_t)i);
    }
  }
  __syncthreads();
  const int cnt = *s_cnt;
  if (cnt > 4 * 32) return topk32(scores, n, lists);  // rare: flat scores
  // 4 warps sort 32 candidates each, then two merge levels
  if (warp < 4) {
    const int i = warp * 32 + lane;
    u64 key = i < cnt ? cand[i] : 0ull;
    lists[warp * 32 + lane] = warp_sort_desc(key);
  }
  __syncthreads();
  if (warp < 2) lists[warp * 32 + lane] = warp_merge_desc(lists[warp * 32 + lane], lists[(warp + 2) * 32 + lane]);
  __syncthreads();
  if (warp == 0) lists[lane] = warp_merge_desc(lists[lane], lists[32 + lane]);
  __syncthreads();
  return lists[lane];
}

// Generic ranking: full bitonic sort (descending) of n keys in shared memory.
__device__ void sort_all_desc(const float* scores, int n, u64* keys, int npow2) {
  for (int i = threadIdx.x; i < npow2; i += blockDim.x)
    keys[i] = i < n ? make_key(__ldcg(scores + i), (uint32_t)i) : 0ull;
  __syncthreads();
  for (int k = 2; k <= npow2; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < npow2; i += blockDim.x) {
        int partner = i ^ j;
        if (partner > i) {
          u64 a = keys[i], b = keys[partner];
          bool desc = (i & k) == 0;
          if ((a < b) == desc) {
            keys[i] = b;
            keys[partner] = a;
          }
        }
      }
      __syncthreads();
    }
  }
}

template <int G>
__global__ void __launch_bounds__(SEL_THREADS) select_kernel(SelectParams p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ float part[SEL_WARPS][8];
  __shared__ u64 lists[SEL_WARPS * 32];
  __shared__ u64 cand[4 * 32];
  __shared__ int s_cnt;
  __shared__ uint32_t s_thr[SEL_WARPS];
  __shared__ unsigned s_ticket;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // a dependent attend launch may begin now; it waits for this grid's
  // completion before it reads the selected ids
  pdl_launch_dependents();
#ifdef NKV_CHECKED
  int* trc = p.trace ? p.trace + blockIdx.x * 8 : nullptr;
#else
  int* trc = nullptr;
#endif
  NKV_STAMP(trc, 0);
  const int b0 = blockIdx.x * p.bpc;
  const int nb = min(p.bpc, p.nblocks - b0);
  const int nrows = p.per_query ? p.nq : 1;
  // protected flags of this CTA's blocks, set in one parallel pass (the list
  // is short; a per-block scan would chain its loads)
  __shared__ unsigned char s_prot[256];
  for (int i = threadIdx.x; i < nb && i < 256; i += blockDim.x) s_prot[i] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < p.n_protected; i += blockDim.x) {
    const int b = __ldg(p.protected_ids + i) - b0;
    if (b >= 0 && b < nb && b < 256) s_prot[b] = 1;
  }
  // (made visible by the barrier that follows the first scoring round)

  // ---- phase 1: scores for this CTA's blocks ---------------------------------
  for (int row = 0; row < nrows; ++row) {
    const int n_lo = p.per_query ? row : 0;
    const int n_hi = p.per_query ? row + 1 : p.nq;
    for (int bl0 = 0; bl0 < nb; bl0 += 8) {
      const int nbl = min(8, nb - bl0);
      // units (h, bl) spread over the warps
      float acc[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = -INFINITY;
      for (int u = warp; u < p.hkv * nbl; u += SEL_WARPS) {
        const int h = u / nbl, bl = u % nbl;
        float s = unit_score<G>(p, h, b0 + bl0 + bl, n_lo, n_hi);
#pragma unroll
        for (int i = 0; i < 8; ++i)
          if (i == bl) acc[i] = fmaxf(acc[i], s);
      }
      if (lane == 0)
#pragma unroll
        for (int i = 0; i < 8; ++i) part[warp][i] = acc[i];
      __syncthreads();
      if (threadIdx.x < nbl) {
        const int b = b0 + bl0 + threadIdx.x;
        float m = -INFINITY;
        for (int w = 0; w < SEL_WARPS; ++w) m = fmaxf(m, part[w][threadIdx.x]);
        if ((bl0 + threadIdx.x < 256) ? s_prot[bl0 + threadIdx.x] : is_protected(p, b)) m = -INFINITY;
        p.scores[(long long)row * p.nblocks + b] = m;
        if (p.out_block_scores) p.out_block_scores[(long long)row * p.nblocks + b] = m;
        if (p.xs_P) {
          const uint32_t ep = ld_peer_u32(p.xs_epoch);
          const u64 w = ((u64)step_tag(ep) << 32) | f32_order(m);
          const long long at = ((long long)(ep & 1u) * p.xs_P + p.xs_rank) * p.xs_cap + b;
          for (int r = 0; r < p.xs_P; ++r) st_peer_u64(p.xs_peer[r] + at, w);
        }
      }
      __syncthreads();
    }
  }

  NKV_STAMP(trc, 1);
  if (p.score_only) return;

  // ---- hand-off: the last CTA ranks --------------------------------------------
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_ticket = atomicAdd(p.ticket, 1u);
  __syncthreads();
  NKV_STAMP(trc, 2);
  if (s_ticket != gridDim.x - 1) return;
  __threadfence();
  if (threadIdx.x == 0) *p.ticket = 0u;  // ready for the next launch

  // stage every score in shared memory with one parallel load
  const int nrows_rank = p.per_query ? p.nq : 1;
  float* sscores = reinterpret_cast<float*>(smem_raw);
  u64* keys = reinterpret_cast<u64*>(smem_raw);
  int npow2 = 1;
  while (npow2 < p.nblocks) npow2 <<= 1;
  const bool generic = !p.per_query && p.k > 32;
  if (!generic) {
    for (int i = threadIdx.x; i < nrows_rank * p.nblocks; i += blockDim.x) sscores[i] = __ldcg(p.scores + i);
    __syncthreads();
  }

  NKV_STAMP(trc, 3);
  if (!p.per_query) {
    if (p.k <= 32) {
      u64 key = p.nblocks <= 4 * SEL_THREADS && p.nblocks >= 32 * 16
                    ? topk32_filtered(sscores, p.nblocks, lists, cand, &s_cnt, s_thr)
                    : topk32(sscores, p.nblocks, lists);
      if (warp == 0 && lane < p.k) {
        p.out_ids[lane] = key_id(key);
        if (p.out_topk_scores) p.out_topk_scores[lane] = key_score(key);
      }
      NKV_STAMP(trc, 4);
    } else {
      sort_all_desc(p.scores, p.nblocks, keys, npow2);  // reads the workspace
      for (int i = threadIdx.x; i < p.k; i += blockDim.x) {
        p.out_ids[i] = key_id(keys[i]);
        if (p.out_topk_scores) p.out_topk_scores[i] = key_score(keys[i]);
      }
    }
    return;
  }

  // ---- per-query rankings, union and allowed mask (k <= 32, nq <= 8) ----------
  __shared__ int ent[8 * 32];
  for (int row = 0; row < p.nq; ++row) {
    u64 key = topk32(sscores + (long long)row * p.nblocks, p.nblocks, lists);
    if (warp == 0 && lane < p.k) ent[row * p.k + lane] = (int)key_id(key);
    __syncthreads();
  }
  const int E = p.nq * p.k;
  __shared__ int s_rank[8 * 32];
  __shared__ int s_first[8 * 32];
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const int id = ent[e];
    int first = 1;
    for (int f = 0; f < e; ++f)
      if (ent[f] == id) first = 0;
    s_first[e] = first;
  }
  __syncthreads();
  // rank = number of distinct ids below mine (each counted at its first entry)
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const int id = ent[e];
    int rank = 0;
    for (int f = 0; f < E; ++f) rank += (s_first[f] && ent[f] < id) ? 1 : 0;
    s_rank[e] = rank;
  }
  __syncthreads();
  int U = 0;
  for (int e = 0; e < E; ++e) U += s_first[e];
  for (int i = threadIdx.x; i < p.nq * E; i += blockDim.x) p.out_allowed[i] = 0;
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const int row = e / p.k;
    if (s_first[e]) p.out_union[s_rank[e]] = ent[e];
    p.out_allowed[row * E + s_rank[e]] = 1;
  }
  if (threadIdx.x == 0) *p.out_count = U;
}

// Score-only form (the decode step's scoring grid, ranked by the attention
// CTAs): a lighter grid of at most one 256-thread CTA per SM, so that the
// attention CTAs launched after it (programmatic dependent launch) are
// resident beside it and run their prologue while it scores.  CTA c owns
// blocks [c * bpc, (c + 1) * bpc) for every KV head; block score = max over
// the CTA's warps' partial maxima, protected blocks -inf.  Two kernels with
// the same interface: score_kernel (fp32 FMA, for up to 4 blocks per CTA)
// and score_kernel_tc (tensor cores, for larger ranges).
// Bulk prefetch of `bytes` (a multiple of 16, 16-byte aligned) into L2.
__device__ __forceinline__ void prefetch_l2_range(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

constexpr int SC_THREADS = 256;
constexpr int SC_WARPS = SC_THREADS / 32;
constexpr int SC_UPW = 4;       // blocks per CTA are a multiple of this
constexpr int SC_BPC_MAX = 64;  // blocks per CTA
constexpr int SC_ROWS = 32;     // representative rows per unit (4 n-tiles)

// Scalar form for small block ranges (up to 4 blocks per CTA, e.g. 32K
// tokens): warp w scores heads w, w + 8, ...; per head the warp takes its
// blocks SC_UPW at a time with every representative load of the group issued
// before the arithmetic (one DRAM round trip per group).  Lane layout and
// summation order are unit_score's, so the scores are bit-identical to
// select_kernel's.  With more blocks per CTA its fp32 FMA stream grows with
// the blocks and score_kernel_tc (below) is faster.
template <int G>
__global__ void __launch_bounds__(SC_THREADS) score_kernel(SelectParams p) {
  __shared__ float part[SC_WARPS][SC_BPC_MAX];
  __shared__ unsigned char s_prot[SC_BPC_MAX];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int j = lane >> 3, c = lane & 7;
  const int b0 = blockIdx.x * p.bpc;
  const int nb = min(p.bpc, p.nblocks - b0);
  // launched with programmatic dependent launch: the CTAs may be resident
  // before the preceding kernel has finished.  Meanwhile each warp prefetches
  // its heads' representative rows into L2 (a prefetch reads nothing into the
  // SM, so it cannot see data older than what the loads below will); every
  // read waits for the preceding kernel, and the dependent attention grid is
  // released only then (its prologue reads q and the current token, which the
  // preceding kernel may produce)
  if (lane == 0 && nb > 0)
    for (int h = warp; h < p.hkv; h += SC_WARPS)
      prefetch_l2_range(p.reps + ((long long)h * p.max_blocks + b0) * p.r * NKV_D, (uint32_t)(nb * p.r * NKV_D * 2));
  pdl_wait();
  pdl_launch_dependents();
  for (int i = threadIdx.x; i < SC_WARPS * SC_BPC_MAX; i += SC_THREADS) (&part[0][0])[i] = -INFINITY;
  for (int i = threadIdx.x; i < SC_BPC_MAX; i += SC_THREADS) s_prot[i] = 0;
  __syncthreads();
  // the protected ids are loaded now and applied after the scoring, so that
  // their round trip overlaps it
  const int prot0 = (int)threadIdx.x < p.n_protected ? __ldg(p.protected_ids + threadIdx.x) : -1;
  const bool jvalid = j < p.r;
  for (int h = warp; h < p.hkv; h += SC_WARPS) {
    // this lane's 16-dim slice of the head's G query rows
    uint4 qa[G], qb[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const __nv_bfloat16* qs = p.q + (long long)(h * G + g) * p.q_head_stride + c * 16;
      if (!NKV_INB(p.err, 51, qs - p.q, 16, p.ext_q)) qs = p.q;
      qa[g] = __ldg(reinterpret_cast<const uint4*>(qs));
      qb[g] = __ldg(reinterpret_cast<const uint4*>(qs + 8));
    }
    for (int u0 = 0; u0 < nb; u0 += SC_UPW) {
      uint4 ra[SC_UPW], rb[SC_UPW];
#pragma unroll
      for (int u = 0; u < SC_UPW; ++u) {
        ra[u] = rb[u] = make_uint4(0u, 0u, 0u, 0u);
        const long long off = (((long long)h * p.max_blocks + b0 + u0 + u) * p.r + j) * NKV_D + c * 16;
        if (u0 + u < nb && jvalid && NKV_INB(p.err, 50, off, 16, p.ext_reps)) {
          ra[u] = __ldg(reinterpret_cast<const uint4*>(p.reps + off));
          rb[u] = __ldg(reinterpret_cast<const uint4*>(p.reps + off + 8));
        }
      }
#pragma unroll
      for (int u = 0; u < SC_UPW; ++u) {
        float rv[16];
        unpack8(ra[u], rv);
        unpack8(rb[u], rv + 8);
        float best = -INFINITY;
#pragma unroll
        for (int g = 0; g < G; ++g) {
          float qv[16];
          unpack8(qa[g], qv);
          unpack8(qb[g], qv + 8);
          float sc = 0.f;
#pragma unroll
          for (int i = 0; i < 16; ++i) sc = fmaf(qv[i], rv[i], sc);
          sc += __shfl_xor_sync(FULL, sc, 1);
          sc += __shfl_xor_sync(FULL, sc, 2);
          sc += __shfl_xor_sync(FULL, sc, 4);
          if (jvalid) best = fmaxf(best, sc);
        }
        best = fmaxf(best, __shfl_xor_sync(FULL, best, 8));
        best = fmaxf(best, __shfl_xor_sync(FULL, best, 16));
        if (lane == 0 && u0 + u < nb) part[warp][u0 + u] = fmaxf(part[warp][u0 + u], best);
      }
    }
  }
  if (prot0 >= b0 && prot0 - b0 < nb) s_prot[prot0 - b0] = 1;
  for (int i = threadIdx.x + SC_THREADS; i < p.n_protected; i += SC_THREADS) {
    const int b = __ldg(p.protected_ids + i) - b0;
    if (b >= 0 && b < nb) s_prot[b] = 1;
  }
  __syncthreads();
  if (threadIdx.x < nb) {
    const int b = b0 + threadIdx.x;
    float m = -INFINITY;
#pragma unroll
    for (int w = 0; w < SC_WARPS; ++w) m = fmaxf(m, part[w][threadIdx.x]);
    if (s_prot[threadIdx.x]) m = -INFINITY;
    p.scores[b] = m;
    if (p.out_block_scores) p.out_block_scores[b] = m;
    if (p.xs_P) {
      const uint32_t ep = ld_peer_u32(p.xs_epoch);
      const u64 w = ((u64)step_tag(ep) << 32) | f32_order(m);
      const long long at = ((long long)(ep & 1u) * p.xs_P + p.xs_rank) * p.xs_cap + b;
      for (int r = 0; r < p.xs_P; ++r) st_peer_u64(p.xs_peer[r] + at, w);
    }
  }
}

// Tensor-core form for larger block ranges (e.g. 16 blocks per CTA at 128K
// tokens).  The work is cut into units of 32 representative rows of one head
// (contiguous in [hkv][max_blocks][r][D]); warp w takes units w, w + 8, ...,
// so every warp has work whatever the number of heads.  A unit is scored with
// mma.sync m16n8k16 (bf16 in, fp32 accumulate): the head's G query rows are
// the M rows (rows >= G zero), the 32 representative rows four n-tiles of 8
// columns, K = D in a permuted order that is the same for both operands (at
// k-steps 2i and 2i + 1 lane quad t holds dims 32 i + 8 t ... + 7, one 16-byte
// load per operand row), so each product is a full dot product.  All 16 loads
// of a lane for the unit are issued before its 32 mma.  Per representative
// row the max over the query rows (shuffles), then per block the max over its
// r rows, kept per (warp, block) in shared memory.  Its sums run in the tensor
// core's order, so its scores can differ from score_kernel's in the last bits.
template <int G>
__global__ void __launch_bounds__(SC_THREADS) score_kernel_tc(SelectParams p) {
  static_assert(G >= 1 && G <= 8, "query rows per KV head fit the 16 M rows");
  __shared__ float part[SC_WARPS][SC_BPC_MAX];
  __shared__ float s_rows[SC_WARPS][SC_ROWS];
  __shared__ unsigned char s_prot[SC_BPC_MAX];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int b0 = blockIdx.x * p.bpc;
  const int nb = min(p.bpc, p.nblocks - b0);
  // launched with programmatic dependent launch: the CTAs may be resident
  // before the preceding kernel has finished.  Meanwhile each warp prefetches
  // its heads' representative rows into L2 (a prefetch reads nothing into the
  // SM, so it cannot see data older than what the loads below will); every
  // read waits for the preceding kernel, and the dependent attention grid is
  // released only then (its prologue reads q and the current token, which the
  // preceding kernel may produce)
  if (lane == 0 && nb > 0)
    for (int h = warp; h < p.hkv; h += SC_WARPS)
      prefetch_l2_range(p.reps + ((long long)h * p.max_blocks + b0) * p.r * NKV_D, (uint32_t)(nb * p.r * NKV_D * 2));
  pdl_wait();
  pdl_launch_dependents();
  for (int i = threadIdx.x; i < SC_WARPS * SC_BPC_MAX; i += SC_THREADS) (&part[0][0])[i] = -INFINITY;
  for (int i = threadIdx.x; i < SC_BPC_MAX; i += SC_THREADS) s_prot[i] = 0;
  __syncthreads();
  // the protected ids are loaded now and applied after the scoring, so that
  // their round trip overlaps it
  const int prot0 = (int)threadIdx.x < p.n_protected ? __ldg(p.protected_ids + threadIdx.x) : -1;
  const int rows = nb * p.r;  // representative rows of one head in this CTA
  const int upr = (rows + SC_ROWS - 1) / SC_ROWS;
  int cur_h = -1;
  uint4 qf[4] = {};
  for (int u = warp; u < upr * p.hkv; u += SC_WARPS) {
    const int h = u / upr, row0 = (u % upr) * SC_ROWS;
    if (h != cur_h) {  // this lane's dims 32 i + 8 t ... + 7 of query row g of head h
      cur_h = h;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        qf[i] = make_uint4(0u, 0u, 0u, 0u);
        if (g < G) {
          const __nv_bfloat16* qs = p.q + (long long)(h * G + g) * p.q_head_stride + i * 32 + t * 8;
          if (NKV_INB(p.err, 51, qs - p.q, 8, p.ext_q)) qf[i] = __ldg(reinterpret_cast<const uint4*>(qs));
        }
      }
    }
    const __nv_bfloat16* rbase = p.reps + ((long long)h * p.max_blocks + b0) * p.r * NKV_D;
    uint4 rf[SC_ROWS / 8][4];
#pragma unroll
    for (int j = 0; j < SC_ROWS / 8; ++j) {
      const int rr = row0 + j * 8 + g;
      const long long off = (long long)rr * NKV_D + t * 8;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        rf[j][i] = make_uint4(0u, 0u, 0u, 0u);
        if (rr < rows &&
            NKV_INB(p.err, 50, ((long long)h * p.max_blocks + b0) * p.r * NKV_D + off + i * 32, 8, p.ext_reps))
          rf[j][i] = __ldg(reinterpret_cast<const uint4*>(rbase + off + i * 32));
      }
    }
    float c[SC_ROWS / 8][4];
#pragma unroll
    for (int j = 0; j < SC_ROWS / 8; ++j) c[j][0] = c[j][1] = c[j][2] = c[j][3] = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
      for (int j = 0; j < SC_ROWS / 8; ++j) mma_bf16(c[j], qf[i].x, 0u, qf[i].y, 0u, rf[j][i].x, rf[j][i].y);
#pragma unroll
      for (int j = 0; j < SC_ROWS / 8; ++j) mma_bf16(c[j], qf[i].z, 0u, qf[i].w, 0u, rf[j][i].z, rf[j][i].w);
    }
    // c[j][0..1]: query row g x representative rows row0 + 8 j + 2 t, + 1;
    // max over the query rows (lanes of a column), then lanes 0..3 hold the
    // unit's 32 row scores
#pragma unroll
    for (int j = 0; j < SC_ROWS / 8; ++j) {
      float v0 = g < G ? c[j][0] : -INFINITY, v1 = g < G ? c[j][1] : -INFINITY;
#pragma unroll
      for (int x = 4; x < 32; x <<= 1) {
        v0 = fmaxf(v0, __shfl_xor_sync(FULL, v0, x));
        v1 = fmaxf(v1, __shfl_xor_sync(FULL, v1, x));
      }
      if (g == 0) {
        s_rows[warp][j * 8 + 2 * t] = v0;
        s_rows[warp][j * 8 + 2 * t + 1] = v1;
      }
    }
    __syncwarp();
    // blocks of the unit: lane l takes block row0 / r + l (its rows inside the unit)
    const int blo = row0 / p.r, bhi = min((row0 + SC_ROWS - 1) / p.r, nb - 1);
    if (lane <= bhi - blo) {
      const int bl = blo + lane;
      const int ra = max(row0, bl * p.r), rb = min(min(row0 + SC_ROWS, (bl + 1) * p.r), rows);
      float m = -INFINITY;
      for (int rr = ra; rr < rb; ++rr) m = fmaxf(m, s_rows[warp][rr - row0]);
      part[warp][bl] = fmaxf(part[warp][bl], m);
    }
    __syncwarp();
  }
  if (prot0 >= b0 && prot0 - b0 < nb) s_prot[prot0 - b0] = 1;
  for (int i = threadIdx.x + SC_THREADS; i < p.n_protected; i += SC_THREADS) {
    const int b = __ldg(p.protected_ids + i) - b0;
    if (b >= 0 && b < nb) s_prot[b] = 1;
  }
  __syncthreads();
  if (threadIdx.x < nb) {
    const int b = b0 + threadIdx.x;
    float m = -INFINITY;
#pragma unroll
    for (int w = 0; w < SC_WARPS; ++w) m = fmaxf(m, part[w][threadIdx.x]);
    if (s_prot[threadIdx.x]) m = -INFINITY;
    p.scores[b] = m;
    if (p.out_block_scores) p.out_block_scores[b] = m;
    if (p.xs_P) {
      const uint32_t ep = ld_peer_u32(p.xs_epoch);
      const u64 w = ((u64)step_tag(ep) << 32) | f32_order(m);
      const long long at = ((long long)(ep & 1u) * p.xs_P + p.xs_rank) * p.xs_cap + b;
      for (int r = 0; r < p.xs_P; ++r) st_peer_u64(p.xs_peer[r] + at, w);
    }
  }
}

}  // namespace nkv

using namespace nkv;

static int launch_score(cudaStream_t st, SelectParams& p, int G) {
  // the blocks are spread over up to 2 CTAs per SM (NKV_SCORE_CPS): at 32K that
  // still rounds to 4 blocks per CTA (128 CTAs, which sit beside the attention
  // CTAs); at 128K it halves the rows per CTA to one 32-row unit per warp (one
  // round trip instead of two): 2.65 -> 2.57 ms per token of the 131072-token
  // model decode, although the attention CTAs then start after the scoring
  const int cps = knob("NKV_SCORE_CPS", 2);
  const int sms = sm_count() * (cps > 1 ? cps : 1);
  const int per = (p.nblocks + sms - 1) / sms;
  p.bpc = (per + SC_UPW - 1) / SC_UPW * SC_UPW;
  const int grid = (p.nblocks + p.bpc - 1) / p.bpc;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = knob("NKV_SCORE_PDL", 1) != 0 ? 1 : 0;
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3(grid);
  lc.blockDim = dim3(SC_THREADS);
  lc.dynamicSmemBytes = 0;
  lc.stream = st;
  lc.attrs = attr;
  lc.numAttrs = 1;
  cudaError_t e;
  // NKV_SCORE_TC: 1 always the tensor-core form, 0 never, default above 4 blocks per CTA
  const int tc_knob = knob("NKV_SCORE_TC", -1);
  const bool tc = tc_knob > 0 || (tc_knob < 0 && p.bpc > SC_UPW);
  switch (G) {
    case 1: e = tc ? cudaLaunchKernelEx(&lc, score_kernel_tc<1>, p) : cudaLaunchKernelEx(&lc, score_kernel<1>, p); break;
    case 2: e = tc ? cudaLaunchKernelEx(&lc, score_kernel_tc<2>, p) : cudaLaunchKernelEx(&lc, score_kernel<2>, p); break;
    case 4: e = tc ? cudaLaunchKernelEx(&lc, score_kernel_tc<4>, p) : cudaLaunchKernelEx(&lc, score_kernel<4>, p); break;
    default:
      set_error("score: unsupported G=%d", G);
      return NKV_ERR_UNSUPPORTED;
  }
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error("score: launch failed: %s", cudaGetErrorString(e));
    return NKV_ERR_CUDA;
  }
  return check_launch("score");
}

static int launch_select(cudaStream_t st, SelectParams& p, int G) {
  const int sms = sm_count();
  // score-only, one query row, r <= 4, G <= 4: the lighter scoring grid
  if (p.score_only && !p.per_query && p.nq == 1 && p.r <= 4 && G <= 4 &&
      (p.nblocks + sms - 1) / sms <= SC_BPC_MAX && knob("NKV_SCORE_GRID", 1))
    return launch_score(st, p, G);
  // one (head, block) unit per warp when the grid fits in one wave (<= 4 CTAs/SM)
  int bpc = (p.nblocks + 4 * sms - 1) / (4 * sms);
  const int unit_bpc = SEL_WARPS / (p.hkv < SEL_WARPS ? p.hkv : SEL_WARPS);
  if (bpc < unit_bpc) bpc = unit_bpc;
  if (knob("NKV_SEL_BPC", 0) > 0) bpc = knob("NKV_SEL_BPC", 0);  // blocks per scoring CTA (tuning override)
  p.bpc = bpc;
  const int grid = (p.nblocks + bpc - 1) / bpc;
  int npow2 = 1;
  while (npow2 < p.nblocks) npow2 <<= 1;
  const size_t rows = p.per_query ? (size_t)p.nq : 1;
  size_t smem = (!p.per_query && p.k > 32) ? (size_t)npow2 * sizeof(u64) : rows * p.nblocks * sizeof(float);
  switch (G) {
#define NKV_SEL_CASE(GG)                                                                       \
  case GG:                                                                                     \
    if (ensure_smem(select_kernel<GG>, smem, "select")) return NKV_ERR_CUDA;                  \
    select_kernel<GG><<<grid, SEL_THREADS, smem, st>>>(p);                                      \
    break;
    NKV_SEL_CASE(1)
    NKV_SEL_CASE(2)
    NKV_SEL_CASE(4)
    NKV_SEL_CASE(8)
#undef NKV_SEL_CASE
    default:
      set_error("select: unsupported G=%d", G);
      return NKV_ERR_UNSUPPORTED;
  }
  return check_launch("select");
}

static size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

extern "C" size_t nkv_select_workspace_bytes(int max_blocks, int nq) {
  if (max_blocks < 1) max_blocks = 1;
  if (nq < 1) nq = 1;
  // header (ticket, error word, the one-launch decode step's epoch and
  // arrivals), the one-launch step's tagged keys, then the block scores
  return 256 + align256((size_t)max_blocks * 8) + align256((size_t)max_blocks * nq * sizeof(float));
}

static int select_common(cudaStream_t st, const void* q, int nq, int64_t q_row_stride,
                         int64_t q_head_stride, int hq, int hkv, int head_dim, const void* reps,
                         int r, int max_blocks, int nblocks, const int32_t* protected_ids,
                         int n_protected, int k, void* workspace, size_t workspace_bytes,
                         int per_query, SelectParams& p) {
  NKV_REQUIRE(q && reps && workspace, "select: null pointer");
  NKV_SUPPORTED(head_dim == NKV_D, "select: head_dim %d unsupported (128 only)", head_dim);
  NKV_REQUIRE(hkv > 0 && hq % hkv == 0, "select: hq %d not a multiple of hkv %d", hq, hkv);
  NKV_SUPPORTED(r >= 1 && r <= 8, "select: r=%d unsupported", r);
  NKV_REQUIRE(nblocks >= 1 && nblocks <= max_blocks, "select: nblocks %d out of [1, %d]", nblocks,
              max_blocks);
  NKV_REQUIRE(nq >= 1, "select: nq must be >= 1");
  NKV_REQUIRE(k >= 1 && k <= nblocks, "select: k=%d out of [1, nblocks=%d]", k, nblocks);
  NKV_REQUIRE(n_protected == 0 || protected_ids, "select: protected ids missing");
  NKV_REQUIRE(workspace_bytes >= nkv_select_workspace_bytes(max_blocks, per_query ? nq : 1),
              "select: workspace too small");
  NKV_REQUIRE(((uintptr_t)q & 15) == 0 && ((uintptr_t)reps & 15) == 0 && (q_head_stride % 8) == 0 &&
                  (q_row_stride % 8) == 0,
              "select: q/reps must be 16-byte aligned with strides multiple of 8 elements");
  p = SelectParams{};  // (xs_P = 0: no peer exchange)
  p.q = (const __nv_bfloat16*)q;
  p.q_row_stride = q_row_stride;
  p.q_head_stride = q_head_stride;
  p.nq = nq;
  p.hq = hq;
  p.hkv = hkv;
  p.r = r;
  p.reps = (const __nv_bfloat16*)reps;
  p.max_blocks = max_blocks;
  p.nblocks = nblocks;
  p.protected_ids = protected_ids;
  p.n_protected = n_protected;
  p.k = k;
  p.per_query = per_query;
  p.ticket = (unsigned*)((char*)workspace + 4);
  p.err = (int*)((char*)workspace + 8);
  p.ext_reps = (long long)hkv * max_blocks * r * NKV_D;
  p.ext_q = (nq - 1) * q_row_stride + (hq - 1) * q_head_stride + NKV_D;
  p.trace = nullptr;
#ifdef NKV_CHECKED
  {
    const size_t need = nkv_select_workspace_bytes(max_blocks, per_query ? nq : 1);
    if (workspace_bytes >= need + (1 << 16)) p.trace = (int*)((char*)workspace + workspace_bytes - (1 << 16));
  }
#endif
  p.scores = (float*)((char*)workspace + 256 + align256((size_t)max_blocks * 8));
  return NKV_OK;
}

extern "C" int nkv_select(nkv_stream_t stream, const void* q, int nq, int64_t q_row_stride,
                          int64_t q_head_stride, int hq, int hkv, int head_dim, const void* reps,
                          int r, int max_blocks, int nblocks, const int32_t* protected_ids,
                          int n_protected, int k, int64_t* out_ids, float* out_topk_scores,
                          float* out_block_scores, void* workspace, size_t workspace_bytes) {
  SelectParams p;
  int rc = select_common((cudaStream_t)stream, q, nq, q_row_stride, q_head_stride, hq, hkv,
                         head_dim, reps, r, max_blocks, nblocks, protected_ids, n_protected, k,
                         workspace, workspace_bytes, 0, p);
  if (rc) return rc;
  NKV_REQUIRE(out_ids, "select: out_ids is null");
  NKV_SUPPORTED(k <= 32 || nblocks <= SEL_MAX_SMEM_SORT,
                "select: k > 32 needs nblocks <= %d", SEL_MAX_SMEM_SORT);
  NKV_SUPPORTED(k <= 256, "select: k=%d > 256", k);
  p.out_ids = (long long*)out_ids;
  p.out_topk_scores = out_topk_scores;
  p.out_block_scores = out_block_scores;
  return launch_select((cudaStream_t)stream, p, hq / hkv);
}

namespace nkv {
int select_scores(cudaStream_t st, const void* q, int64_t q_row_stride, int64_t q_head_stride, int hq, int hkv,
                  int head_dim, const void* reps, int r, int max_blocks, int nblocks, const int32_t* protected_ids,
                  int n_protected, int k, void* workspace, size_t workspace_bytes, const float** scores,
                  float* out_block_scores, const PeerArgs* peer) {
  SelectParams p;
  int rc = select_common(st, q, 1, q_row_stride, q_head_stride, hq, hkv, head_dim, reps, r, max_blocks, nblocks,
                         protected_ids, n_protected, k, workspace, workspace_bytes, 0, p);
  if (rc) return rc;
  p.score_only = 1;
  if (peer) {
    NKV_REQUIRE(peer->P >= 1 && peer->P <= NKV_MAX_PEERS && peer->rank >= 0 && peer->rank < peer->P && peer->exch &&
                    nblocks <= peer->cap,
                "select_scores: bad peer exchange (P=%d, rank=%d, cap=%d)", peer->P, peer->rank, peer->cap);
    p.xs_P = peer->P;
    p.xs_rank = peer->rank;
    p.xs_cap = peer->cap;
    p.xs_epoch = (const uint32_t*)peer->exch[peer->rank];
    for (int i = 0; i < peer->P; ++i) {
      NKV_REQUIRE(peer->exch[i] && ((uintptr_t)peer->exch[i] & 15) == 0, "select_scores: exchange %d missing", i);
      p.xs_peer[i] = (u64*)((char*)peer->exch[i] + peer_xs_offset());
    }
  }
  p.out_block_scores = out_block_scores;
  *scores = p.scores;
  return launch_select(st, p, hq / hkv);
}
}  // namespace nkv

extern "C" int nkv_select_per_query(nkv_stream_t stream, const void* q, int nq, int64_t q_row_stride,
                                    int64_t q_head_stride, int hq, int hkv, int head_dim,
                                    const void* reps, int r, int max_blocks, int nblocks,
                                    const int32_t* protected_ids, int n_protected, int k,
                                    int64_t* out_union, int32_t* out_count, uint8_t* out_allowed,
                                    float* out_scores, void* workspace, size_t workspace_bytes) {
  SelectParams p;
  int rc = select_common((cudaStream_t)stream, q, nq, q_row_stride, q_head_stride, hq, hkv,
                         head_dim, reps, r, max_blocks, nblocks, protected_ids, n_protected, k,
                         workspace, workspace_bytes, 1, p);
  if (rc) return rc;
  NKV_REQUIRE(out_union && out_count && out_allowed, "select_per_query: null output");
  NKV_SUPPORTED(nq <= 8 && k <= 32, "select_per_query: needs nq <= 8 and k <= 32");
  NKV_SUPPORTED((size_t)nq * nblocks * 4 <= 200 * 1024, "select_per_query: nq * nblocks too large");
  p.out_union = (long long*)out_union;
  p.out_count = out_count;
  p.out_allowed = out_allowed;
  p.out_block_scores = out_scores;
  return launch_select((cudaStream_t)stream, p, hq / hkv);
}
