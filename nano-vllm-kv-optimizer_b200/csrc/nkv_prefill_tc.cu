// Kernel (4) on the 5th-generation tensor cores: tcgen05.mma with TMEM
// accumulators, TMA-fed operands.
//
// Same contract as the mma.sync prefill kernel (nkv_prefill.cu): one chunk of
// nq queries (nq == n_cur) attends, per KV head, to its selected blocks, sink,
// recent ring slice and the causal chunk.  Softmax is order-independent, so the
// keys are laid out in 64-key tiles per segment: one tile per selected block
// (block_size 64), one sink tile, the ring slice as its run before and after
// the physical wrap (each padded to whole tiles), then the chunk.  Padding rows
// are masked; every tile is one 64-row TMA box per 64-column half.
//
// CTA = two query tiles of 128 rows (128 / G positions x G heads of one KV head
// each) sharing every K/V tile, 320 threads:
//   warp 0     TMA producer: Q of both tiles once (3D map over [T][hq][D]), K and V of each
//              tile into a 3-stage ring (2D maps over the store, sink and ring,
//              3D maps over the chunk), 128-byte swizzle.
//   warp 1     owns all 512 TMEM columns (per query tile: two S buffers and O)
//              and issues the MMAs from one thread: S_j = Q_t K_j^T for both
//              tiles (M 128, N 64, K 128), then O_t += P_t,{j-1} V_{j-1}
//              (M 128, N 128, K 64; V as an MN-major operand), tcgen05.commit
//              to mbarriers.
//   warps 2-5  query tile 0, warps 6-9 query tile 1, one row (TMEM lane) per
//              thread: S from TMEM, mask, online softmax in the exp2 domain with
//              lazy rescaling of O (only when the row max grows by more than
//              2^8), P as bf16 into a double-buffered swizzled shared tile (the A
//              operand of the next MMA), and the epilogue O / l -> bf16.  The
//              softmax stream is issue-bound, so it is kept short: row max by
//              3-input max, exponent arguments and row sums on packed fp32
//              pairs, ex2.approx on the MUFU unit (moving a share of the
//              exponentials to an FMA-pipe polynomial measured slower).
// Every wait is bounded (error word + fall through); TMEM is freed by warp 1
// after all warps meet at the end.
#include <cuda.h>

#include "nkv_common.cuh"
#include "nkv_host.h"

namespace nkv {

constexpr int TC_THREADS = 320;  // warp 0 TMA, warp 1 MMA + TMEM, warps 2-5 / 6-9 softmax of query tile 0 / 1
constexpr int TC_M = 128;        // rows per query tile
constexpr int TC_QT = 2;         // query tiles per CTA (sharing every K/V tile)
constexpr int TC_N = 64;
constexpr int TC_STAGES = 3;
// TMEM columns: tile t's S buffers at t*128 + {0, 64}, its O at 256 + t*128
constexpr uint32_t TC_TMEM_COLS = 512;
constexpr int TC_Q_BYTES = TC_M * 256;   // per query tile: [2 halves][128 rows][128 B]
constexpr int TC_KV_BYTES = TC_N * 256;  // [2 halves][64 rows][128 B]
constexpr int TC_P_BYTES = TC_M * 128;   // per query tile and buffer: [128 rows][128 B] (64 keys)
constexpr size_t TC_SMEM = 1024 + TC_QT * TC_Q_BYTES + 2 * TC_STAGES * TC_KV_BYTES + TC_QT * 2 * TC_P_BYTES;

struct TcMaps {
  CUtensorMap q, ck, cv;  // 3D: [T][heads][128]
  CUtensorMap ks, vs;     // 2D rows of the block store
  CUtensorMap sk, sv;     // 2D rows of the sink
  CUtensorMap rk, rv;     // 2D rows of the ring
};

struct TcParams {
  int nq, hkv;
  float sl2;  // softmax scale * log2(e)
  const long long* ids;
  int n_sel, max_blocks;
  int sink_len, sink_cap;
  int ring_start, ring_len, ring_cap;
  int n_cur;
  __nv_bfloat16* out;
  long long out_row, out_head;
  int* err;
};

// ---- tcgen05 / TMA wrappers ------------------------------------------------------------
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void tma2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tma3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}
// Shared-memory matrix descriptor, 128-byte swizzle (SM100 version field 1).
// K-major operands: LBO 16 B (unused), SBO = 1024 B between 8-row groups.
// MN-major operands: LBO = bytes between 64-element groups along MN, SBO = 1024 B
// between 8-row groups along K.
__device__ __forceinline__ uint64_t sdesc(const void* p, uint32_t lbo, uint32_t sbo) {
  const uint32_t a = smem_u32(p);
  return (uint64_t)((a >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}
__device__ __forceinline__ void umma(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Bounded wait that fails fast: the first wait to run out (0.2 s) records
// ERR_WAIT_TIMEOUT and raises the CTA's flag, after which every wait returns
// at once, so a broken hand-off ends the kernel instead of stalling it.
__device__ __forceinline__ bool tc_try(uint64_t* bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(phase)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ void tc_wait(uint64_t* bar, uint32_t phase, int* err, volatile int* fail) {
  if (tc_try(bar, phase)) return;
  if (*fail) return;
  for (long long t0 = clock64(); clock64() - t0 < 400000000ll;) {  // ~0.2 s at 2 GHz
    if (tc_try(bar, phase)) return;
    if (*fail) return;
  }
  *fail = 1;
  if (err) atomicExch(err, ERR_WAIT_TIMEOUT);
}

// Bounded wait that ignores the fail flag: used to drain the CTA's own copies
// and MMAs before TMEM is freed and the CTA exits.
__device__ __forceinline__ void tc_drain(uint64_t* bar, uint32_t phase, int* err) {
  for (int i = 0; i < 2000; ++i)
    if (mbar_try_wait(bar, phase)) return;
  if (err) atomicExch(err, ERR_WAIT_TIMEOUT);
}

// ---- the key tiles of a CTA --------------------------------------------------------------
// Tile order: selected blocks [0, n_sel) | sink (when sink_len > 0) | ring run
// before the wrap | ring run after it | chunk tiles.  src: 0 store, 1 sink,
// 2 ring, 3 chunk.  y: first source row (2D maps) or first chunk position.
struct Tile {
  int src, y, valid;
};
__device__ __forceinline__ Tile tile_of(const TcParams& p, int h, int j, int lenA, int nA, int nB,
                                        bool rows = true) {
  Tile t;
  t.valid = TC_N;
  if (j < p.n_sel) {
    t.src = 0;
    t.y = 0;
    if (!rows) return t;  // the softmax threads need only the kind of tile
    long long id = __ldg(p.ids + j);
    if (id < 0 || id >= p.max_blocks) {
      if (p.err) atomicExch(p.err, ERR_BAD_INDEX);
      id = 0;
    }
    t.src = 0;
    t.y = (int)((id * p.hkv + h) * TC_N);
    return t;
  }
  j -= p.n_sel;
  if (p.sink_len > 0) {
    if (j == 0) {
      t.src = 1;
      t.y = h * p.sink_cap;
      t.valid = p.sink_len;
      return t;
    }
    --j;
  }
  if (j < nA) {
    t.src = 2;
    t.y = h * p.ring_cap + p.ring_start + j * TC_N;
    t.valid = min(TC_N, lenA - j * TC_N);
    return t;
  }
  j -= nA;
  if (j < nB) {
    t.src = 2;
    t.y = h * p.ring_cap + j * TC_N;
    t.valid = min(TC_N, (p.ring_len - lenA) - j * TC_N);
    return t;
  }
  j -= nB;
  t.src = 3;
  t.y = j * TC_N;
  return t;
}

// Three-input maximum (one instruction on sm_100a) and packed fp32 pairs.
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
// 2^x with the MUFU instruction alone (subnormal results flush to zero: such
// terms are below 2^-126 of the row maximum's).
__device__ __forceinline__ float ex2_mufu(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
  unsigned long long ra = (unsigned long long)__float_as_uint(a.x) | ((unsigned long long)__float_as_uint(a.y) << 32);
  unsigned long long rb = (unsigned long long)__float_as_uint(b.x) | ((unsigned long long)__float_as_uint(b.y) << 32);
  unsigned long long rd;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(rd) : "l"(ra), "l"(rb));
  return make_float2(__uint_as_float((uint32_t)rd), __uint_as_float((uint32_t)(rd >> 32)));
}

template <int G>
__global__ void __launch_bounds__(TC_THREADS, 1) prefill_tc_kernel(const TcParams p, const __grid_constant__ TcMaps tm) {
  extern __shared__ __align__(16) unsigned char sm_raw[];
  // [query tile][buffer] where two buffers alternate by key tile.  Every
  // barrier a side can run ahead on is one per buffer: the softmax threads may
  // publish P of tile j+1 before the MMA thread has waited for tile j's, and a
  // single P barrier would then be two phases ahead of that wait (its parity
  // would alias and the wait would miss the completed phase).
  __shared__ __align__(8) uint64_t q_full, kv_full[TC_STAGES], kv_empty[TC_STAGES], s_full[TC_QT][2],
      s_free[TC_QT][2], p_full[TC_QT][2], o_done[TC_QT][2], fin;
  __shared__ uint32_t s_tmem;
  __shared__ volatile int s_fail;
  unsigned char* sm = sm_raw + ((1024u - (smem_u32(sm_raw) & 1023u)) & 1023u);
  unsigned char* qs = sm;                                  // [tile] x TC_Q_BYTES
  unsigned char* ks = qs + TC_QT * TC_Q_BYTES;
  unsigned char* vs = ks + TC_STAGES * TC_KV_BYTES;
  unsigned char* ps = vs + TC_STAGES * TC_KV_BYTES;        // [tile][buffer] x TC_P_BYTES
  constexpr int P = TC_M / G;  // positions per query tile

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // grid (heads, position tiles), heads fastest: CTAs start in order of
  // decreasing work (the latest positions attend the most causal keys) across
  // all heads, so the last wave holds the lightest tiles
  const int h = blockIdx.x;
  const int p0 = ((int)gridDim.y - 1 - (int)blockIdx.y) * (TC_QT * P);  // latest positions first
  const int off = p.n_cur - p.nq;
  const int last_pos = min(p.nq, p0 + TC_QT * P) - 1;
  const int lenA = min(p.ring_len, p.ring_cap - p.ring_start);
  const int nA = (lenA + TC_N - 1) / TC_N, nB = (p.ring_len - lenA + TC_N - 1) / TC_N;
  const int nhist = p.n_sel + (p.sink_len > 0 ? 1 : 0) + nA + nB;
  const int nct = (min(p.n_cur, last_pos + off + 1) + TC_N - 1) / TC_N;
  const int ntiles = nhist + nct;

  if (threadIdx.x == 0) {
    s_fail = 0;
    mbar_init(&q_full, 1);
    for (int s = 0; s < TC_STAGES; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int t = 0; t < TC_QT; ++t) {
      for (int b = 0; b < 2; ++b) {
        mbar_init(&s_full[t][b], 1);
        mbar_init(&s_free[t][b], 128);
        mbar_init(&o_done[t][b], 1);
        mbar_init(&p_full[t][b], 128);
      }
    }
    mbar_init(&fin, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                 "r"(TC_TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = s_tmem;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      mbar_expect_tx(&q_full, TC_QT * TC_Q_BYTES);
      for (int t = 0; t < TC_QT; ++t) {
        tma3d(qs + t * TC_Q_BYTES, &tm.q, 0, h * G, p0 + t * P, &q_full);
        tma3d(qs + t * TC_Q_BYTES + TC_M * 128, &tm.q, 64, h * G, p0 + t * P, &q_full);
      }
      for (int j = 0; j < ntiles; ++j) {
        const int st = j % TC_STAGES;
        if (j >= TC_STAGES) tc_wait(&kv_empty[st], ((j / TC_STAGES) - 1) & 1, p.err, &s_fail);
        mbar_expect_tx(&kv_full[st], 2 * TC_KV_BYTES);
        const Tile t = tile_of(p, h, j, lenA, nA, nB);
        unsigned char* kd = ks + st * TC_KV_BYTES;
        unsigned char* vd = vs + st * TC_KV_BYTES;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          if (t.src == 3) {
            tma3d(kd + half * (TC_N * 128), &tm.ck, half * 64, h, t.y, &kv_full[st]);
            tma3d(vd + half * (TC_N * 128), &tm.cv, half * 64, h, t.y, &kv_full[st]);
          } else {
            const CUtensorMap* km = t.src == 0 ? &tm.ks : t.src == 1 ? &tm.sk : &tm.rk;
            const CUtensorMap* vm = t.src == 0 ? &tm.vs : t.src == 1 ? &tm.sv : &tm.rv;
            tma2d(kd + half * (TC_N * 128), km, half * 64, t.y, &kv_full[st]);
            tma2d(vd + half * (TC_N * 128), vm, half * 64, t.y, &kv_full[st]);
          }
        }
      }
      // drain: the last copies of every stage have landed
      tc_drain(&q_full, 0, p.err);
      for (int j = ntiles - TC_STAGES < 0 ? 0 : ntiles - TC_STAGES; j < ntiles; ++j)
        tc_drain(&kv_full[j % TC_STAGES], (j / TC_STAGES) & 1, p.err);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer: S of both query tiles, then their P.V ----------------
    if (lane == 0) {
      // f32 accumulate, bf16 A and B; S: K-major A and B, N 64; O: MN-major B (V), N 128; M 128
      constexpr uint32_t ID_S = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(TC_N >> 3) << 17) |
                                ((uint32_t)(TC_M >> 4) << 24);
      constexpr uint32_t ID_O = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 16) | ((uint32_t)(128 >> 3) << 17) |
                                ((uint32_t)(TC_M >> 4) << 24);
      tc_wait(&q_full, 0, p.err, &s_fail);
      for (int j = 0; j <= ntiles; ++j) {
        if (j < ntiles) {
          const int st = j % TC_STAGES, sb = j & 1;
          tc_wait(&kv_full[st], (j / TC_STAGES) & 1, p.err, &s_fail);
          const unsigned char* kt = ks + st * TC_KV_BYTES;
#pragma unroll
          for (int t = 0; t < TC_QT; ++t) {
            if (j >= 2) tc_wait(&s_free[t][sb], ((j >> 1) - 1) & 1, p.err, &s_fail);
            tc_fence_after();
            const unsigned char* qt = qs + t * TC_Q_BYTES;
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const uint64_t a = sdesc(qt + (k >> 2) * (TC_M * 128) + (k & 3) * 32, 16, 1024);
              const uint64_t b = sdesc(kt + (k >> 2) * (TC_N * 128) + (k & 3) * 32, 16, 1024);
              umma(tbase + t * 128 + sb * TC_N, a, b, ID_S, k > 0 ? 1u : 0u);
            }
            umma_commit(&s_full[t][sb]);
          }
        }
        if (j >= 1) {
          const int jj = j - 1, st = jj % TC_STAGES;
          const unsigned char* vt = vs + st * TC_KV_BYTES;
#pragma unroll
          for (int t = 0; t < TC_QT; ++t) {
            tc_wait(&p_full[t][jj & 1], (jj >> 1) & 1, p.err, &s_fail);
            tc_fence_after();
            const unsigned char* pt = ps + (t * 2 + (jj & 1)) * TC_P_BYTES;
#pragma unroll
            for (int k = 0; k < TC_N / 16; ++k) {
              const uint64_t a = sdesc(pt + k * 32, 16, 1024);
              const uint64_t b = sdesc(vt + k * 16 * 128, TC_N * 128, 1024);
              umma(tbase + 256 + t * 128, a, b, ID_O, (jj > 0 || k > 0) ? 1u : 0u);
            }
            umma_commit(&o_done[t][jj & 1]);
          }
          umma_commit(&kv_empty[st]);
        }
      }
      // drain: every MMA of this thread has completed (and its commits landed)
      umma_commit(&fin);
      tc_drain(&fin, 0, p.err);
    }
    __syncwarp();
  } else {
    // ---------------- softmax / correction / epilogue ----------------
    // warps 2-5 own query tile 0, warps 6-9 tile 1; one row (TMEM lane) per thread
    const int t = (warp - 2) >> 2;
    const int q4 = warp & 3;
    const int row = q4 * 32 + lane;
    const uint32_t trow = tbase + ((uint32_t)(q4 * 32) << 16);
    const uint32_t s_col = t * 128, o_col = 256 + t * 128;
    const int tp0 = p0 + t * P;  // first position of this query tile
    const int pos = tp0 + row / G, g = row % G;
    float m_ref = -INFINITY, l = 0.f;
    for (int j = 0; j < ntiles; ++j) {
      const int sb = j & 1;
      tc_wait(&s_full[t][sb], (j >> 1) & 1, p.err, &s_fail);
      __syncwarp();  // the TMEM loads below are warp-collective
      tc_fence_after();
      uint32_t sr[64];
      {
        uint32_t (&lo)[32] = *reinterpret_cast<uint32_t(*)[32]>(sr);
        uint32_t (&hi)[32] = *reinterpret_cast<uint32_t(*)[32]>(sr + 32);
        tmem_ld32(trow + s_col + sb * TC_N, lo);
        tmem_ld32(trow + s_col + sb * TC_N + 32, hi);
      }
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&s_free[t][sb]);
      const Tile ti = tile_of(p, 0, j, lenA, nA, nB, false);  // only src / valid / chunk base are used
      // masking only where a tile has padding rows or chunk keys past the
      // tile's first position; the scale is applied inside the exponent
      const bool need_mask = ti.src == 3 ? (ti.y + TC_N - 1 > tp0 + off) : (ti.valid < TC_N);
      if (need_mask) {
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          const bool vis = ti.src == 3 ? (ti.y + c <= pos + off) : (c < ti.valid);
          if (!vis) sr[c] = __float_as_uint(-INFINITY);
        }
      }
      // row max: 8 independent partial maxima, two new columns per 3-input max
      float mp[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) mp[u] = fmaxf(__uint_as_float(sr[2 * u]), __uint_as_float(sr[2 * u + 1]));
#pragma unroll
      for (int c = 16; c < 64; c += 2)
        mp[(c >> 1) & 7] = fmax3(mp[(c >> 1) & 7], __uint_as_float(sr[c]), __uint_as_float(sr[c + 1]));
      const float mxr = fmax3(fmax3(mp[0], mp[1], mp[2]), fmax3(mp[3], mp[4], mp[5]), fmaxf(mp[6], mp[7]));
      const float m_new = fmaxf(m_ref, mxr * p.sl2);
      const bool rescale = m_new > m_ref + 8.f;
      // P buffer j % 2 is free once PV_{j-2} is done; O is current once PV_{j-1} is
      if (j >= 2) tc_wait(&o_done[t][j & 1], ((j - 2) >> 1) & 1, p.err, &s_fail);
      // O and l hold partial sums at the old reference: rows whose maximum grew
      // rescale them.  tcgen05.ld/st are warp-collective (.sync.aligned), so the
      // whole warp takes the TMEM round trip when any of its rows needs it; the
      // other rows scale by 1.
      const bool own = rescale && m_ref != -INFINITY;
      if (__any_sync(0xffffffffu, own)) {
        tc_wait(&o_done[t][(j - 1) & 1], ((j - 1) >> 1) & 1, p.err, &s_fail);
        __syncwarp();
        const float alpha = own ? exp2f(m_ref - m_new) : 1.f;
        tc_fence_after();
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          uint32_t o[32];
          tmem_ld32(trow + o_col + cc * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_st32(trow + o_col + cc * 32, o);
        }
        tmem_wait_st();
        l *= alpha;
      }
      if (rescale) m_ref = m_new;
      const float nbase = m_ref == -INFINITY ? 0.f : -m_ref;
      uint32_t pw[32];
      // exponent arguments and row sums on packed fp32 pairs (4 independent sum chains)
      float2 lp[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
      const float2 sl2 = make_float2(p.sl2, p.sl2), nb2 = make_float2(nbase, nbase);
#pragma unroll
      for (int c = 0; c < 64; c += 2) {
        const float2 x = ffma2(make_float2(__uint_as_float(sr[c]), __uint_as_float(sr[c + 1])), sl2, nb2);
        const float2 e = make_float2(ex2_mufu(x.x), ex2_mufu(x.y));
        lp[(c >> 1) & 3] = fadd2(lp[(c >> 1) & 3], e);
        const __nv_bfloat162 hb = __floats2bfloat162_rn(e.x, e.y);
        pw[c / 2] = *reinterpret_cast<const uint32_t*>(&hb);
      }
      l += ((lp[0].x + lp[0].y) + (lp[1].x + lp[1].y)) + ((lp[2].x + lp[2].y) + (lp[3].x + lp[3].y));
      unsigned char* prow = ps + (t * 2 + (j & 1)) * TC_P_BYTES + row * 128;
#pragma unroll
      for (int ch = 0; ch < 8; ++ch)
        *reinterpret_cast<uint4*>(prow + ((ch ^ (row & 7)) << 4)) =
            make_uint4(pw[ch * 4], pw[ch * 4 + 1], pw[ch * 4 + 2], pw[ch * 4 + 3]);
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full[t][j & 1]);
    }
    // epilogue: O / l -> bf16
    if (ntiles > 0) tc_wait(&o_done[t][(ntiles - 1) & 1], ((ntiles - 1) >> 1) & 1, p.err, &s_fail);
    __syncwarp();
    tc_fence_after();
    const float inv = 1.f / l;
    __nv_bfloat16* dst = p.out + (long long)pos * p.out_row + (long long)(h * G + g) * p.out_head;
#pragma unroll
    for (int cc = 0; cc < 4; ++cc) {
      uint32_t o[32];
      tmem_ld32(trow + o_col + cc * 32, o);
      tmem_wait_ld();
      if (pos < p.nq) {
#pragma unroll
        for (int e = 0; e < 32; e += 8) {
          uint4 w;
          w.x = pack_bf16x2(__uint_as_float(o[e]) * inv, __uint_as_float(o[e + 1]) * inv);
          w.y = pack_bf16x2(__uint_as_float(o[e + 2]) * inv, __uint_as_float(o[e + 3]) * inv);
          w.z = pack_bf16x2(__uint_as_float(o[e + 4]) * inv, __uint_as_float(o[e + 5]) * inv);
          w.w = pack_bf16x2(__uint_as_float(o[e + 6]) * inv, __uint_as_float(o[e + 7]) * inv);
          *reinterpret_cast<uint4*>(dst + cc * 32 + e) = w;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase), "r"(TC_TMEM_COLS) : "memory");
}

// ---- host ------------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFnTc)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
static EncodeTiledFnTc encode_fn_tc() {
  static EncodeTiledFnTc fn = []() -> EncodeTiledFnTc {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      f = nullptr;
    cudaGetLastError();
    return reinterpret_cast<EncodeTiledFnTc>(f);
  }();
  return fn;
}

static bool is_device_memory(const void* p) {
  cudaPointerAttributes pa;
  const bool ok = cudaPointerGetAttributes(&pa, p) == cudaSuccess && pa.type == cudaMemoryTypeDevice;
  cudaGetLastError();
  return ok;
}

// 2D map over `rows` rows of 128 bf16, 64 x 64 boxes, 128-byte swizzle.
static bool map_rows64(CUtensorMap* m, const void* base, long long rows) {
  EncodeTiledFnTc fn = encode_fn_tc();
  if (!fn || !base || rows < 64 || rows >= (1ll << 31) || ((uintptr_t)base & 15) || !is_device_memory(base))
    return false;
  const cuuint64_t dims[2] = {128, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {256};
  const cuuint32_t box[2] = {64, 64};
  const cuuint32_t es[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 3D map over [T][heads][128] bf16 with element strides (row, head), boxes of
// 64 columns x bh heads x bt rows, 128-byte swizzle.
static bool map_3d(CUtensorMap* m, const void* base, int T, int heads, long long row_stride, long long head_stride,
                   int bh, int bt) {
  EncodeTiledFnTc fn = encode_fn_tc();
  if (!fn || !base || T < 1 || ((uintptr_t)base & 15) || (row_stride % 8) || (head_stride % 8) || !is_device_memory(base))
    return false;
  const cuuint64_t dims[3] = {128, (cuuint64_t)heads, (cuuint64_t)T};
  const cuuint64_t strides[2] = {(cuuint64_t)head_stride * 2, (cuuint64_t)row_stride * 2};
  const cuuint32_t box[3] = {64, (cuuint32_t)bh, (cuuint32_t)bt};
  const cuuint32_t es[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Launches the tcgen05 kernel when the call fits it (bf16 history in device
// memory, block_size 64, TMA-addressable sources); returns NKV_ERR_UNSUPPORTED
// without launching otherwise, so that the caller takes the mma.sync kernel.
int prefill_tc(cudaStream_t st, const nkv_attend_args* a) {
  const int G = a->hq / a->hkv;
  if (a->block_size != 64 || (a->n_sel > 0 && a->store_kind != NKV_STORE_BF16) || a->allowed) return NKV_ERR_UNSUPPORTED;
  if (((uintptr_t)a->out & 15) || a->out_row_stride % 8 || a->out_head_stride % 8) return NKV_ERR_UNSUPPORTED;
  TcMaps m;
  memset(&m, 0, sizeof(m));
  if (!map_3d(&m.q, a->q, a->nq, a->hq, a->q_row_stride, a->q_head_stride, G, TC_M / G)) return NKV_ERR_UNSUPPORTED;
  if (!map_3d(&m.ck, a->cur_k, a->n_cur, a->hkv, a->cur_row_stride, a->cur_head_stride, 1, TC_N) ||
      !map_3d(&m.cv, a->cur_v, a->n_cur, a->hkv, a->cur_row_stride, a->cur_head_stride, 1, TC_N))
    return NKV_ERR_UNSUPPORTED;
  if (a->n_sel > 0) {
    const long long rows = (long long)a->max_blocks * a->hkv * 64;
    if (!map_rows64(&m.ks, a->k_store, rows) || !map_rows64(&m.vs, a->v_store, rows)) return NKV_ERR_UNSUPPORTED;
  }
  if (a->sink_len > 0) {
    const long long rows = (long long)a->hkv * a->sink_cap;
    if (!map_rows64(&m.sk, a->sink_k, rows) || !map_rows64(&m.sv, a->sink_v, rows)) return NKV_ERR_UNSUPPORTED;
  }
  if (a->ring_len > 0) {
    const long long rows = (long long)a->hkv * a->ring_cap;
    if (!map_rows64(&m.rk, a->ring_k, rows) || !map_rows64(&m.rv, a->ring_v, rows)) return NKV_ERR_UNSUPPORTED;
  }
  TcParams p;
  p.nq = a->nq;
  p.hkv = a->hkv;
  p.sl2 = a->scale * 1.4426950408889634f;
  p.ids = (const long long*)a->block_ids;
  p.n_sel = a->n_sel;
  p.max_blocks = a->max_blocks;
  p.sink_len = a->sink_len;
  p.sink_cap = a->sink_cap;
  p.ring_start = a->ring_start;
  p.ring_len = a->ring_len;
  p.ring_cap = a->ring_cap;
  p.n_cur = a->n_cur;
  p.out = (__nv_bfloat16*)a->out;
  p.out_row = a->out_row_stride;
  p.out_head = a->out_head_stride;
  p.err = (int*)a->workspace;
  const int P = TC_QT * TC_M / G;  // positions per CTA
  dim3 grid(a->hkv, (a->nq + P - 1) / P);
  switch (G) {
#define NKV_TC_CASE(GG)                                                                \
  case GG:                                                                             \
    if (ensure_smem(prefill_tc_kernel<GG>, TC_SMEM, "prefill_tc")) return NKV_ERR_CUDA; \
    prefill_tc_kernel<GG><<<grid, TC_THREADS, TC_SMEM, st>>>(p, m);                    \
    break;
    NKV_TC_CASE(1)
    NKV_TC_CASE(2)
    NKV_TC_CASE(4)
    NKV_TC_CASE(8)
#undef NKV_TC_CASE
    default:
      return NKV_ERR_UNSUPPORTED;
  }
  return check_launch("prefill_tc");
}

}  // namespace nkv
