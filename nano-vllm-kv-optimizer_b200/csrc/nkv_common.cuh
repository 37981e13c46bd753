// Shared device helpers for the NanoKV B200 kernels (sm_100a).
//
// Layouts used throughout (all row-major, D = head_dim = 128 contiguous):
//   block store   k_store / v_store  [max_blocks][Hkv][B][D]   bf16 (or int8 offload)
//   representatives reps             [Hkv][max_blocks][r][D]   bf16
//   sink window    sink_k / sink_v   [Hkv][S][D]                bf16
//   recent ring    ring_k / ring_v   [Hkv][R][D]                bf16, logical slot i
//                                     lives at physical (head + i) % R
// One (block, kv head) tile of the store is B*D*2 = 16 KiB contiguous, which is
// what lets a single cp.async.bulk move it.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define NKV_D 128

namespace nkv {

typedef unsigned long long u64;
constexpr unsigned FULL = 0xffffffffu;

// ---------------------------------------------------------------------------
// Error word written by kernels into the caller's workspace (bounded waits).
// ---------------------------------------------------------------------------
enum : int {
  ERR_NONE = 0,
  ERR_WAIT_TIMEOUT = 1,  // an mbarrier wait exceeded its iteration budget
  ERR_BAD_INDEX = 2,     // a block id outside [0, nblocks)
  ERR_BOUNDS = 3,        // (checked builds) an access outside its buffer; detail in err[1..3]
};

// Checked builds (-DNKV_CHECKED) verify every global access of the hot kernels
// against the extent of its buffer; a violation records (code, site, offset)
// in the error word and the access is skipped instead of performed.
#ifdef NKV_CHECKED
__device__ __forceinline__ bool nkv_inb(int* err, int site, long long off, long long len, long long ext) {
  if (off >= 0 && off + len <= ext) return true;
  if (err && atomicCAS(err, 0, ERR_BOUNDS) == 0) {
    err[1] = site;
    reinterpret_cast<long long*>(err)[1] = off;
    reinterpret_cast<long long*>(err)[2] = ext;
  }
  return false;
}
#define NKV_INB(err, site, off, len, ext) ::nkv::nkv_inb((err), (site), (long long)(off), (long long)(len), (long long)(ext))
__device__ __forceinline__ unsigned long long nkv_gtime() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
// phase timestamp into a per-CTA trace record (lower 32 bits of ns)
#define NKV_STAMP(trace, slot) do { if ((trace) && threadIdx.x == 0) (trace)[(slot)] = (int)::nkv::nkv_gtime(); } while (0)
#else
#define NKV_INB(err, site, off, len, ext) true
#define NKV_STAMP(trace, slot) do { } while (0)
#endif

// ---------------------------------------------------------------------------
// bf16 helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }
__device__ __forceinline__ void unpack8(const uint4& v, float* f) {
  f[0] = bf_lo(v.x); f[1] = bf_hi(v.x); f[2] = bf_lo(v.y); f[3] = bf_hi(v.y);
  f[4] = bf_lo(v.z); f[5] = bf_hi(v.z); f[6] = bf_lo(v.w); f[7] = bf_hi(v.w);
}
// bf16 pair (low half first) -> float2
__device__ __forceinline__ float2 bf2(uint32_t w) { return make_float2(bf_lo(w), bf_hi(w)); }
// Packed fp32x2 fused multiply-add (Blackwell): two IEEE fmaf in one instruction.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  unsigned long long ra, rb, rc, rd;
  ra = (unsigned long long)__float_as_uint(a.x) | ((unsigned long long)__float_as_uint(a.y) << 32);
  rb = (unsigned long long)__float_as_uint(b.x) | ((unsigned long long)__float_as_uint(b.y) << 32);
  rc = (unsigned long long)__float_as_uint(c.x) | ((unsigned long long)__float_as_uint(c.y) << 32);
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(rd) : "l"(ra), "l"(rb), "l"(rc));
  return make_float2(__uint_as_float((uint32_t)rd), __uint_as_float((uint32_t)(rd >> 32)));
}
__device__ __forceinline__ uint16_t f2bf(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

// ---------------------------------------------------------------------------
// Orderable keys for exact, deterministic top-k.
// key = (orderable(score) << 32) | (0xffffffff - id): a larger key is a higher
// score, and among equal scores the smaller block id.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t f32_order(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float f32_unorder(uint32_t u) {
  return __uint_as_float((u & 0x80000000u) ? (u & 0x7fffffffu) : ~u);
}
// Words exchanged with peer GPUs through their memory (KV-head sharding): a
// 64-bit word carries a 32-bit payload and a 32-bit tag of the step that wrote
// it, so one 8-byte store is both data and flag (a reader polls until the tag
// is the current one).  Volatile accesses: no caching in L1 on either side.
__device__ __forceinline__ void st_peer_u64(u64* a, u64 v) {
  asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(a), "l"(v) : "memory");
}
__device__ __forceinline__ u64 ld_peer_u64(const u64* a) {
  u64 v;
  asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(a) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t ld_peer_u32(const uint32_t* a) {
  uint32_t v;
  asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(v) : "l"(a) : "memory");
  return v;
}
// Tag of the step with epoch e: never 0, so zeroed memory holds no valid word.
__device__ __forceinline__ uint32_t step_tag(uint32_t e) { return e % 0xfffffffeu + 1u; }

__device__ __forceinline__ u64 make_key(float score, uint32_t id) {
  return ((u64)f32_order(score) << 32) | (u64)(0xffffffffu - id);
}
__device__ __forceinline__ uint32_t key_id(u64 k) { return 0xffffffffu - (uint32_t)(k & 0xffffffffu); }
__device__ __forceinline__ float key_score(u64 k) { return f32_unorder((uint32_t)(k >> 32)); }

__device__ __forceinline__ u64 shfl_xor64(u64 v, int m) {
  uint32_t lo = __shfl_xor_sync(FULL, (uint32_t)v, m);
  uint32_t hi = __shfl_xor_sync(FULL, (uint32_t)(v >> 32), m);
  return ((u64)hi << 32) | lo;
}
__device__ __forceinline__ u64 shfl64(u64 v, int src) {
  uint32_t lo = __shfl_sync(FULL, (uint32_t)v, src);
  uint32_t hi = __shfl_sync(FULL, (uint32_t)(v >> 32), src);
  return ((u64)hi << 32) | lo;
}
__device__ __forceinline__ u64 umax64(u64 a, u64 b) { return a > b ? a : b; }
__device__ __forceinline__ u64 umin64(u64 a, u64 b) { return a < b ? a : b; }

// Bitonic sort of one key per lane, descending (lane 0 holds the largest).
__device__ __forceinline__ u64 warp_sort_desc(u64 x) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      u64 y = shfl_xor64(x, j);
      bool lower = (lane & j) == 0;
      bool desc = (lane & k) == 0;
      x = (lower == desc) ? umax64(x, y) : umin64(x, y);
    }
  }
  return x;
}
// Top 32 of two descending warp lists, returned descending.
__device__ __forceinline__ u64 warp_merge_desc(u64 a, u64 b) {
  const int lane = threadIdx.x & 31;
  u64 x = umax64(a, shfl64(b, 31 - lane));  // bitonic: holds top 32 of a U b
#pragma unroll
  for (int j = 16; j > 0; j >>= 1) {
    u64 y = shfl_xor64(x, j);
    x = ((lane & j) == 0) ? umax64(x, y) : umin64(x, y);
  }
  return x;
}

// ---------------------------------------------------------------------------
// mbarrier + bulk async copy (TMA, untiled).  Sizes and addresses must be
// 16-byte multiples / aligned.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// try_wait with a suspend-time hint: the thread sleeps until the phase
// completes or ~hint_ns elapse, instead of spinning on issue slots.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t phase, uint32_t hint_ns = 100000) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(phase), "r"(hint_ns)
      : "memory");
  return ok != 0;
}
// Bounded wait: returns false (and records ERR_WAIT_TIMEOUT) after max_iter
// suspended polls (each at most ~0.1 ms, so ~2 s in total by default).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t phase, int* err,
                                                  long long max_iter = 20000) {
  for (long long i = 0; i < max_iter; ++i)
    if (mbar_try_wait(bar, phase)) return true;
  if (err) atomicExch(err, ERR_WAIT_TIMEOUT);
  return false;
}

// Polled wait (no suspend hint: a suspended thread can wake long after the
// phase completes).  Bounded by ~0.2 s of SM clock; returns false and records
// ERR_WAIT_TIMEOUT when the bound is hit.
__device__ __forceinline__ bool mbar_try_wait_poll(uint64_t* bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(phase)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_poll(uint64_t* bar, uint32_t phase, int* err) {
  if (mbar_try_wait_poll(bar, phase)) return true;
  for (long long t0 = clock64(); clock64() - t0 < 400000000ll;)
    if (mbar_try_wait_poll(bar, phase)) return true;
  if (err) atomicExch(err, ERR_WAIT_TIMEOUT);
  return false;
}

// 16-byte asynchronous global->shared copies (the L1 path); completion is
// tracked per thread by commit groups.
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Programmatic dependent launch: a primary grid lets its dependent start early;
// the dependent waits for the primary's completion before reading its output.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// ---------------------------------------------------------------------------
// Tensor-core helpers (mma.sync m16n8k16, bf16 inputs, fp32 accumulate).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  return (uint32_t)f2bf(lo) | ((uint32_t)f2bf(hi) << 16);
}

// Swizzled tile addressing: a tile of nrows rows of 128 bf16 is stored as two
// 64-column halves [2][nrows][128 B]; 16-byte chunk c of row r sits at chunk
// c ^ (r & 7) (the 128-byte swizzle TMA writes, with 1024-byte aligned tiles).
// Returns the byte offset of element (row, col).
__device__ __forceinline__ uint32_t swz(int nrows, int row, int col) {
  return (uint32_t)((((col >> 6) * nrows + row) << 7) + ((((col & 63) >> 3) ^ (row & 7)) << 4) + ((col & 7) << 1));
}

}  // namespace nkv
