// Host-side helpers shared by the C-ABI entry points: status codes, the
// thread-local error message, launch-shape queries.
#pragma once
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>

#include "../../include/nanokv.h"

namespace nkv {

constexpr int NKV_MAX_PEERS = 8;  // ranks of a KV-head-sharded layer exchanging through peer memory

void set_error(const char* fmt, ...);

// Integer tuning knob from the environment (NKV_*): `dflt` when unset or
// empty.  Read once per thread and cached; nkv_reload_env() makes every thread
// read the environment again.
int knob(const char* name, int dflt);

inline int sm_count() {
  static thread_local int cached_dev = -1, cached = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev != cached_dev) {
    cudaDeviceGetAttribute(&cached, cudaDevAttrMultiProcessorCount, dev);
    cached_dev = dev;
  }
  return cached > 0 ? cached : 148;
}

inline int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: launch failed: %s", what, cudaGetErrorString(e));
    return NKV_ERR_CUDA;
  }
  return NKV_OK;
}

// Raise a kernel's dynamic shared-memory limit to `bytes` (cached per kernel,
// device and size).  Returns NKV_OK or NKV_ERR_CUDA with a message.
template <typename Kernel>
inline int ensure_smem(Kernel kernel, size_t bytes, const char* what) {
  if (bytes <= 48 * 1024) return 0;
  struct Entry { const void* fn; int dev; size_t bytes; };
  static thread_local Entry cache[64];
  static thread_local int used = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  const void* fn = reinterpret_cast<const void*>(kernel);
  int slot = -1;
  for (int i = 0; i < used; ++i)
    if (cache[i].fn == fn && cache[i].dev == dev) slot = i;
  if (slot >= 0 && cache[slot].bytes >= bytes) return 0;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error("%s: cannot reserve %zu bytes of shared memory: %s", what, bytes, cudaGetErrorString(e));
    return -3;
  }
  if (slot < 0 && used < 64) slot = used++;
  if (slot >= 0) cache[slot] = Entry{fn, dev, bytes};
  return 0;
}

// Allow clusters above the portable size of 8 for `kernel` (once per device).
template <typename Kernel>
inline int ensure_nonportable_cluster(Kernel kernel, const char* what) {
  struct Entry { const void* fn; int dev; };
  static thread_local Entry cache[32];
  static thread_local int used = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  const void* fn = reinterpret_cast<const void*>(kernel);
  for (int i = 0; i < used; ++i)
    if (cache[i].fn == fn && cache[i].dev == dev) return 0;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error("%s: cluster size above 8 not available: %s", what, cudaGetErrorString(e));
    return -3;
  }
  if (used < 32) cache[used++] = Entry{fn, dev};
  return 0;
}

// Internal launchers of the fused decode step (nkv_decode_step).
// select_scores: the scoring half of nkv_select for one query row; writes the
// protected-masked block scores into the select workspace (and to
// out_block_scores when given) and returns the workspace copy's address (the
// grid signals programmatic dependents at its start).
// KV-head sharding over peer memory: the P ranks' exchange buffers (one per
// layer and rank, each readable and writable by every rank), laid out as
//   [0, 256)  epoch (u32), ticket (u32) of this rank
//   xs        [2 parities][P ranks][cap blocks] u64 tagged block scores
//   xo        [2 parities][hq_all * D / 2] u64 tagged bf16 output pairs
// A step writes the parity and tag of its epoch; the attention grid advances
// the epoch once every one of its readers is done.
struct PeerArgs {
  void* const* exch;  // P device pointers, index = rank
  int P, rank;
  int cap;     // block capacity of the score area
  int hq_all;  // query heads over all ranks
};
inline size_t peer_xs_offset() { return 256; }
inline size_t peer_xo_offset(int P, int cap) { return 256 + (size_t)2 * P * cap * 8; }
inline size_t peer_exchange_bytes(int P, int cap, int hq_all) {
  return peer_xo_offset(P, cap) + (size_t)2 * hq_all * 64 * 8;  // head_dim 128: 64 pairs per row
}

int select_scores(cudaStream_t st, const void* q, int64_t q_row_stride, int64_t q_head_stride, int hq, int hkv,
                  int head_dim, const void* reps, int r, int max_blocks, int nblocks, const int32_t* protected_ids,
                  int n_protected, int k, void* workspace, size_t workspace_bytes, const float** scores,
                  float* out_block_scores, const PeerArgs* peer = nullptr);
// attend_ranked: nkv_attend for one query whose CTAs rank the block scores of
// a preceding select_scores themselves (top args->n_sel), after waiting for it.
// The ranked ids (and scores, when out_scores != NULL) are written to out_ids.
// With ring_head != NULL the recent ring's head is device-resident (see
// nkv_decode_args.ring_head).
int attend_ranked(nkv_stream_t stream, const nkv_attend_args* args, const float* scores, int nblocks,
                  int64_t* out_ids, float* out_scores, const PeerArgs* peer = nullptr, void* out_full = nullptr,
                  int32_t* ring_head = nullptr);
// attend_step: the whole decode step (scoring of every block, protection,
// top args->n_sel selection, attention) as one cooperative cluster launch.
// The keys it publishes live in the select workspace, which must start at
// zero and belong to one stream.  Returns FS_DECLINED, with nothing launched,
// where the configuration is outside it (the caller then runs select_scores +
// attend_ranked).
constexpr int FS_DECLINED = 1;
// ring_head: a device-resident recent-ring head (graph replay) or null;
// split_only: launch only the fused tile-split kernel (FS_DECLINED where it
// does not apply), not the cooperative one-launch decode kernel.
int attend_step(nkv_stream_t stream, const nkv_attend_args* args, const void* reps, int r, int reps_blocks,
                int nblocks, const int32_t* protected_ids, int n_protected, void* select_workspace,
                size_t select_workspace_bytes, int64_t* out_ids, float* out_scores, int32_t* ring_head,
                int split_only);

// prefill_tc: kernel (4) on tcgen05/TMEM for the calls it supports (bf16
// history in device memory, block_size 64, TMA-addressable tensors); returns
// NKV_ERR_UNSUPPORTED without launching for the others.
int prefill_tc(cudaStream_t st, const nkv_attend_args* args);

}  // namespace nkv

#define NKV_REQUIRE(cond, ...)              \
  do {                                      \
    if (!(cond)) {                          \
      ::nkv::set_error(__VA_ARGS__);        \
      return NKV_ERR_ARG;                   \
    }                                       \
  } while (0)

#define NKV_SUPPORTED(cond, ...)            \
  do {                                      \
    if (!(cond)) {                          \
      ::nkv::set_error(__VA_ARGS__);        \
      return NKV_ERR_UNSUPPORTED;           \
    }                                       \
  } while (0)
