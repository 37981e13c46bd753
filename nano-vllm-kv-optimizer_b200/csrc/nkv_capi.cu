// C-ABI plumbing shared by all entry points: error message, version, and the
// read-back of the error word kernels leave in a workspace.
#include <stdarg.h>
#include <stdlib.h>
#include <stdio.h>
#include <string.h>

#include <atomic>

#include "nkv_host.h"

namespace nkv {
static thread_local char g_err[512] = "";
void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}
}  // namespace nkv

namespace nkv {
static std::atomic<unsigned> g_env_gen{1};
int knob(const char* name, int dflt) {
  struct Entry { const char* name; int dflt, value; };
  static thread_local Entry cache[32];
  static thread_local int used = 0;
  static thread_local unsigned gen = 0;
  const unsigned g = g_env_gen.load(std::memory_order_relaxed);
  if (gen != g) {
    used = 0;
    gen = g;
  }
  for (int i = 0; i < used; ++i)
    if (cache[i].name == name && cache[i].dflt == dflt) return cache[i].value;
  const char* v = getenv(name);
  const int value = (v && *v) ? atoi(v) : dflt;
  if (used < 32) cache[used++] = Entry{name, dflt, value};
  return value;
}
}  // namespace nkv

extern "C" void nkv_reload_env(void) { nkv::g_env_gen.fetch_add(1, std::memory_order_relaxed); }

extern "C" const char* nkv_last_error(void) { return nkv::g_err; }

extern "C" int nkv_version(void) { return 1; }

extern "C" int nkv_check(nkv_stream_t stream, void* workspace) {
  NKV_REQUIRE(workspace, "check: null workspace");
  int word = 0;
  cudaError_t e = cudaMemcpyAsync(&word, workspace, sizeof(int), cudaMemcpyDeviceToHost,
                                  (cudaStream_t)stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize((cudaStream_t)stream);
  if (e != cudaSuccess) {
    nkv::set_error("check: %s", cudaGetErrorString(e));
    return NKV_ERR_CUDA;
  }
  if (word != 0) {
    const int zero = 0;
    cudaMemcpyAsync(workspace, &zero, sizeof(int), cudaMemcpyHostToDevice, (cudaStream_t)stream);
    cudaStreamSynchronize((cudaStream_t)stream);
    nkv::set_error("check: kernel error word %d (%s)", word,
                   word == 1 ? "bounded wait timed out" : word == 2 ? "block id out of range" : "?");
    return NKV_ERR_DEVICE;
  }
  return NKV_OK;
}

extern "C" int nkv_map_host(void* host_ptr, void** dev_ptr) {
  NKV_REQUIRE(host_ptr && dev_ptr, "map_host: null pointer");
  cudaError_t e = cudaHostGetDevicePointer(dev_ptr, host_ptr, 0);
  if (e != cudaSuccess) {
    cudaGetLastError();
    nkv::set_error("map_host: %p is not mapped pinned memory: %s", host_ptr, cudaGetErrorString(e));
    return NKV_ERR_ARG;
  }
  return NKV_OK;
}

static thread_local int g_decode_form = 0;
extern "C" int nkv_decode_last_form(void) { return g_decode_form; }

extern "C" int nkv_decode_step(nkv_stream_t stream, const nkv_decode_args* a) {
  NKV_REQUIRE(a, "decode_step: null args");
  const nkv_attend_args& t = a->attend;
  NKV_REQUIRE(t.nq == 1 && t.n_cur == 1, "decode_step: needs one query and one current token");
  // one launch (NKV_DECODE_ONE=1): the attention grid scores and selects the
  // blocks itself; falls through where it does not apply.  Off by default:
  // on B200 at 32K it measured 16.7 us per layer against 14.9 us for the two
  // launches below (its in-CTA scoring and selection take longer than the
  // scoring grid and the launch it saves).
  if (nkv::knob("NKV_DECODE_ONE", 0) != 0 && !a->ring_head) {
    nkv_attend_args b = t;
    b.block_ids = a->out_ids;
    b.n_sel = a->k;
    b.overlap_select = 0;
    const int rc = nkv::attend_step(stream, &b, a->reps, a->r, a->reps_blocks, a->nblocks, a->protected_ids,
                                    a->n_protected, a->select_workspace, a->select_workspace_bytes, a->out_ids,
                                    a->out_topk_scores, nullptr, 0);
    if (rc != nkv::FS_DECLINED) {
      g_decode_form = 1;
      return rc;
    }
  }
  // one launch of the tile-split kernel with the scoring inside (bf16 block
  // store in device memory, 64-token blocks, G = 4, k <= 32); NKV_DECODE_SPLIT=0
  // or a call outside that cover takes the two launches below
  if (nkv::knob("NKV_DECODE_SPLIT", 1) != 0 && nkv::knob("NKV_SPLIT_FUSED", 0) != 0 && a->k <= 32 &&
      a->nblocks <= 2048) {
    nkv_attend_args b = t;
    b.block_ids = a->out_ids;
    b.n_sel = a->k;
    b.overlap_select = nkv::knob("NKV_PDL", 1) != 0 ? 1 : 0;
    const int rc = nkv::attend_step(stream, &b, a->reps, a->r, a->reps_blocks, a->nblocks, a->protected_ids,
                                    a->n_protected, a->select_workspace, a->select_workspace_bytes, a->out_ids,
                                    a->out_topk_scores, a->ring_head, 1);
    if (rc != nkv::FS_DECLINED) {
      g_decode_form = 4;
      return rc;
    }
  }
  // two launches: a scoring grid, then the attention grid ranks the scores in
  // each CTA (no ranking tail between the two); NKV_DECODE_FUSED=0 selects
  // the two public kernels instead
  if (nkv::knob("NKV_DECODE_FUSED", 1) != 0 && a->k <= 32 && a->nblocks <= 2048) {
    const float* scores = nullptr;
    int rc = nkv::select_scores((cudaStream_t)stream, t.q, t.q_row_stride, t.q_head_stride, t.hq, t.hkv, t.head_dim,
                                a->reps, a->r, a->reps_blocks, a->nblocks, a->protected_ids, a->n_protected, a->k,
                                a->select_workspace, a->select_workspace_bytes, &scores, nullptr);
    if (rc != NKV_OK) return rc;
    nkv_attend_args b = t;
    b.block_ids = a->out_ids;
    b.n_sel = a->k;
    b.overlap_select = nkv::knob("NKV_PDL", 1) != 0 ? 1 : 0;  // NKV_PDL=0: plain stream order (measurement)
    g_decode_form = 2;
    return nkv::attend_ranked(stream, &b, scores, a->nblocks, a->out_ids, a->out_topk_scores, nullptr, nullptr,
                              a->ring_head);
  }
  NKV_SUPPORTED(!a->ring_head, "decode_step: a device ring head needs the two-launch form (k <= 32, nblocks <= 2048)");
  int rc = nkv_select(stream, t.q, 1, t.q_row_stride, t.q_head_stride, t.hq, t.hkv, t.head_dim, a->reps, a->r,
                      a->reps_blocks, a->nblocks, a->protected_ids, a->n_protected, a->k, a->out_ids,
                      a->out_topk_scores, nullptr, a->select_workspace, a->select_workspace_bytes);
  if (rc != NKV_OK) return rc;
  nkv_attend_args b = t;
  b.block_ids = a->out_ids;
  b.n_sel = a->k;
  b.overlap_select = 1;
  g_decode_form = 3;
  return nkv_attend(stream, &b);
}

extern "C" int nkv_select_scores(nkv_stream_t stream, const void* q, int64_t q_row_stride, int64_t q_head_stride,
                                 int hq, int hkv, int head_dim, const void* reps, int r, int max_blocks, int nblocks,
                                 const int32_t* protected_ids, int n_protected, float* out_scores, void* workspace,
                                 size_t workspace_bytes) {
  NKV_REQUIRE(out_scores, "select_scores: null out_scores");
  const float* ws_scores = nullptr;
  return nkv::select_scores((cudaStream_t)stream, q, q_row_stride, q_head_stride, hq, hkv, head_dim, reps, r,
                            max_blocks, nblocks, protected_ids, n_protected, 1, workspace, workspace_bytes, &ws_scores,
                            out_scores);
}

extern "C" int nkv_attend_ranked(nkv_stream_t stream, const nkv_attend_args* a, const float* scores, int nblocks,
                                 int64_t* out_ids, float* out_scores) {
  NKV_REQUIRE(a && a->block_ids == out_ids, "attend_ranked: args->block_ids must be out_ids");
  return nkv::attend_ranked(stream, a, scores, nblocks, out_ids, out_scores);
}

// ---- KV-head sharding over peer memory ----------------------------------------------
extern "C" size_t nkv_shard_exchange_bytes(int n_ranks, int max_blocks, int hq_all) {
  if (n_ranks < 1) n_ranks = 1;
  if (max_blocks < 1) max_blocks = 1;
  if (hq_all < 1) hq_all = 1;
  return nkv::peer_exchange_bytes(n_ranks, max_blocks, hq_all);
}

extern "C" int nkv_peer_alloc(size_t bytes, void** dptr, void* ipc_handle) {
  NKV_REQUIRE(dptr && ipc_handle && bytes > 0, "peer_alloc: bad arguments");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e == cudaSuccess) e = cudaMemset(p, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaGetLastError();
    if (p) cudaFree(p);
    nkv::set_error("peer_alloc: %s", cudaGetErrorString(e));
    return NKV_ERR_CUDA;
  }
  memcpy(ipc_handle, &h, sizeof(h));
  *dptr = p;
  return NKV_OK;
}

extern "C" int nkv_peer_open(const void* ipc_handle, void** dptr) {
  NKV_REQUIRE(ipc_handle && dptr, "peer_open: bad arguments");
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(dptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    cudaGetLastError();
    nkv::set_error("peer_open: %s", cudaGetErrorString(e));
    return NKV_ERR_CUDA;
  }
  return NKV_OK;
}

extern "C" int nkv_peer_close(void* dptr) {
  NKV_REQUIRE(dptr, "peer_close: null pointer");
  cudaError_t e = cudaIpcCloseMemHandle(dptr);
  if (e != cudaSuccess) {
    cudaGetLastError();
    nkv::set_error("peer_close: %s", cudaGetErrorString(e));
    return NKV_ERR_CUDA;
  }
  return NKV_OK;
}

extern "C" int nkv_peer_free(void* dptr) {
  NKV_REQUIRE(dptr, "peer_free: null pointer");
  cudaError_t e = cudaFree(dptr);
  if (e != cudaSuccess) {
    cudaGetLastError();
    nkv::set_error("peer_free: %s", cudaGetErrorString(e));
    return NKV_ERR_CUDA;
  }
  return NKV_OK;
}

extern "C" int nkv_shard_scores(nkv_stream_t stream, const void* q, int64_t q_row_stride, int64_t q_head_stride,
                                int hq, int hkv, int head_dim, const void* reps, int r, int max_blocks, int nblocks,
                                const int32_t* protected_ids, int n_protected, void* const* exchanges, int n_ranks,
                                int rank, void* workspace, size_t workspace_bytes) {
  NKV_REQUIRE(exchanges, "shard_scores: null exchanges");
  const nkv::PeerArgs pa{exchanges, n_ranks, rank, max_blocks, hq * n_ranks};
  const float* ws_scores = nullptr;
  return nkv::select_scores((cudaStream_t)stream, q, q_row_stride, q_head_stride, hq, hkv, head_dim, reps, r,
                            max_blocks, nblocks, protected_ids, n_protected, 1, workspace, workspace_bytes, &ws_scores,
                            nullptr, &pa);
}

extern "C" int nkv_shard_attend(nkv_stream_t stream, const nkv_attend_args* a, void* const* exchanges, int n_ranks,
                                int rank, int max_blocks, int nblocks, int64_t* out_ids, float* out_scores,
                                void* out_full) {
  NKV_REQUIRE(a && exchanges && a->block_ids == out_ids, "shard_attend: args->block_ids must be out_ids");
  const nkv::PeerArgs pa{exchanges, n_ranks, rank, max_blocks, a->hq * n_ranks};
  return nkv::attend_ranked(stream, a, nullptr, nblocks, out_ids, out_scores, &pa, out_full);
}
