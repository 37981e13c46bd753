/*
 * nanokv.h — C ABI of the NanoKV block-sparse attention path on B200 (sm_100a).
 *
 * Plain pointers and sizes only: every tensor argument is a device pointer (or a
 * host pointer that is mapped into the device address space, where stated) plus
 * its shape/stride integers.  Every entry point is asynchronous on the given
 * CUDA stream, returns NKV_OK or a negative status, and leaves a message for
 * nkv_last_error() on failure.  No entry point allocates device memory: the
 * caller passes a workspace sized by the matching *_workspace_bytes() query.
 *
 * Geometry supported by the kernels: head_dim 128, bf16 activations, query heads
 * per KV head G in {1, 2, 4, 8}, block_size in {16, 32, 64, 128}, r <= 8.
 * Anything else returns NKV_ERR_UNSUPPORTED (there is no fallback path).
 *
 * Each declaration names the reference interface it replaces
 * (Tao20060602/nano-vllm-kv-optimizer, path:line).
 */
#ifndef NANOKV_H
#define NANOKV_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NKV_OK 0
#define NKV_ERR_ARG (-1)         /* bad shape, pointer or size                        */
#define NKV_ERR_UNSUPPORTED (-2) /* geometry outside what the kernels are built for   */
#define NKV_ERR_CUDA (-3)        /* a CUDA call or launch failed                      */
#define NKV_ERR_DEVICE (-4)      /* a kernel recorded an error word (see nkv_check)   */

/* History storage kinds for the selected-block segment. */
#define NKV_STORE_BF16 0        /* bf16 [max_blocks][Hkv][B][D]                          */
#define NKV_STORE_INT8_REF 1    /* int8 store, K scale [Hkv][D], V scale [max_blocks][Hkv] */
#define NKV_STORE_INT8_TOKEN 2  /* int8 store, bf16 scale per (block, head, token) for K and V */

typedef void* nkv_stream_t; /* a cudaStream_t */

const char* nkv_last_error(void);
int nkv_version(void);

/* Device address of pinned host memory (cudaHostGetDevicePointer); fails unless
 * the range is mapped.  The offload mode passes such addresses as k_store /
 * v_store.  Replaces nothing in the reference (whose host history is pageable
 * and gathered on the CPU, m12_runtime.py:1213-1238). */
int nkv_map_host(void* host_ptr, void** dev_ptr);

/* Reads the 32-bit error word kernels write into a workspace (bounded waits,
 * out-of-range ids).  Synchronous: copies 4 bytes device->host on `stream`.
 * Returns NKV_OK when clear, NKV_ERR_DEVICE (and clears it) otherwise. */
int nkv_check(nkv_stream_t stream, void* workspace);

/* ------------------------------------------------------------------------ */
/* (1) Block-representative scoring + protection mask + exact Top-K.
 *
 * Replaces M12LayerRuntime._gpu_select (nanovllm/sparse/m12_runtime.py:959-1055)
 * and the Triton fused_block_scores (nanovllm/sparse/fused_select.py:57-79).
 *
 * score[b] = max over query rows n < nq, query heads h < hq, reps j < r of
 *            fp32(q[n][h]) . fp32(reps[h / G][b][j])          (G = hq / hkv)
 * Blocks listed in protected_ids (ids >= nblocks are ignored) score -inf.
 * Writes the k best block ids to out_ids (int64, ordered by score descending,
 * equal scores by ascending id) and, when non-NULL, their scores to
 * out_topk_scores and the masked per-block scores to out_block_scores.
 * q: bf16 rows with the given strides (elements), head_dim contiguous.
 * reps: bf16 [hkv][max_blocks][r][head_dim].  1 <= k <= min(nblocks, 256).  */
size_t nkv_select_workspace_bytes(int max_blocks, int nq);
int nkv_select(nkv_stream_t stream, const void* q, int nq, int64_t q_row_stride,
               int64_t q_head_stride, int hq, int hkv, int head_dim, const void* reps, int r,
               int max_blocks, int nblocks, const int32_t* protected_ids, int n_protected, int k,
               int64_t* out_ids, float* out_topk_scores, float* out_block_scores, void* workspace,
               size_t workspace_bytes);

/* Lossless-verify selection: a separate Top-K per query row, their sorted
 * union and the per-row allowed mask.
 * Replaces M12LayerRuntime._gpu_select_per_query (m12_runtime.py:1057-1087).
 * out_union: int64 [nq * k] (first *out_count valid, ascending);
 * out_count: int32 device scalar; out_allowed: uint8 [nq][nq * k]. nq <= 8. */
int nkv_select_per_query(nkv_stream_t stream, const void* q, int nq, int64_t q_row_stride,
                         int64_t q_head_stride, int hq, int hkv, int head_dim, const void* reps,
                         int r, int max_blocks, int nblocks, const int32_t* protected_ids,
                         int n_protected, int k, int64_t* out_union, int32_t* out_count,
                         uint8_t* out_allowed, float* out_scores, void* workspace,
                         size_t workspace_bytes);

/* ------------------------------------------------------------------------ */
/* (2)+(3) Fused gather-and-attend GQA attention over the sparse key set.
 *
 * Replaces the decode gather/pack + packed attention of M12LayerRuntime.decode
 * (m12_runtime.py:1164-1320, _fused_attention fast path :868-873), the int8
 * dequant-and-pack (fused_dequant.py:47-63, m12_runtime.py:1243-1278) and the
 * verify attention of verify_tokens (m12_runtime.py:716-760, masked path
 * :875-896).  Keys are read in place from four segments, in this order:
 *   0. selected history blocks  block_ids[0..n_sel) of the block store
 *   1. sink window              sink[h][0..sink_len)
 *   2. recent ring slice        ring[h][(ring_start + i) % ring_cap], i < ring_len
 *   3. current tokens           cur[j], j < n_cur (0 or nq): query n sees j <= n
 * With allowed != NULL, query n sees block_ids[u] only if allowed[n][u] != 0.
 * ring_write_pos >= 0 additionally stores current token 0 into that ring slot
 * (the decode recent-window append).  Works for nq <= 8. */
typedef struct nkv_attend_args {
  const void* q; /* bf16 [nq][hq][head_dim] */
  int64_t q_row_stride, q_head_stride;
  int nq, hq, hkv, head_dim, block_size;
  float scale;
  /* segment 0 */
  const int64_t* block_ids; /* device int64 [n_sel] */
  int n_sel;
  int max_blocks;           /* bound for block ids (store capacity)          */
  int store_kind;           /* NKV_STORE_*                                   */
  const void* k_store;      /* [max_blocks][hkv][B][D]; may be host-mapped   */
  const void* v_store;
  const float* k_chan_scale;  /* NKV_STORE_INT8_REF: [hkv][D]             */
  const float* v_block_scale; /* NKV_STORE_INT8_REF: [max_blocks][hkv]    */
  const void* k_tok_scale;    /* NKV_STORE_INT8_TOKEN: bf16 [max_blocks][hkv][B] */
  const void* v_tok_scale;
  const uint8_t* allowed; /* optional [nq][allowed_stride] */
  int allowed_stride;
  /* segment 1 */
  const void* sink_k;
  const void* sink_v; /* bf16 [hkv][sink_cap][D] */
  int sink_cap, sink_len;
  /* segment 2 */
  void* ring_k;
  void* ring_v; /* bf16 [hkv][ring_cap][D] */
  int ring_cap, ring_start, ring_len;
  /* segment 3 */
  const void* cur_k;
  const void* cur_v; /* bf16 rows [n_cur][hkv][D] with strides */
  int64_t cur_row_stride, cur_head_stride;
  int n_cur;
  int ring_write_pos;
  /* output */
  void* out; /* bf16 [nq][hq][D] */
  int64_t out_row_stride, out_head_stride;
  void* workspace;
  size_t workspace_bytes;
  /* 1: the kernel launched just before on this stream is the nkv_select that
   * writes block_ids, and every other input was complete before that launch.
   * The attend kernel then starts while the selection runs (programmatic
   * dependent launch) and waits for it only before reading block_ids. */
  int overlap_select;
} nkv_attend_args;

/* max_tokens bounds n_sel * block_size + sink_len + ring_len + n_cur. */
size_t nkv_attend_workspace_bytes(int hkv, int hq, int nq, int max_tokens);
int nkv_attend(nkv_stream_t stream, const nkv_attend_args* args);
/* Launch shape chosen by the last nkv_attend on the calling thread: whether the
 * splits of a head were merged inside a thread-block cluster (0: no, 1: yes,
 * 2: yes, by the tile-split decode kernel of a ranked single-query call), the
 * number of splits per head and the keys per CTA.  Host only (no GPU work). */
int nkv_attend_last_config(int* cluster, int* splits, int* keys_per_cta);

/* nkv_attend without a caller workspace.  No counterpart in the reference (its
 * attention has no workspace argument).  It serves callers that cannot
 * allocate device memory when they call: hosts whose device memory belongs to
 * another framework's pool, serving loops that forbid allocation after
 * warm-up, and code that must not synchronise the device (cudaMalloc and
 * cudaFree may).
 *
 * The workspace is a scratch array of NKV_ATTEND_STATIC_SCRATCH_BYTES inside
 * the library, one per device; args->workspace and workspace_bytes are
 * ignored, and a call whose nkv_attend_workspace_bytes exceeds the scratch
 * fails with NKV_ERR_ARG.  At the reference geometry (hkv 8, hq 32, one query)
 * that is at most 8048 keys per call: Top-32 of 64-token blocks with a 64-token
 * sink, a 512-token recent window and the current token (2625 keys) fits, and
 * so does any selection of up to 116 such blocks.  The first call on a device
 * looks the scratch up (cudaGetSymbolAddress, which may load the module
 * there): make it before any stream capture.  The address is cached per device
 * ordinal for the life of the process, so it does not survive a
 * cudaDeviceReset of that device.  Each call clears the scratch's error word
 * and merge counters with cudaMemsetAsync on `stream` and ignores
 * overlap_select.  Calls on one device share the scratch, so calls that can
 * overlap in time (several streams or host threads) race; serialise them. */
#define NKV_ATTEND_STATIC_SCRATCH_BYTES ((size_t)8 << 20)
int nkv_attend_static(nkv_stream_t stream, const nkv_attend_args* args);

/* The error word of the static scratch on the current device, which the
 * kernels of nkv_attend_static write (a bounded wait that ran out, a block id
 * outside the store).  Same contract as nkv_check on a caller workspace:
 * synchronous on `stream`, NKV_OK when clear, NKV_ERR_DEVICE (and cleared)
 * otherwise.  The next nkv_attend_static call clears the word, so check after
 * each call whose result matters.  No counterpart in the reference. */
int nkv_attend_static_check(nkv_stream_t stream);

/* One decode step of a layer: nkv_select over the layer's representatives
 * for the single query, then nkv_attend of that query over the selected
 * blocks, sink, recent ring and the current token (which it appends to the
 * ring at attend.ring_write_pos).  attend.block_ids / n_sel are replaced by
 * out_ids / k, attend.overlap_select is ignored.
 * The step is a scoring grid followed by the attention grid ranking the
 * scores in each CTA (programmatic dependent launch overlaps the two).  With
 * the environment variable NKV_DECODE_ONE=1, and where it applies (k <= 32,
 * r in {1, 2, 4}, nblocks <= 2048, one thread-block cluster per KV head that
 * the device holds all at once), it is ONE cooperative launch instead: every
 * CTA scores a share of the blocks for all heads on the tensor cores,
 * publishes the masked block scores as keys tagged with a per-launch epoch in
 * the select workspace, and selects the top k from all published keys itself
 * (nkv_select's order; scores equal to fp32 rounding).  The select workspace
 * must start at zero and is used by one stream at a time.
 * Replaces the device work of M12LayerRuntime.decode (m12_runtime.py:1141-1346:
 * recent shift and append :1166-1172, select :1193-1198, gather and pack
 * :1213-1309, attention :1316-1320) in one host call. */
typedef struct {
  nkv_attend_args attend; /* nq == n_cur == 1 */
  const void* reps;       /* bf16 [hkv][reps_blocks][r][head_dim] */
  int r, reps_blocks, nblocks;
  const int32_t* protected_ids;
  int n_protected, k;
  int64_t* out_ids;       /* [k], device */
  float* out_topk_scores; /* [k] or NULL */
  void* select_workspace;
  size_t select_workspace_bytes;
  /* Optional device int32 [2], 8-byte aligned: {ring head, 0}.  NULL: the
   * recent window is attend.ring_start / ring_len / ring_write_pos as given.
   * Otherwise the step reads the head from the device instead of
   * attend.ring_start / ring_write_pos (current token written at slot head,
   * window = the ring_len slots after it) and advances it by one, so a CUDA
   * graph of decode steps replays with the window moving on every replay.
   * Needs a full window (ring_len == ring_cap - 1) and the two-launch form
   * (the one-launch form and NKV_DECODE_FUSED=0 return NKV_ERR_UNSUPPORTED).
   * Word 1 counts the CTAs that have read the head and must start at 0.
   * Replaces the host-side shift of the recent window of
   * M12LayerRuntime.decode (m12_runtime.py:1166-1172) for graph replay. */
  int32_t* ring_head;
} nkv_decode_args;
int nkv_decode_step(nkv_stream_t stream, const nkv_decode_args* args);
/* How the calling thread's last nkv_decode_step ran: 1 one launch, 2 a
 * scoring grid + ranked attention, 3 nkv_select + nkv_attend, 0 none yet.
 * (Introspection for tests and benchmarks; no counterpart in the reference.) */
int nkv_decode_last_form(void);

/* The NKV_* tuning variables of the environment (launch shapes, merge form,
 * the decode step's form) are read once per host thread and cached; after
 * changing them, call nkv_reload_env() to have every thread read them again.
 * (No counterpart in the reference.) */
void nkv_reload_env(void);

/* The two halves of nkv_decode_step, for a caller that combines block scores
 * across devices between them (KV heads sharded over GPUs: each rank scores
 * its own heads, the scores are max-reduced over the ranks, then every rank
 * attends its heads to the blocks ranked from the reduced scores).
 * nkv_select_scores writes the protection-masked block scores of one query
 * row (max over the given heads and reps) to out_scores [nblocks]; it is
 * M12LayerRuntime._gpu_select's scoring (m12_runtime.py:999-1003) without the
 * topk.  nkv_attend_ranked is nkv_attend for one query whose CTAs rank
 * `scores` themselves (top args->n_sel, nkv_select's order; n_sel <= 32,
 * nblocks <= 2048); the ranked ids (and scores when out_scores != NULL) are
 * written to out_ids.  args->block_ids must equal out_ids. */
int nkv_select_scores(nkv_stream_t stream, const void* q, int64_t q_row_stride, int64_t q_head_stride, int hq,
                      int hkv, int head_dim, const void* reps, int r, int max_blocks, int nblocks,
                      const int32_t* protected_ids, int n_protected, float* out_scores, void* workspace,
                      size_t workspace_bytes);
int nkv_attend_ranked(nkv_stream_t stream, const nkv_attend_args* args, const float* scores, int nblocks,
                      int64_t* out_ids, float* out_scores);

/* KV-head sharding with the exchange inside the kernels (no collective
 * library on the data path).  The P ranks of a layer (one GPU each, P <= 8)
 * each allocate one exchange buffer of nkv_shard_exchange_bytes() with
 * nkv_peer_alloc (device memory, zeroed, plus a 64-byte CUDA IPC handle), send
 * the handle to the other ranks (any host channel), and open theirs with
 * nkv_peer_open.  `exchanges` is then the host array of the P buffers as this
 * rank addresses them (its own at [rank]).  Per decode step:
 *   nkv_shard_scores: the masked block scores of this rank's heads (as
 *     nkv_select_scores), written as step-tagged words into every rank's
 *     buffer over NVLink;
 *   nkv_shard_attend: nkv_attend_ranked whose CTAs poll every rank's scores in
 *     this rank's buffer (bounded waits), rank the max over ranks (the same
 *     ids as one GPU), attend this rank's heads, write this rank's rows of the
 *     full-width output out_full [hq * n_ranks][128] and push them as tagged
 *     words to every other rank, and pull the other ranks' rows into
 *     out_full before the grid ends.  args->out must be this rank's rows of
 *     out_full (offset rank * hq * 128, head stride 128).
 * Every rank must run the same steps in the same order (the step tags are a
 * per-buffer epoch advanced by nkv_shard_attend); a peer that stops leaves the
 * others' waits to time out (error word of the attend workspace).
 * Replaces the MAX all-reduce of the scores and the all-gather of the outputs
 * around the reference's per-layer decode (m12_runtime.py:999-1003, 1316-1320;
 * the reference itself runs on one GPU). */
#define NKV_IPC_HANDLE_BYTES 64
size_t nkv_shard_exchange_bytes(int n_ranks, int max_blocks, int hq_all);
int nkv_peer_alloc(size_t bytes, void** dptr, void* ipc_handle);
int nkv_peer_open(const void* ipc_handle, void** dptr);
int nkv_peer_close(void* dptr);
int nkv_peer_free(void* dptr);
int nkv_shard_scores(nkv_stream_t stream, const void* q, int64_t q_row_stride, int64_t q_head_stride, int hq,
                     int hkv, int head_dim, const void* reps, int r, int max_blocks, int nblocks,
                     const int32_t* protected_ids, int n_protected, void* const* exchanges, int n_ranks, int rank,
                     void* workspace, size_t workspace_bytes);
int nkv_shard_attend(nkv_stream_t stream, const nkv_attend_args* args, void* const* exchanges, int n_ranks, int rank,
                     int max_blocks, int nblocks, int64_t* out_ids, float* out_scores, void* out_full);

/* ------------------------------------------------------------------------ */
/* (4) Segmented prefill attention on the tensor cores: the same four segments
 * as nkv_attend for a whole chunk of nq queries (nq == n_cur, causal in-chunk,
 * bottom-right aligned), without packing.  With n_sel = sink_len = ring_len = 0
 * it is the dense causal attention of the first chunk.
 * Replaces prefill_chunk's pack + _prefill_attention (m12_runtime.py:589-642,
 * 809-839; FA2 flash_attn_func call :834-839), the first-chunk FA2 call
 * (nanovllm/layers/attention.py:80-85) and the segmented adapter's
 * prepare/attend contract (nanovllm/sparse/segmented_prefill_adapter.py:95-147).
 * Any store_kind (int8 selected blocks are dequantised on load); requires
 * allowed == NULL.  The workspace holds only the error word. */
size_t nkv_prefill_workspace_bytes(int hkv, int hq, int nq, int max_tokens);
int nkv_prefill(nkv_stream_t stream, const nkv_attend_args* args);

/* The selected blocks of a prefill call (args->block_ids[0, n_sel) of the block
 * store args->k_store / v_store, any store_kind, in device or mapped pinned host
 * memory) copied into a device bf16 staging store k_out / v_out laid out as
 * [n_sel][hkv][block_size][head_dim] (staging block i = history block ids[i]),
 * int8 kinds dequantised with the attention kernels' rounding (bf16 of the fp32
 * product).  Passing the staging store with block ids 0 .. n_sel - 1 and
 * store_kind NKV_STORE_BF16 to nkv_prefill then runs the tensor-core kernel,
 * and each selected block crosses the host link once per call.  The error word
 * goes to args->workspace.  Replaces the reference's staging of the selected
 * blocks for the packed prefill (m12_runtime.py:560-586) and the dequant pack
 * of the int8 history (:1243-1267, fused_dequant.py:47-63). */
int nkv_prefill_gather(nkv_stream_t stream, const nkv_attend_args* args, void* k_out, void* v_out);

/* ------------------------------------------------------------------------ */
/* (5) KV store + representative refresh for one prefill chunk.
 *
 * Replaces M12LayerRuntime._store_kv (m12_runtime.py:420-513: block padding,
 * history append, sink/recent update) and _build_reps_gpu (:354-395).
 * Writes ceil(T / B) blocks starting at start_block (zero padded), rebuilds
 * their r representatives (mean direction, then farthest point with the
 * reference's clamp-at-zero criterion), copies tokens [0, sink_write) into
 * the sink and tokens [ring_first, T) into ring slots (ring_pos0 + i) % cap.
 * k_store == v_store == NULL rebuilds representatives only (the reference's
 * standalone _build_reps_gpu). */
typedef struct nkv_store_args {
  const void* k;
  const void* v; /* bf16 rows [T][hkv][D] with strides */
  int64_t k_row_stride, k_head_stride, v_row_stride, v_head_stride;
  int T, hkv, head_dim, block_size, r;
  int start_block;
  int max_blocks;   /* block dimension of reps / rep_index                */
  int store_blocks; /* capacity (blocks) of the block store and its scales */
  int store_kind;
  void* k_store;
  void* v_store;        /* may be host-mapped (offload)                     */
  const float* k_chan_scale; /* INT8_REF: [hkv][D] input (see nkv_k_channel_scale) */
  float* v_block_scale;      /* INT8_REF: [max_blocks][hkv] output             */
  void* k_tok_scale;
  void* v_tok_scale;    /* INT8_TOKEN: bf16 [max_blocks][hkv][B] outputs       */
  void* reps;           /* bf16 [hkv][max_blocks][r][D]                      */
  int16_t* rep_index;   /* optional [hkv][max_blocks][r]: chosen token       */
  void* sink_k;
  void* sink_v;
  int sink_cap, sink_write;
  void* ring_k;
  void* ring_v;
  int ring_cap, ring_pos0, ring_first;
} nkv_store_args;

int nkv_store_chunk(nkv_stream_t stream, const nkv_store_args* args);

/* Recent-window append of T tokens: token i (i >= max(0, T - ring_cap)) goes to
 * ring slot (ring_pos0 + i) % ring_cap of every head.  With ring_pos0 =
 * head + min(ring_cap, valid_len) this is the reference's left-aligned window
 * update with carry (m12_runtime.py:488-503) and commit_verified (:777-803). */
int nkv_ring_append(nkv_stream_t stream, const void* k, const void* v, int T, int64_t k_row_stride,
                    int64_t k_head_stride, int64_t v_row_stride, int64_t v_head_stride, int hkv,
                    int head_dim, void* ring_k, void* ring_v, int ring_cap, int ring_pos0);

/* Self-test of the division the store kernel uses for the key directions
 * (a correctly rounded reciprocal and one fma correction instead of a divide
 * per element): out[i] = a[i] / b[i] for b[i] > 0 normal and a finite quotient,
 * to be compared with the division operator.  No counterpart in the reference. */
int nkv_selftest_div(nkv_stream_t stream, const float* a, const float* b, float* out, int n);

/* Per-(kv head, channel) K scale of the reference int8 scheme, from one chunk:
 * scale[h][d] = max(max_t |k[t][h][d]|, 1e-8) / 127   (m12_runtime.py:463-465). */
int nkv_k_channel_scale(nkv_stream_t stream, const void* k, int T, int64_t row_stride,
                        int64_t head_stride, int hkv, int head_dim, float* out_scale);

/* Bf16 mean of each of nseg consecutive query segments (torch.tensor_split
 * sizes).  Replaces prefill_query_summaries (m12_runtime.py:53-67). */
int nkv_query_summaries(nkv_stream_t stream, const void* q, int T, int64_t row_stride,
                        int64_t head_stride, int hq, int head_dim, int nseg, void* out);

/* Dense paged-cache row scatter, the twin of the Triton store_kvcache
 * (nanovllm/layers/attention.py:11-41): for every i with slot[i] != -1,
 * k_cache[slot[i]][:] = key[i][:], v_cache[slot[i]][:] = value[i][:].
 * Rows hold row_elems = num_heads * head_dim bf16 values; key/value rows are
 * key_stride / value_stride elements apart; cache rows are row_elems apart. */
int nkv_store_kvcache(nkv_stream_t stream, const void* key, int64_t key_stride,
                      const void* value, int64_t value_stride, void* k_cache, void* v_cache,
                      const int64_t* slot_mapping, int n, int row_elems);

/* ------------------------------------------------------------------------ */
/* The callers either side of the sparse path in a Qwen3 decoder layer (the
 * full-model harness).  bf16 rows, fp32 arithmetic, no host synchronisation. */

/* Per-head RMSNorm of q and k followed by the rotary embedding, in place on the
 * fused qkv projection output [T][(hq + 2*hkv) * head_dim] (row_stride elements
 * apart): for every token t and q/k head, x <- bf16(bf16(x * rsqrt(mean(x^2) +
 * eps)) * weight), then (x1, x2) = halves of x, y1 = x1*cos - x2*sin,
 * y2 = x2*cos + x1*sin with cos/sin = cos_sin[positions[t]] ([P][head_dim] fp32,
 * cos in the first half).  v is untouched.  A position outside [0, P) records
 * an error in *err (may be null) and uses row 0.  Replaces the q_norm/k_norm
 * + rotary_emb calls of Qwen3Attention.forward (nanovllm/models/qwen3.py:91-98,
 * nanovllm/layers/layernorm.py:16-26, nanovllm/layers/rotary_embedding.py:7-15,
 * 138-151), which produce the q/k the sparse runtime reads. */
int nkv_qk_norm_rope(nkv_stream_t stream, void* qkv, long long row_stride, int T, int hq, int hkv,
                     int head_dim, const void* q_weight, const void* k_weight, const float* cos_sin,
                     const long long* positions, long long max_positions, float eps, int* err);

/* Residual add + RMSNorm over [T][H] rows (H a multiple of 8, <= 4096): with
 * has_residual, s = x + residual (fp32), residual <- bf16(s); else s = x and
 * residual <- x; out <- bf16(bf16(s * rsqrt(mean(s^2) + eps)) * weight).  out
 * may alias x.  Replaces RMSNorm.forward (nanovllm/layers/layernorm.py:16-50). */
int nkv_add_rms_norm(nkv_stream_t stream, const void* x, void* residual, const void* weight, void* out,
                     int T, int H, float eps, int has_residual);

/* SwiGLU: out[t][j] = bf16(silu(g) * u), g = gate_up[t][j], u = gate_up[t][I + j]
 * (fp32).  Replaces SiluAndMul (nanovllm/layers/activation.py:6-11). */
int nkv_silu_mul(nkv_stream_t stream, const void* gate_up, void* out, int T, int I);

/* y[r][n] = bf16(sum_k x[r][k] * w[n][k]) for rows = 1..4 rows of x (fp32
 * accumulation): the decode-time projections and LM head of one or a few
 * tokens, weights [N][K] row-major (K a multiple of 8, rows 16-byte aligned),
 * streamed from HBM once.  Replaces the M = 1 linear layers
 * (nanovllm/layers/linear.py, embed_head.py) during decode. */
int nkv_gemv_bf16(nkv_stream_t stream, const void* x, long long x_row_stride, int rows, const void* w,
                  long long w_row_stride, int N, int K, void* y, long long y_row_stride);

#ifdef __cplusplus
}
#endif
#endif /* NANOKV_H */
