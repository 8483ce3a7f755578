/*
 * shardserve_b200 — C ABI of the B200 (sm_100a) ragged paged-attention hot path.
 *
 * Two device operations replace the two halves of the ShardServe attention path:
 *
 *   ss_kv_append               replaces Cache.write            (shardserve/cache.py:47-49)
 *   ss_ragged_paged_attention  replaces ragged_attention_direct (shardserve/kernel.py:11-82)
 *                              and its Triton kernel           (shardserve/kernel.py:85-166)
 *
 * Every entry point takes plain device pointers, element strides and sizes; nothing here
 * depends on PyTorch. Strides are in ELEMENTS (not bytes), exactly like torch's
 * Tensor.stride(), which the reference passes to its kernel (kernel.py:61-76).
 * `stream` is a cudaStream_t passed as void* (NULL = legacy default stream). No entry point
 * allocates device memory, synchronises the stream or reads device memory on the host, so
 * all of them can be recorded into a CUDA graph (the reference captures the attention
 * call in runtime.py:68-71).
 *
 * Return value: SS_OK (0) or one of the SS_ERR_* codes; ss_last_error_message() gives a
 * human-readable reason for the last failure on the calling thread.
 *
 * Device-side problems that the host cannot see without reading device memory (a page id
 * outside the pool, a sequence id outside the block table, a position past the block-table
 * width, an append slot outside the pool) never fault: the offending page reads as zeros
 * (attention) or the row is skipped (append), and a bit is OR-ed into the 32-bit error word
 * at byte offset 0 of the workspace (SS_DEVERR_* below). ss_fetch_device_errors() reads it.
 */
#ifndef SHARDSERVE_B200_H
#define SHARDSERVE_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define SS_API __attribute__((visibility("default")))
#else
#define SS_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---------------------------------------------------------------------- */
#define SS_OK 0
#define SS_ERR_INVALID 1     /* bad argument: shape, dtype flag, null pointer, stride      */
#define SS_ERR_UNSUPPORTED 2 /* valid for the reference but not for this build (none today) */
#define SS_ERR_CUDA 3        /* a CUDA runtime call failed                                  */
#define SS_ERR_WORKSPACE 4   /* workspace missing or smaller than ss_attention_workspace_bytes */

/* ---- device error bits (OR-ed into the workspace error word) --------------------------- */
#define SS_DEVERR_PAGE 0x1u     /* block-table entry outside [0, num_pages)              */
#define SS_DEVERR_SEQ 0x2u      /* query_seq_ids entry outside [0, block_table rows)     */
#define SS_DEVERR_POS 0x4u      /* position < 0 or position + 1 > 16 * block_table cols   */
#define SS_DEVERR_SLOT 0x8u     /* append slot outside [0, 16 * num_pages)               */
#define SS_DEVERR_TIMEOUT 0x10u /* a bounded on-chip wait gave up (never expected)        */

/* Page size of the paged pool: the reference supports exactly 16 (kernel.py:8, 36-37). */
#define SS_BLOCK_SIZE 16

/* Library version (major * 10000 + minor * 100 + patch). */
SS_API int ss_version(void);

/* Text for a status code; never NULL. */
SS_API const char* ss_status_string(int status);

/* Reason for the last non-OK return on the calling thread ("" if none). */
SS_API const char* ss_last_error_message(void);

/*
 * Slot-mapped KV append.  Replaces Cache.write (shardserve/cache.py:47-49):
 *     k_pool.flatten(0, 1)[slots[i]] = k[i];  v_pool.flatten(0, 1)[slots[i]] = v[i]
 * k, v        : bf16 [tokens, kv_heads, head_dim]   (strides k_strides / v_strides)
 * k_pool/v_pool: bf16 [num_pages, 16, kv_heads, head_dim] (strides *_pool_strides)
 * slots       : [tokens] int32 (slots_is_int64 = 0) or int64 (= 1); slot s is row s % 16 of
 *               page s / 16 (the reference builds s = table[p // 16] * 16 + p % 16,
 *               runtime.py:38).
 * workspace   : optional (may be NULL); if given, its error word receives SS_DEVERR_SLOT.
 * Copies are bit-exact.  Slots outside the pool are skipped.  Duplicate slots within one
 * call leave one of the candidate rows, unspecified which (as index_copy_ does).
 */
SS_API int ss_kv_append(const void* k, const int64_t k_strides[3], const void* v,
                 const int64_t v_strides[3], void* k_pool, const int64_t k_pool_strides[4],
                 void* v_pool, const int64_t v_pool_strides[4], const void* slots,
                 int slots_is_int64, int64_t tokens, int64_t num_pages, int kv_heads,
                 int head_dim, void* workspace, void* stream);

/*
 * Rotary position embedding of q and k fused with the slot-mapped KV append.  Replaces
 *     q, k = apply_rope(q, k, cos, sin, positions)   (shardserve/math.py:28-38, model.py:25)
 *     cache.write(layer, k, v, slots)                 (shardserve/cache.py:47-49, model.py:32)
 * in one launch, bit-exact with torch's bf16 arithmetic (one bf16 rounding per multiply and
 * per add, cos / sin rows rounded to bf16 first, math.py:36-38).
 * q, q_out     : bf16 [tokens, heads, head_dim]; q_out receives the rotated queries and may
 *                be q itself (rotation in place)
 * k, v         : bf16 [tokens, kv_heads, head_dim]: unrotated keys, values
 * cos_table, sin_table: fp32 [table_rows, head_dim] (the caller's tables, as built by
 *                math.build_rope_cache, math.py:12-20), element strides cos/sin_strides
 * positions    : [tokens] int32 / int64 row of each token in the tables
 * k_pool/v_pool, slots: as ss_kv_append; the rotated k and v land in row slot % 16 of page
 *                slot / 16
 * head_dim even.  A token whose position lies outside [0, table_rows) is skipped entirely
 * (SS_DEVERR_POS); a slot outside the pool skips that token's append (SS_DEVERR_SLOT).
 * workspace    : optional error word, as ss_kv_append.
 */
SS_API int ss_rope_kv_append(const void* q, const int64_t q_strides[3], void* q_out,
                      const int64_t q_out_strides[3], const void* k, const int64_t k_strides[3],
                      const void* v, const int64_t v_strides[3], const float* cos_table,
                      const int64_t cos_strides[2], const float* sin_table,
                      const int64_t sin_strides[2], int64_t table_rows, const void* positions,
                      int positions_is_int64, void* k_pool, const int64_t k_pool_strides[4],
                      void* v_pool, const int64_t v_pool_strides[4], const void* slots,
                      int slots_is_int64, int64_t tokens, int heads, int kv_heads, int head_dim,
                      int64_t num_pages, void* workspace, void* stream);

/*
 * Per-step attention metadata built on the device.  Replaces the host loops and copies of
 * metadata(plan, cache, device, context, bucket) (shardserve/runtime.py:28-49), with the
 * same output bit for bit.  The caller keeps every live request's block list on the device
 * (`store`: int32 rows of stride store_row_stride, `store_lens`: blocks per row), written
 * once when the request is admitted, and passes per step one packed int64 device buffer:
 *     packed[4 r + 0..3] = store row (-1 for a graph-padding row), query length, first
 *                          position, offset of the row's first token     (r < rows)
 *     packed[4 rows + s] = sampled token index s                          (s < n_selected)
 *     packed[4 rows + n_selected + t] = token id t                        (t < tokens)
 * Outputs (device): tables int32 [rows, table_cols] (row stride table_row_stride), ids /
 * positions / slots int64 [tokens], seqs int32 [tokens], selected int64 [n_selected].
 * Padding rows get tables[r, 0] = pad_block_base + r and one token (id 0, position 0,
 * slot (pad_block_base + r) * 16), as runtime.py:41-44.  A store row outside the store
 * (SS_DEVERR_SEQ) or a position outside the request's blocks (SS_DEVERR_POS) yields slot -1.
 * workspace: optional error word, as ss_kv_append.
 */
SS_API int ss_build_metadata(const int64_t* packed, int64_t rows, int64_t n_selected,
                      int64_t tokens, const int32_t* store, const int32_t* store_lens,
                      int64_t store_rows, int64_t store_row_stride, int64_t pad_block_base,
                      int32_t* tables, int64_t table_cols, int64_t table_row_stride,
                      int64_t* ids, int64_t* positions, int32_t* seqs, int64_t* slots,
                      int64_t* selected, void* workspace, void* stream);

/*
 * TP2 attention output projection fused with its all-reduce over NVLink (two ranks).
 * Replaces, per layer and rank, reduce(F.linear(attention, w_o)) of shardserve/model.py:40
 * with reduce = the two-rank all-reduce of shardserve/runtime.py:17-24:
 *     out = bf16(P_0 + P_1),  P_r = bf16(attn_r w_o,r^T)  (fp32 accumulation, as F.linear)
 * Both ranks make the same sequence of calls and both receive `out`.
 * attn        : bf16 [tokens, in_features] (this rank's heads), unit column stride
 * w_o         : bf16 [out_features, in_features] (this rank's column shard of o_proj)
 * out         : bf16 [tokens, out_features]
 * local_inbox / peer_inbox: 6 * ceil(max_tokens / 32) * 32 * out_features bytes on this
 *               rank / the other rank (its buffer opened with ss_ipc_open), zeroed once
 *               (ss_device_alloc_zeroed) and never cleared again
 * epoch_counter: 8 zeroed device bytes per rank that count its calls (the kernel advances
 *               them, so calls can be replayed from a CUDA graph)
 * out_features a multiple of 128, in_features of 256.  Tiles are 128 tokens x 32
 * features; all tiles of a call must fit one wave of the GPU (tiles <= SM count, so
 * ceil(tokens / 128) * out_features / 32 <= SMs).  workspace: the 4-byte error word (a
 * partner that does not arrive within ~1 s sets SS_DEVERR_TIMEOUT instead of hanging).
 * Calls on one rank are stream-ordered; the two ranks' n-th calls run concurrently.
 */
SS_API int ss_tp2_oproj_allreduce(const void* attn, const int64_t attn_strides[2],
                           const void* w_o, const int64_t w_strides[2], void* out,
                           const int64_t out_strides[2], int64_t tokens, int out_features,
                           int in_features, const void* local_inbox, void* peer_inbox,
                           int64_t max_tokens, void* epoch_counter, void* workspace,
                           void* stream);

/* Zero-filled device allocation / release (inboxes and flags of ss_tp2_oproj_allreduce). */
SS_API int ss_device_alloc_zeroed(size_t bytes, void** ptr);
SS_API int ss_device_free(void* ptr);
/* CUDA IPC: export a ss_device_alloc_zeroed allocation as a 64-byte handle, open another
 * process's handle (peer access over NVLink), close it. */
SS_API int ss_ipc_handle(void* ptr, void* handle64);
SS_API int ss_ipc_open(const void* handle64, void** ptr);
SS_API int ss_ipc_close(void* ptr);

/*
 * Workspace size (bytes) that ss_ragged_paged_attention needs on `device` for this geometry.
 * Byte 0..3 of the workspace is the device error word (zero it to start clean).  Bytes
 * 64..71 hold the chunked-prefill work counter and bytes 72..79 the decode kernel's grid
 * barrier counter: they must be zero before the first call (a freshly zeroed buffer, or the
 * first 256 bytes zeroed) and every call leaves them consistent.  The rest is scratch that every
 * call rewrites before reading (split-K partial states and per-row split descriptors), so
 * one buffer can be reused across calls on one stream without clearing.  Calls that run
 * concurrently on different streams need different workspaces.
 */
SS_API int ss_attention_workspace_bytes(int device, int64_t tokens, int heads, int kv_heads,
                                 int head_dim, size_t* bytes);

/*
 * Ragged paged attention over a flat batch of query tokens.  Replaces
 * ragged_attention_direct(q, k_pool_layer, v_pool_layer, block_tables, query_seq_ids,
 * positions, sm_scale) (shardserve/kernel.py:11-82) and its kernel (kernel.py:85-166):
 * token t attends, for every head h, to the keys at absolute positions 0..positions[t] of
 * sequence row query_seq_ids[t], found through block_tables[row, p // 16] (page) and
 * p % 16 (row in page), using K/V head h / (heads / kv_heads).  Softmax is fp32 with scale
 * sm_scale; output is bf16.
 *
 * q            : bf16 [tokens, heads, head_dim]
 * k_pool/v_pool: bf16 [num_pages, 16, kv_heads, head_dim]
 * block_tables : [bt_rows, bt_cols] int32 (bt_is_int64 = 0) or int64 (= 1)
 * query_seq_ids: [tokens] int32 / int64 ; positions: [tokens] int32 / int64
 * out          : bf16 [tokens, heads, head_dim] (may not alias q)
 * head_dim in {64, 128}; heads % kv_heads == 0; tokens >= 1.
 * workspace    : >= ss_attention_workspace_bytes(...) bytes (see above).
 */
SS_API int ss_ragged_paged_attention(const void* q, const int64_t q_strides[3], const void* k_pool,
                              const int64_t k_pool_strides[4], const void* v_pool,
                              const int64_t v_pool_strides[4], const void* block_tables,
                              const int64_t bt_strides[2], int64_t bt_rows, int64_t bt_cols,
                              int bt_is_int64, const void* query_seq_ids, int seq_ids_is_int64,
                              const void* positions, int positions_is_int64, void* out,
                              const int64_t out_strides[3], int64_t tokens, int heads,
                              int kv_heads, int head_dim, int64_t num_pages, float sm_scale,
                              void* workspace, size_t workspace_bytes, void* stream);

/*
 * Slot-mapped KV append followed by ragged paged attention, in one call: the result of
 * ss_kv_append(k, v -> k_pool / v_pool at slots) then ss_ragged_paged_attention(...) with
 * the same arguments, the way the reference model calls them per layer
 * (cache.write then ragged_attention_direct, shardserve/model.py:32-37).
 * For decode-only launches (query tokens <= block-table rows) whose k / v rows have unit
 * stride along head_dim and 16-byte aligned starts (element strides multiples of 8), the
 * append runs inside the attention kernel: the CTA that loads a page writes the new rows of
 * its token's sequence that fall in that page before loading it, so no append kernel runs.
 * This needs slots[t] to be token t's own position in its row,
 * block_tables[seq, pos // 16] * 16 + pos % 16, as the reference builds them
 * (runtime.py:38); a slot that is not sets SS_DEVERR_SLOT (the row is still written to its
 * slot when it lies in the pool, but attention then reads the token's page without it).
 * Other launches run the append kernel first.  ss_last_attention_path() returns 4 when the
 * append was folded in.  No counterpart in the reference (it fuses two of its calls).
 * k, v : bf16 [tokens, kv_heads, head_dim]; slots: [tokens] int32 / int64; the rest as
 * ss_ragged_paged_attention (k_pool / v_pool are written).
 */
SS_API int ss_append_ragged_paged_attention(
    const void* k, const int64_t k_strides[3], const void* v, const int64_t v_strides[3],
    const void* slots, int slots_is_int64, const void* q, const int64_t q_strides[3],
    void* k_pool, const int64_t k_pool_strides[4], void* v_pool, const int64_t v_pool_strides[4],
    const void* block_tables, const int64_t bt_strides[2], int64_t bt_rows, int64_t bt_cols,
    int bt_is_int64, const void* query_seq_ids, int seq_ids_is_int64, const void* positions,
    int positions_is_int64, void* out, const int64_t out_strides[3], int64_t tokens, int heads,
    int kv_heads, int head_dim, int64_t num_pages, float sm_scale, void* workspace,
    size_t workspace_bytes, void* stream);

/*
 * ss_ragged_paged_attention without a workspace argument: allocation-free.  No counterpart
 * in the reference; it exists for callers that cannot allocate device memory around the
 * call, such as code being recorded into a CUDA graph (cudaMalloc is illegal during stream
 * capture), serving loops that plan all device memory ahead and must never stall on an
 * allocator, and plain C / FFI hosts without a caching allocator to keep a workspace alive.
 *
 * The split-K scratch is a fixed 16 MiB array of this library's own device memory
 * (file-scope __device__ storage, present on every GPU that loads the library until the
 * process exits).  Calls whose scratch need (ss_attention_workspace_bytes) exceeds it are
 * rejected with SS_ERR_WORKSPACE and a message; use ss_ragged_paged_attention instead.
 * The first call on a device looks up the array's device address (cudaGetSymbolAddress) and
 * the kernels' launch attributes; make that first call before any stream capture.  All
 * calls on a device share the one array and each call overwrites its scratch part, so
 * calls that can overlap on the GPU (different streams, or concurrent graph replays) race
 * and must be serialised by the caller.  The array's error word (SS_DEVERR_* bits) starts
 * at zero when the library loads and collects the bits of every call on the device until
 * ss_noalloc_fetch_device_errors reads and clears it.
 * Arguments and results are those of ss_ragged_paged_attention.
 */
SS_API int ss_ragged_paged_attention_noalloc(
    const void* q, const int64_t q_strides[3], const void* k_pool, const int64_t k_pool_strides[4],
    const void* v_pool, const int64_t v_pool_strides[4], const void* block_tables,
    const int64_t bt_strides[2], int64_t bt_rows, int64_t bt_cols, int bt_is_int64,
    const void* query_seq_ids, int seq_ids_is_int64, const void* positions,
    int positions_is_int64, void* out, const int64_t out_strides[3], int64_t tokens, int heads,
    int kv_heads, int head_dim, int64_t num_pages, float sm_scale, void* stream);

/*
 * Reads (and, if clear != 0, zeroes) the device error word at the start of `workspace`.
 * Synchronises `stream`.  For tests and debugging, not for the hot path.
 */
SS_API int ss_fetch_device_errors(void* workspace, int clear, uint32_t* flags, void* stream);

/*
 * The error word of ss_ragged_paged_attention_noalloc's fixed scratch on `device`: reads the
 * SS_DEVERR_* bits its calls on that device have collected and, if clear != 0, zeroes them.
 * No counterpart in the reference (it completes the allocation-free entry point, whose
 * callers have no workspace pointer to pass to ss_fetch_device_errors).  Synchronises
 * `stream` (a stream of `device`); for tests and debugging, not for the hot path.
 */
SS_API int ss_noalloc_fetch_device_errors(int device, int clear, uint32_t* flags, void* stream);

/*
 * Which kernel family the last successful ss_ragged_paged_attention call on this thread
 * used: 1 = TMA/tensor-core split-K kernel, 2 = generic strided kernel (layouts the TMA
 * path cannot describe), 3 = split-K kernel for isolated tokens plus tcgen05 tiles for the
 * chunked-prefill runs, 4 = split-K kernel with the KV append folded in
 * (ss_append_ragged_paged_attention), 0 = none yet.  Lets tests assert the fast path really ran.
 */
SS_API int ss_last_attention_path(void);

/*
 * Kernels this library has enqueued since it was loaded (every entry point, all threads;
 * a launch recorded into a CUDA graph counts once, when it is recorded).  Lets a benchmark
 * state how many of its own kernels one step runs.  No counterpart in the reference.
 */
SS_API unsigned long long ss_kernel_launch_count(void);

#ifdef __cplusplus
}
#endif

#endif /* SHARDSERVE_B200_H */
