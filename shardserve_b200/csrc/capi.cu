// C ABI (include/shardserve_b200.h): argument validation, TMA descriptor encoding and
// kernel dispatch.  Validation mirrors the reference wrapper (shardserve/kernel.py:28-49);
// the Python layer raises KernelUnsupported before calling here, so the checks below are
// the last line for C callers.
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "attention.cuh"

namespace {

thread_local std::string g_message;
thread_local int g_last_path = 0;
// Kernels this library has enqueued (launched, or recorded into a stream capture).
std::atomic<unsigned long long> g_launches{0};
void count_launch(unsigned n = 1) { g_launches.fetch_add(n, std::memory_order_relaxed); }

int fail(int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_message = buf;
  return status;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(SS_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static std::once_flag once;
  static EncodeTiledFn fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 5-D view of a pool [N, 16, KVH, D] (element strides sn, ss, sh, 1) whose box is one page
// of `kvb` heads laid out as [head][d / 64][key][d % 64] in shared memory with the 128-byte
// swizzle: each 128-byte line holds 64 values of one key, and the 8 keys an ldmatrix reads
// fall in 8 different swizzle phases (bank-conflict free).
// `dhalves` = 64-dim halves per box: D / 64 for the decode kernel (whole page of `kvb` heads),
// 1 for the prefill tiles (one half of one head per box).
bool encode_pool_map(CUtensorMap* map, const void* base, long long N, int KVH, int D,
                     const int64_t* st, int kvb, int dhalves) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[5] = {64, 16, static_cast<cuuint64_t>(D / 64), static_cast<cuuint64_t>(KVH),
                        static_cast<cuuint64_t>(N)};
  cuuint64_t strides[4] = {static_cast<cuuint64_t>(st[1]) * 2, 64 * 2,
                           static_cast<cuuint64_t>(st[2]) * 2, static_cast<cuuint64_t>(st[0]) * 2};
  cuuint32_t box[5] = {64, 16, static_cast<cuuint32_t>(dhalves), static_cast<cuuint32_t>(kvb), 1};
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 5, const_cast<void*>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// q [T, H, D] as (d % 64, d / 64, head, token) with a box of 64 dims x 8 heads x 16 tokens
// for the prefill tiles (rows = token * 8 + head, 128-byte swizzle).
bool encode_q_map(CUtensorMap* map, const void* q, long long T, int H, int D, const int64_t* st) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[4] = {64, static_cast<cuuint64_t>(D / 64), static_cast<cuuint64_t>(H),
                        static_cast<cuuint64_t>(T)};
  cuuint64_t strides[3] = {64 * 2, static_cast<cuuint64_t>(st[1]) * 2,
                           static_cast<cuuint64_t>(st[0]) * 2};
  cuuint32_t box[4] = {64, 1, 8, 16};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(q), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Can the TMA kernel address this pool?  Unit stride along head_dim, every other stride a
// multiple of 8 elements (16 bytes), 16-byte aligned base, strides below 2^39 elements.
bool pool_tma_ok(const void* base, const int64_t* st) {
  if (st[3] != 1) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) return false;
  for (int i = 0; i < 3; ++i) {
    if (st[i] <= 0 || (st[i] % 8) != 0 || st[i] >= (1LL << 39)) return false;
  }
  return true;
}

bool finite_nonneg_strides(const int64_t* st, int n) {
  for (int i = 0; i < n; ++i)
    if (st[i] < 0) return false;
  return true;
}

}  // namespace

namespace ss {
void set_error_message(const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_message = buf;
}
}  // namespace ss

extern "C" {

int ss_version(void) { return 100; }

const char* ss_status_string(int status) {
  switch (status) {
    case SS_OK: return "ok";
    case SS_ERR_INVALID: return "invalid argument";
    case SS_ERR_UNSUPPORTED: return "unsupported";
    case SS_ERR_CUDA: return "CUDA error";
    case SS_ERR_WORKSPACE: return "workspace too small";
    default: return "unknown status";
  }
}

const char* ss_last_error_message(void) { return g_message.c_str(); }

int ss_last_attention_path(void) { return g_last_path; }

unsigned long long ss_kernel_launch_count(void) {
  return g_launches.load(std::memory_order_relaxed);
}

int ss_kv_append(const void* k, const int64_t k_strides[3], const void* v,
                 const int64_t v_strides[3], void* k_pool, const int64_t k_pool_strides[4],
                 void* v_pool, const int64_t v_pool_strides[4], const void* slots,
                 int slots_is_int64, int64_t tokens, int64_t num_pages, int kv_heads,
                 int head_dim, void* workspace, void* stream) {
  if (tokens < 0) return fail(SS_ERR_INVALID, "tokens must be >= 0");
  if (tokens == 0) return SS_OK;
  if (!k || !v || !k_pool || !v_pool || !slots || !k_strides || !v_strides || !k_pool_strides ||
      !v_pool_strides)
    return fail(SS_ERR_INVALID, "null pointer argument");
  if (kv_heads < 1 || head_dim < 1 || num_pages < 1)
    return fail(SS_ERR_INVALID, "kv_heads, head_dim and num_pages must be positive");
  if (!finite_nonneg_strides(k_strides, 3) || !finite_nonneg_strides(v_strides, 3) ||
      !finite_nonneg_strides(k_pool_strides, 4) || !finite_nonneg_strides(v_pool_strides, 4))
    return fail(SS_ERR_INVALID, "negative strides are not supported");
  ss::AppendArgs a;
  a.k = static_cast<const __nv_bfloat16*>(k);
  a.k_st = k_strides[0]; a.k_sh = k_strides[1]; a.k_sd = k_strides[2];
  a.v = static_cast<const __nv_bfloat16*>(v);
  a.v_st = v_strides[0]; a.v_sh = v_strides[1]; a.v_sd = v_strides[2];
  a.kp = static_cast<__nv_bfloat16*>(k_pool);
  a.kp_sn = k_pool_strides[0]; a.kp_ss = k_pool_strides[1];
  a.kp_sh = k_pool_strides[2]; a.kp_sd = k_pool_strides[3];
  a.vp = static_cast<__nv_bfloat16*>(v_pool);
  a.vp_sn = v_pool_strides[0]; a.vp_ss = v_pool_strides[1];
  a.vp_sh = v_pool_strides[2]; a.vp_sd = v_pool_strides[3];
  a.slots = slots;
  a.slots64 = slots_is_int64 ? 1 : 0;
  a.T = tokens;
  a.N = num_pages;
  a.KVH = kv_heads;
  a.D = head_dim;
  a.err = workspace ? static_cast<unsigned*>(workspace) : nullptr;
  auto vec_ok = [](const void* p, const int64_t* st, int n) {
    if ((reinterpret_cast<uintptr_t>(p) & 15) != 0 || st[n - 1] != 1) return false;
    for (int i = 0; i < n - 1; ++i)
      if (st[i] % 8) return false;
    return true;
  };
  const bool vec = (head_dim % 8 == 0) && vec_ok(k, k_strides, 3) && vec_ok(v, v_strides, 3) &&
                   vec_ok(k_pool, k_pool_strides, 4) && vec_ok(v_pool, v_pool_strides, 4);
  const cudaError_t e = ss::launch_kv_append(a, vec, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "kv_append launch");
  count_launch();
  return SS_OK;
}

int ss_rope_kv_append(const void* q, const int64_t q_strides[3], void* q_out,
                      const int64_t q_out_strides[3], const void* k, const int64_t k_strides[3],
                      const void* v, const int64_t v_strides[3], const float* cos_table,
                      const int64_t cos_strides[2], const float* sin_table,
                      const int64_t sin_strides[2], int64_t table_rows, const void* positions,
                      int positions_is_int64, void* k_pool, const int64_t k_pool_strides[4],
                      void* v_pool, const int64_t v_pool_strides[4], const void* slots,
                      int slots_is_int64, int64_t tokens, int heads, int kv_heads, int head_dim,
                      int64_t num_pages, void* workspace, void* stream) {
  if (tokens < 0) return fail(SS_ERR_INVALID, "tokens must be >= 0");
  if (tokens == 0) return SS_OK;
  if (!q || !q_out || !k || !v || !cos_table || !sin_table || !positions || !k_pool ||
      !v_pool || !slots || !q_strides || !q_out_strides || !k_strides || !v_strides ||
      !cos_strides || !sin_strides || !k_pool_strides || !v_pool_strides)
    return fail(SS_ERR_INVALID, "null pointer argument");
  if (heads < 1 || kv_heads < 1 || num_pages < 1 || table_rows < 1)
    return fail(SS_ERR_INVALID, "heads, kv_heads, num_pages and table_rows must be positive");
  if (head_dim < 2 || head_dim % 2)
    return fail(SS_ERR_INVALID, "head_dim must be even (RoPE rotates the two halves)");
  if (!finite_nonneg_strides(q_strides, 3) || !finite_nonneg_strides(q_out_strides, 3) ||
      !finite_nonneg_strides(k_strides, 3) || !finite_nonneg_strides(v_strides, 3) ||
      !finite_nonneg_strides(cos_strides, 2) || !finite_nonneg_strides(sin_strides, 2) ||
      !finite_nonneg_strides(k_pool_strides, 4) || !finite_nonneg_strides(v_pool_strides, 4))
    return fail(SS_ERR_INVALID, "negative strides are not supported");
  ss::RopeArgs r;
  ss::AppendArgs& a = r.app;
  a.k = static_cast<const __nv_bfloat16*>(k);
  a.k_st = k_strides[0]; a.k_sh = k_strides[1]; a.k_sd = k_strides[2];
  a.v = static_cast<const __nv_bfloat16*>(v);
  a.v_st = v_strides[0]; a.v_sh = v_strides[1]; a.v_sd = v_strides[2];
  a.kp = static_cast<__nv_bfloat16*>(k_pool);
  a.kp_sn = k_pool_strides[0]; a.kp_ss = k_pool_strides[1];
  a.kp_sh = k_pool_strides[2]; a.kp_sd = k_pool_strides[3];
  a.vp = static_cast<__nv_bfloat16*>(v_pool);
  a.vp_sn = v_pool_strides[0]; a.vp_ss = v_pool_strides[1];
  a.vp_sh = v_pool_strides[2]; a.vp_sd = v_pool_strides[3];
  a.slots = slots;
  a.slots64 = slots_is_int64 ? 1 : 0;
  a.T = tokens;
  a.N = num_pages;
  a.KVH = kv_heads;
  a.D = head_dim;
  a.err = workspace ? static_cast<unsigned*>(workspace) : nullptr;
  r.q = static_cast<const __nv_bfloat16*>(q);
  r.q_st = q_strides[0]; r.q_sh = q_strides[1]; r.q_sd = q_strides[2];
  r.qo = static_cast<__nv_bfloat16*>(q_out);
  r.qo_st = q_out_strides[0]; r.qo_sh = q_out_strides[1]; r.qo_sd = q_out_strides[2];
  r.cos = cos_table;
  r.cos_sr = cos_strides[0]; r.cos_sd = cos_strides[1];
  r.sin = sin_table;
  r.sin_sr = sin_strides[0]; r.sin_sd = sin_strides[1];
  r.rows = table_rows;
  r.pos = positions;
  r.pos64 = positions_is_int64 ? 1 : 0;
  r.H = heads;
  auto vec_ok = [](const void* p, const int64_t* st, int n, int mult) {
    if ((reinterpret_cast<uintptr_t>(p) & 15) != 0 || st[n - 1] != 1) return false;
    for (int i = 0; i < n - 1; ++i)
      if (st[i] % mult) return false;
    return true;
  };
  const bool vec = (head_dim % 16 == 0) && vec_ok(q, q_strides, 3, 8) &&
                   vec_ok(q_out, q_out_strides, 3, 8) && vec_ok(k, k_strides, 3, 8) &&
                   vec_ok(v, v_strides, 3, 8) && vec_ok(k_pool, k_pool_strides, 4, 8) &&
                   vec_ok(v_pool, v_pool_strides, 4, 8) && vec_ok(cos_table, cos_strides, 2, 4) &&
                   vec_ok(sin_table, sin_strides, 2, 4);
  const cudaError_t e = ss::launch_rope_append(r, vec, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "rope_kv_append launch");
  count_launch();
  return SS_OK;
}

int ss_build_metadata(const int64_t* packed, int64_t rows, int64_t n_selected, int64_t tokens,
                      const int32_t* store, const int32_t* store_lens, int64_t store_rows,
                      int64_t store_row_stride, int64_t pad_block_base, int32_t* tables,
                      int64_t table_cols, int64_t table_row_stride, int64_t* ids,
                      int64_t* positions, int32_t* seqs, int64_t* slots, int64_t* selected,
                      void* workspace, void* stream) {
  if (rows < 0 || n_selected < 0 || tokens < 0 || table_cols < 1 || store_rows < 0)
    return fail(SS_ERR_INVALID, "negative size or empty table width");
  if (rows == 0) return SS_OK;
  if (!packed || !tables || (tokens > 0 && (!ids || !positions || !seqs || !slots)) ||
      (n_selected > 0 && !selected) || (store_rows > 0 && (!store || !store_lens)))
    return fail(SS_ERR_INVALID, "null pointer argument");
  if (table_row_stride < table_cols || (store_rows > 0 && store_row_stride < 1))
    return fail(SS_ERR_INVALID, "row strides must cover the rows");
  ss::MetadataArgs m;
  m.packed = reinterpret_cast<const long long*>(packed);
  m.rows = rows;
  m.n_sel = n_selected;
  m.tokens = tokens;
  m.store = store;
  m.store_lens = store_lens;
  m.store_rows = store_rows;
  m.store_rs = store_row_stride;
  m.pad_base = pad_block_base;
  m.tables = tables;
  m.table_cols = table_cols;
  m.table_rs = table_row_stride;
  m.ids = reinterpret_cast<long long*>(ids);
  m.positions = reinterpret_cast<long long*>(positions);
  m.seqs = seqs;
  m.slots = reinterpret_cast<long long*>(slots);
  m.selected = reinterpret_cast<long long*>(selected);
  m.err = workspace ? static_cast<unsigned*>(workspace) : nullptr;
  const cudaError_t e = ss::launch_build_metadata(m, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "build_metadata launch");
  count_launch();
  return SS_OK;
}

int ss_device_alloc_zeroed(size_t bytes, void** ptr) {
  if (!ptr || bytes == 0) return fail(SS_ERR_INVALID, "ptr is null or bytes is zero");
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e == cudaSuccess) e = cudaMemset(*ptr, 0, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "device allocation");
  return SS_OK;
}

int ss_device_free(void* ptr) {
  const cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? SS_OK : cuda_fail(e, "cudaFree");
}

int ss_ipc_handle(void* ptr, void* handle64) {
  if (!ptr || !handle64) return fail(SS_ERR_INVALID, "null pointer argument");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, ptr);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
  static_assert(sizeof(h) == 64, "IPC handles are 64 bytes");
  memcpy(handle64, &h, sizeof(h));
  return SS_OK;
}

int ss_ipc_open(const void* handle64, void** ptr) {
  if (!ptr || !handle64) return fail(SS_ERR_INVALID, "null pointer argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  return e == cudaSuccess ? SS_OK : cuda_fail(e, "cudaIpcOpenMemHandle");
}

int ss_ipc_close(void* ptr) {
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  return e == cudaSuccess ? SS_OK : cuda_fail(e, "cudaIpcCloseMemHandle");
}

namespace {
// Row-major bf16 matrix [rows, cols] (unit column stride) as a 3-D TMA map (64 columns,
// rows, column atoms of 64) whose box is box_rows rows x `atoms` atoms: shared memory gets
// [atom][row][128 B] with the 128-byte swizzle.
bool encode_rows_map(CUtensorMap* map, const void* base, long long rows, long long cols,
                     long long row_stride, int box_rows, int atoms) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {64, static_cast<cuuint64_t>(rows), static_cast<cuuint64_t>(cols / 64)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(row_stride) * 2, 128};
  cuuint32_t box[3] = {64, static_cast<cuuint32_t>(box_rows), static_cast<cuuint32_t>(atoms)};
  cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
}  // namespace

int ss_tp2_oproj_allreduce(const void* attn, const int64_t attn_strides[2], const void* w_o,
                           const int64_t w_strides[2], void* out, const int64_t out_strides[2],
                           int64_t tokens, int out_features, int in_features,
                           const void* local_inbox, void* peer_inbox, int64_t max_tokens,
                           void* epoch_counter, void* workspace, void* stream) {
  if (tokens < 0) return fail(SS_ERR_INVALID, "tokens must be >= 0");
  if (tokens == 0) return SS_OK;
  if (!attn || !w_o || !out || !local_inbox || !peer_inbox || !attn_strides || !w_strides ||
      !out_strides || !workspace || !epoch_counter)
    return fail(SS_ERR_INVALID, "null pointer argument");
  const int tn = ss::oproj_tile_n(tokens), tm = ss::oproj_tile_tokens();
  const int ks = ss::oproj_min_k_step();
  if (out_features < 128 || out_features % 128 || in_features < 4 * ks / 2 ||
      in_features % (2 * ks))
    return fail(SS_ERR_INVALID, "out_features must be a multiple of 128 and in_features of %d",
                2 * ks);
  if (tokens > max_tokens) return fail(SS_ERR_INVALID, "tokens exceed the inbox capacity");
  const long long tiles = (tokens + tm - 1) / tm * (out_features / tn);
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return fail(SS_ERR_CUDA, "device query failed");
  if (tiles > sms)
    return fail(SS_ERR_INVALID, "%lld tiles exceed one wave of %d SMs (both ranks' tiles must "
                "be resident together)", tiles, sms);
  if (attn_strides[0] < in_features || w_strides[0] < in_features ||
      out_strides[0] < out_features)
    return fail(SS_ERR_INVALID, "row strides must cover a row");
  auto ok16 = [](const void* p, const int64_t* st) {
    return (reinterpret_cast<uintptr_t>(p) & 15) == 0 && st[1] == 1 && st[0] % 8 == 0 && st[0] > 0;
  };
  if (!ok16(attn, attn_strides) || !ok16(w_o, w_strides) || !ok16(out, out_strides))
    return fail(SS_ERR_INVALID, "attn, w_o and out need unit column stride, row strides that "
                "are multiples of 8 elements and 16-byte aligned bases");
  // Rows of the attention tile actually loaded: all 128 MMA rows only when the call has
  // them; rows past it hold stale shared memory and give output rows that are never stored.
  const int a_rows = static_cast<int>(tokens >= tm ? tm : (tokens + 7) / 8 * 8);
  int atoms = 0, stages = 0;
  ss::oproj_ring(a_rows, tn, in_features, &atoms, &stages);
  CUtensorMap tmA, tmW;
  if (!encode_rows_map(&tmA, attn, tokens, in_features, attn_strides[0], a_rows, atoms) ||
      !encode_rows_map(&tmW, w_o, out_features, in_features, w_strides[0], tn, atoms))
    return fail(SS_ERR_INVALID, "tensor map encoding failed");
  ss::OprojArgs o;
  o.T = tokens;
  o.T_max = max_tokens;
  o.N = out_features;
  o.K = in_features;
  o.out = static_cast<__nv_bfloat16*>(out);
  o.out_rs = out_strides[0];
  o.local_inbox = local_inbox;
  o.peer_inbox = peer_inbox;
  o.a_rows = a_rows;
  o.tile_n = tn;
  o.atoms = atoms;
  o.stages = stages;
  o.epoch_ctr = static_cast<unsigned*>(epoch_counter);
  o.err = static_cast<unsigned*>(workspace);
  const cudaError_t e = ss::launch_tp2_oproj(tmA, tmW, o, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "tp2_oproj launch");
  count_launch();
  return SS_OK;
}

int ss_attention_workspace_bytes(int device, int64_t tokens, int heads, int kv_heads,
                                 int head_dim, size_t* bytes) {
  if (!bytes) return fail(SS_ERR_INVALID, "bytes is null");
  if (tokens < 1 || heads < 1 || kv_heads < 1 || heads % kv_heads)
    return fail(SS_ERR_INVALID, "invalid geometry");
  ss::DecodeGeometry g;
  const char* why = "";
  size_t need = ss::kWsHeader;
  if (ss::decode_geometry(device, tokens, heads, kv_heads, head_dim, false, &g, &why))
    need += g.desc_bytes + g.part_bytes;
  *bytes = need;
  return SS_OK;
}

}  // extern "C"

namespace {

// The step's new K/V rows of ss_append_ragged_paged_attention.
struct AppendIn {
  const void* k;
  const int64_t* ks;
  const void* v;
  const int64_t* vs;
  const void* slots;
  int slots64;
};

int attention_impl(const void* q, const int64_t q_strides[3], const void* k_pool,
                   const int64_t k_pool_strides[4], const void* v_pool,
                   const int64_t v_pool_strides[4], const void* block_tables,
                   const int64_t bt_strides[2], int64_t bt_rows, int64_t bt_cols, int bt_is_int64,
                   const void* query_seq_ids, int seq_ids_is_int64, const void* positions,
                   int positions_is_int64, void* out, const int64_t out_strides[3],
                   int64_t tokens, int heads, int kv_heads, int head_dim, int64_t num_pages,
                   float sm_scale, void* workspace, size_t workspace_bytes, void* stream,
                   const AppendIn* app) {
  // Checks of the reference wrapper, kernel.py:28-49 (dtype/device checks live in Python).
  if (head_dim != 64 && head_dim != 128)
    return fail(SS_ERR_INVALID, "ragged q must be [tokens, heads, 64|128], got head_dim %d", head_dim);
  if (tokens < 1) return fail(SS_ERR_INVALID, "ragged batch cannot be empty");
  if (heads < 1 || kv_heads < 1 || heads % kv_heads)
    return fail(SS_ERR_INVALID, "query heads must be divisible by KV heads");
  if (bt_rows < 1 || bt_cols < 1) return fail(SS_ERR_INVALID, "block_tables must be non-empty");
  if (num_pages < 1) return fail(SS_ERR_INVALID, "KV pool must hold at least one page");
  if (!q || !k_pool || !v_pool || !block_tables || !query_seq_ids || !positions || !out ||
      !q_strides || !k_pool_strides || !v_pool_strides || !bt_strides || !out_strides)
    return fail(SS_ERR_INVALID, "null pointer argument");
  if (!workspace || workspace_bytes < ss::kWsHeader)
    return fail(SS_ERR_WORKSPACE, "a workspace of at least %zu bytes is required", ss::kWsHeader);
  if (!std::isfinite(sm_scale)) return fail(SS_ERR_INVALID, "sm_scale must be finite");
  if (!finite_nonneg_strides(q_strides, 3) || !finite_nonneg_strides(k_pool_strides, 4) ||
      !finite_nonneg_strides(v_pool_strides, 4) || !finite_nonneg_strides(bt_strides, 2) ||
      !finite_nonneg_strides(out_strides, 3))
    return fail(SS_ERR_INVALID, "negative strides are not supported");

  ss::AttnArgs a;
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.q_st = q_strides[0]; a.q_sh = q_strides[1]; a.q_sd = q_strides[2];
  a.bt = block_tables;
  a.bt_sb = bt_strides[0]; a.bt_sn = bt_strides[1];
  a.bt64 = bt_is_int64 ? 1 : 0;
  a.seq = query_seq_ids; a.seq64 = seq_ids_is_int64 ? 1 : 0;
  a.pos = positions; a.pos64 = positions_is_int64 ? 1 : 0;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.o_st = out_strides[0]; a.o_sh = out_strides[1]; a.o_sd = out_strides[2];
  a.kp = static_cast<const __nv_bfloat16*>(k_pool);
  a.k_sn = k_pool_strides[0]; a.k_ss = k_pool_strides[1];
  a.k_sh = k_pool_strides[2]; a.k_sd = k_pool_strides[3];
  a.vp = static_cast<const __nv_bfloat16*>(v_pool);
  a.v_sn = v_pool_strides[0]; a.v_ss = v_pool_strides[1];
  a.v_sh = v_pool_strides[2]; a.v_sd = v_pool_strides[3];
  a.T = tokens; a.B = bt_rows; a.W = bt_cols; a.N = num_pages;
  a.H = heads; a.KVH = kv_heads; a.D = head_dim; a.group = heads / kv_heads;
  a.sm_scale = sm_scale;
  a.scale_log2 = sm_scale * 1.4426950408889634f;
  a.err = static_cast<unsigned*>(workspace);
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");

  // ---- fast path: TMA + tensor-core split-K kernel ------------------------------------
  ss::DecodeGeometry g;
  const char* why = "";
  // The split-K kernel reads q rows and writes output rows as vectors: unit head_dim
  // stride, head and token strides multiples of 8 elements, 16-byte aligned base (other
  // layouts run on the generic kernel).
  auto rows16_ok = [](const void* p, const int64_t* st) {
    return st[2] == 1 && st[1] % 8 == 0 && st[0] % 8 == 0 &&
           (reinterpret_cast<uintptr_t>(p) & 15) == 0;
  };
  const bool tma_layout = rows16_ok(q, q_strides) && rows16_ok(out, out_strides) &&
                          pool_tma_ok(k_pool, k_pool_strides) && pool_tma_ok(v_pool, v_pool_strides);
  // Chunked-prefill tiles when the batch must hold a multi-token run (more query tokens than
  // sequence rows) and the layout suits the tile kernel; the decode kernel then takes its
  // wide configuration on half of the SMs so that the tiles start on the other half at once.
  const bool want_prefill = tokens > bt_rows && ss::prefill_supported(a);
  // The append folds into the decode kernel for decode-only launches whose new rows are
  // 16-byte addressable; otherwise the append kernel runs first.
  auto rows16 = [](const void* p, const int64_t* st) {
    return (reinterpret_cast<uintptr_t>(p) & 15) == 0 && st[2] == 1 && st[1] % 8 == 0 &&
           st[0] % 8 == 0;
  };
  const bool fuse = app && tma_layout && !want_prefill && rows16(app->k, app->ks) &&
                    rows16(app->v, app->vs);
  if (app && !fuse) {
    const int rc = ss_kv_append(app->k, app->ks, app->v, app->vs, const_cast<void*>(k_pool),
                                k_pool_strides, const_cast<void*>(v_pool), v_pool_strides,
                                app->slots, app->slots64, tokens, num_pages, kv_heads, head_dim,
                                workspace, stream);
    if (rc != SS_OK) return rc;
  }
  if (tma_layout &&
      ss::decode_geometry(device, tokens, heads, kv_heads, head_dim, want_prefill, &g, &why)) {
    const size_t need = ss::kWsHeader + g.desc_bytes + g.part_bytes;
    if (workspace_bytes < need)
      return fail(SS_ERR_WORKSPACE, "workspace holds %zu bytes, %zu needed", workspace_bytes, need);
    CUtensorMap tmK, tmV;
    if (encode_pool_map(&tmK, k_pool, num_pages, kv_heads, head_dim, k_pool_strides, g.kvb,
                        head_dim / 64) &&
        encode_pool_map(&tmV, v_pool, num_pages, kv_heads, head_dim, v_pool_strides, g.kvb,
                        head_dim / 64)) {
      // Otherwise the split-K kernel computes every token.  Only the wide decode shape
      // evaluates the run predicate, so tiles run only beside it.
      CUtensorMap tmQ, tmKp, tmVp;
      const bool prefill = want_prefill && g.pr > 2 &&
                           encode_q_map(&tmQ, q, tokens, heads, head_dim, q_strides) &&
                           encode_pool_map(&tmKp, k_pool, num_pages, kv_heads, head_dim,
                                           k_pool_strides, 1, 1) &&
                           encode_pool_map(&tmVp, v_pool, num_pages, kv_heads, head_dim,
                                           v_pool_strides, 1, 1);
      ss::DecodeArgs d;
      d.a = a;
      d.kvb = g.kvb;
      d.nkvblk = g.nkvblk;
      d.min_run = prefill ? ss::prefill_min_run() : 0;
      d.lo_ctas = g.G;
      d.wide_per = 1;
      if (g.pr > 2) d.lo_ctas = ss::wide_grid(&g, device, bt_rows, bt_cols, tokens, &d.wide_per);
      d.G = g.G;
      uint8_t* ws = static_cast<uint8_t*>(workspace);
      d.part = reinterpret_cast<float*>(ws + ss::kWsHeader);
      d.desc = reinterpret_cast<int4*>(ws + ss::kWsHeader + g.part_bytes);
      d.gbar = reinterpret_cast<unsigned*>(ws + 72);
      d.app_k = nullptr;
      d.app_v = nullptr;
      d.ak_st = d.ak_sh = d.av_st = d.av_sh = 0;
      d.app_slots = nullptr;
      d.app_slots64 = 0;
      if (fuse) {
        d.app_k = static_cast<const __nv_bfloat16*>(app->k);
        d.app_v = static_cast<const __nv_bfloat16*>(app->v);
        d.ak_st = app->ks[0];
        d.ak_sh = app->ks[1];
        d.av_st = app->vs[0];
        d.av_sh = app->vs[1];
        d.app_slots = app->slots;
        d.app_slots64 = app->slots64;
      }
      e = ss::launch_decode(g, tmK, tmV, d, s);
      if (e != cudaSuccess) return cuda_fail(e, "decode attention launch");
      count_launch();
      if (prefill) {
        e = ss::launch_prefill(tmQ, tmKp, tmVp, a, s);
        if (e != cudaSuccess) return cuda_fail(e, "prefill attention launch");
        count_launch();
      }
      g_last_path = prefill ? 3 : (fuse ? 4 : 1);
      return SS_OK;
    }
  }
  // ---- generic strided path -------------------------------------------------------------
  if (fuse) {  // the TMA path was not taken after all: append first, then the generic kernel
    const int rc = ss_kv_append(app->k, app->ks, app->v, app->vs, const_cast<void*>(k_pool),
                                k_pool_strides, const_cast<void*>(v_pool), v_pool_strides,
                                app->slots, app->slots64, tokens, num_pages, kv_heads, head_dim,
                                workspace, stream);
    if (rc != SS_OK) return rc;
  }
  e = ss::launch_generic_attention(a, s);
  if (e != cudaSuccess) return cuda_fail(e, "generic attention launch");
  count_launch();
  g_last_path = 2;
  return SS_OK;
}

}  // namespace

extern "C" {

int ss_ragged_paged_attention(const void* q, const int64_t q_strides[3], const void* k_pool,
                              const int64_t k_pool_strides[4], const void* v_pool,
                              const int64_t v_pool_strides[4], const void* block_tables,
                              const int64_t bt_strides[2], int64_t bt_rows, int64_t bt_cols,
                              int bt_is_int64, const void* query_seq_ids, int seq_ids_is_int64,
                              const void* positions, int positions_is_int64, void* out,
                              const int64_t out_strides[3], int64_t tokens, int heads,
                              int kv_heads, int head_dim, int64_t num_pages, float sm_scale,
                              void* workspace, size_t workspace_bytes, void* stream) {
  return attention_impl(q, q_strides, k_pool, k_pool_strides, v_pool, v_pool_strides,
                        block_tables, bt_strides, bt_rows, bt_cols, bt_is_int64, query_seq_ids,
                        seq_ids_is_int64, positions, positions_is_int64, out, out_strides,
                        tokens, heads, kv_heads, head_dim, num_pages, sm_scale, workspace,
                        workspace_bytes, stream, nullptr);
}

int ss_append_ragged_paged_attention(
    const void* k, const int64_t k_strides[3], const void* v, const int64_t v_strides[3],
    const void* slots, int slots_is_int64, const void* q, const int64_t q_strides[3],
    void* k_pool, const int64_t k_pool_strides[4], void* v_pool, const int64_t v_pool_strides[4],
    const void* block_tables, const int64_t bt_strides[2], int64_t bt_rows, int64_t bt_cols,
    int bt_is_int64, const void* query_seq_ids, int seq_ids_is_int64, const void* positions,
    int positions_is_int64, void* out, const int64_t out_strides[3], int64_t tokens, int heads,
    int kv_heads, int head_dim, int64_t num_pages, float sm_scale, void* workspace,
    size_t workspace_bytes, void* stream) {
  if (!k || !v || !slots || !k_strides || !v_strides)
    return fail(SS_ERR_INVALID, "null pointer argument");
  if (!finite_nonneg_strides(k_strides, 3) || !finite_nonneg_strides(v_strides, 3))
    return fail(SS_ERR_INVALID, "negative strides are not supported");
  const AppendIn app{k, k_strides, v, v_strides, slots, slots_is_int64 ? 1 : 0};
  return attention_impl(q, q_strides, k_pool, k_pool_strides, v_pool, v_pool_strides,
                        block_tables, bt_strides, bt_rows, bt_cols, bt_is_int64, query_seq_ids,
                        seq_ids_is_int64, positions, positions_is_int64, out, out_strides,
                        tokens, heads, kv_heads, head_dim, num_pages, sm_scale, workspace,
                        workspace_bytes, stream, &app);
}

int ss_fetch_device_errors(void* workspace, int clear, uint32_t* flags, void* stream) {
  if (!workspace || !flags) return fail(SS_ERR_INVALID, "null pointer argument");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint32_t host = 0;
  cudaError_t e = cudaMemcpyAsync(&host, workspace, sizeof(host), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e == cudaSuccess && clear) e = cudaMemsetAsync(workspace, 0, sizeof(uint32_t), s);
  if (e == cudaSuccess && clear) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, "reading the device error word");
  *flags = host;
  return SS_OK;
}

}  // extern "C"
