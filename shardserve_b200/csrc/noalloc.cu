// Allocation-free variant of ss_ragged_paged_attention.
//
// Who needs it: callers that must not allocate device memory on their hot path.  Examples
// are a host runtime that records its decode step into a CUDA graph (cudaMalloc is not
// allowed while a stream is being captured), a serving loop that plans all device memory up
// front and treats any allocation as a stall (cudaMalloc/cudaFree can synchronise the whole
// device), and thin FFI hosts (C, Go, Java, ...) that have no caching allocator of their own
// and no convenient place to keep a workspace buffer alive between calls.
//
// How: the split-K scratch lives in a fixed-size array in this library's own device memory
// (file-scope __device__ storage), and the call passes that array as the workspace of the
// ordinary entry point.  The array exists on every GPU that loads this library, from load
// until process exit, whether or not this entry point is used.  It is zero when the library
// loads; every call leaves the chunked-prefill work counter in it at zero, and the error
// word at its start collects SS_DEVERR_* bits across calls until
// ss_noalloc_fetch_device_errors reads and clears it.
#include <cuda_runtime.h>

#include <mutex>

#include "attention.cuh"

namespace {

// Scratch of the allocation-free path: 16 MiB, enough for the split-K partial states of
// the largest decode kernel instance on a 148-SM B200 plus the per-row split descriptors
// of ~120 000 (token, KV-head block) rows.  Larger calls are rejected.
constexpr size_t kScratchBytes = static_cast<size_t>(16) << 20;
static __device__ __align__(256) unsigned char g_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of g_scratch on `device`, which must be the current device, looked up once
// per device.  The host symbol g_scratch is only a stand-in for the device array and must
// never be handed to a kernel; cudaGetSymbolAddress gives the real device address.
int scratch_address_on(int device, void** out) {
  if (device < 0 || device >= kMaxDevices) {
    ss::set_error_message("device %d is beyond the %d devices the no-allocation path supports",
                          device, kMaxDevices);
    return SS_ERR_UNSUPPORTED;
  }
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch_addr[device]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_scratch);
    if (e != cudaSuccess || !p) {
      ss::set_error_message("cudaGetSymbolAddress of the static scratch failed: %s",
                            cudaGetErrorString(e));
      return SS_ERR_CUDA;
    }
    g_scratch_addr[device] = p;
  }
  *out = g_scratch_addr[device];
  return SS_OK;
}

int scratch_address(void** out, int* device) {
  const cudaError_t e = cudaGetDevice(device);
  if (e != cudaSuccess) {
    ss::set_error_message("cudaGetDevice failed: %s", cudaGetErrorString(e));
    return SS_ERR_CUDA;
  }
  return scratch_address_on(*device, out);
}

}  // namespace

extern "C" int ss_ragged_paged_attention_noalloc(
    const void* q, const int64_t q_strides[3], const void* k_pool, const int64_t k_pool_strides[4],
    const void* v_pool, const int64_t v_pool_strides[4], const void* block_tables,
    const int64_t bt_strides[2], int64_t bt_rows, int64_t bt_cols, int bt_is_int64,
    const void* query_seq_ids, int seq_ids_is_int64, const void* positions,
    int positions_is_int64, void* out, const int64_t out_strides[3], int64_t tokens, int heads,
    int kv_heads, int head_dim, int64_t num_pages, float sm_scale, void* stream) {
  void* scratch = nullptr;
  int device = 0;
  int rc = scratch_address(&scratch, &device);
  if (rc != SS_OK) return rc;
  if (tokens < 1 || heads < 1 || kv_heads < 1 || heads % kv_heads)
    return ss_ragged_paged_attention(q, q_strides, k_pool, k_pool_strides, v_pool,
                                     v_pool_strides, block_tables, bt_strides, bt_rows, bt_cols,
                                     bt_is_int64, query_seq_ids, seq_ids_is_int64, positions,
                                     positions_is_int64, out, out_strides, tokens, heads,
                                     kv_heads, head_dim, num_pages, sm_scale, scratch,
                                     kScratchBytes, stream);  // reports the invalid argument
  size_t need = 0;
  rc = ss_attention_workspace_bytes(device, tokens, heads, kv_heads, head_dim, &need);
  if (rc != SS_OK) return rc;
  if (need > kScratchBytes) {
    ss::set_error_message(
        "this call needs %zu bytes of scratch but the no-allocation path has a fixed %zu; "
        "use ss_ragged_paged_attention with a caller-provided workspace",
        need, kScratchBytes);
    return SS_ERR_WORKSPACE;
  }
  return ss_ragged_paged_attention(q, q_strides, k_pool, k_pool_strides, v_pool, v_pool_strides,
                                   block_tables, bt_strides, bt_rows, bt_cols, bt_is_int64,
                                   query_seq_ids, seq_ids_is_int64, positions, positions_is_int64,
                                   out, out_strides, tokens, heads, kv_heads, head_dim, num_pages,
                                   sm_scale, scratch, kScratchBytes, stream);
}

extern "C" int ss_noalloc_fetch_device_errors(int device, int clear, uint32_t* flags,
                                              void* stream) {
  if (!flags) {
    ss::set_error_message("null pointer argument");
    return SS_ERR_INVALID;
  }
  int prev = 0;
  cudaError_t e = cudaGetDevice(&prev);
  if (e != cudaSuccess) {
    ss::set_error_message("cudaGetDevice failed: %s", cudaGetErrorString(e));
    return SS_ERR_CUDA;
  }
  if (device != prev && (e = cudaSetDevice(device)) != cudaSuccess) {
    ss::set_error_message("cudaSetDevice(%d) failed: %s", device, cudaGetErrorString(e));
    return SS_ERR_CUDA;
  }
  void* scratch = nullptr;
  int rc = scratch_address_on(device, &scratch);
  if (rc == SS_OK) rc = ss_fetch_device_errors(scratch, clear, flags, stream);
  if (device != prev) cudaSetDevice(prev);
  return rc;
}
