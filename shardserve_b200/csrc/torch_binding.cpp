// Python binding of the per-layer hot calls over torch tensors.
//
// `ragged_attention_direct`, `kv_append` and `rope_kv_append` are the calls a serving loop
// makes for every layer of every step (reference: shardserve/kernel.py:11-82 and
// shardserve/cache.py:47-49, called from model.py:25-33).  Their argument checks, in the
// reference's order and with its messages, and the marshalling into the C ABI of
// include/shardserve_b200.h run here in C++ on at::Tensor, so a call costs a few
// microseconds of host time instead of tens in Python.  The C ABI itself lives in
// libshardserve_b200.so, loaded once by the package; `bind()` hands this module the
// addresses of its entry points, so both paths share one copy of the library's state (last
// error message, attention path, per-device geometry caches).
//
// The per-device workspace (error word, split-K partial states, split descriptors) is kept
// here: one zero-filled byte buffer per device, grown (never during CUDA graph capture) to
// what ss_attention_workspace_bytes asks for.  A buffer that is replaced by a larger one is
// never freed: CUDA graphs captured while it was current keep its address in their kernel
// arguments and write into it on every replay (decode-bucket graphs captured at start-up,
// then a larger eager chunked-prefill step, as the reference engine runs).
#include <torch/extension.h>

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <string>
#include <tuple>
#include <vector>

#include "shardserve_b200.h"

namespace py = pybind11;

namespace {

decltype(&ss_ragged_paged_attention) p_attention = nullptr;
decltype(&ss_append_ragged_paged_attention) p_append_attention = nullptr;
decltype(&ss_kv_append) p_append = nullptr;
decltype(&ss_rope_kv_append) p_rope = nullptr;
decltype(&ss_attention_workspace_bytes) p_ws_bytes = nullptr;
decltype(&ss_last_error_message) p_last_error = nullptr;
PyObject* g_unsupported = nullptr;  // shardserve_b200.kernel.KernelUnsupported (a ValueError)

constexpr int64_t kBlockSize = 16;

void require_bound() {
  if (!p_attention || !p_append_attention || !p_append || !p_rope || !p_ws_bytes ||
      !p_last_error || !g_unsupported)
    throw std::runtime_error("shardserve_b200 torch binding used before bind()");
}

[[noreturn]] void unsupported(const std::string& msg) {
  PyErr_SetString(g_unsupported, msg.c_str());
  throw py::error_already_set();
}

std::string last_error() {
  const char* m = p_last_error();
  return m ? std::string(m) : std::string();
}

// Raises like the Python wrappers did: SS_ERR_INVALID -> KernelUnsupported(message), any
// other failure -> RuntimeError("<entry point>: message").
void check_rc(int rc, const char* what) {
  if (rc == SS_OK) return;
  if (rc == SS_ERR_INVALID) unsupported(last_error());
  throw std::runtime_error(std::string(what) + ": " + last_error());
}

// tuple(t.shape) as Python prints it.  (No iostreams in this file: with this toolchain and
// torch build, std::ostringstream in an extension module crashes the process.)
std::string shape_str(const at::Tensor& t) {
  std::string s = "(";
  for (int64_t i = 0; i < t.dim(); ++i) {
    if (i) s += ", ";
    s += std::to_string(t.size(i));
  }
  if (t.dim() == 1) s += ",";
  return s + ")";
}

int index_flag(const at::Tensor& t, const char* name) {
  if (t.scalar_type() == at::kLong) return 1;
  if (t.scalar_type() == at::kInt) return 0;
  const std::string dt = py::str(py::cast(t).attr("dtype"));
  unsupported(std::string(name) + " must be int32 or int64, got " + dt);
}

// A 1-D contiguous view of an index tensor (t.reshape(-1), made contiguous if needed).
at::Tensor flat_index(const at::Tensor& t) {
  at::Tensor f = t.dim() == 1 ? t : t.reshape({-1});
  return f.is_contiguous() ? f : f.contiguous();
}

template <int N>
struct Strides {
  int64_t v[N];
  explicit Strides(const at::Tensor& t) {
    for (int i = 0; i < N; ++i) v[i] = t.stride(i);
  }
};

void* stream_of(const at::Device& d) {
  return static_cast<void*>(at::cuda::getCurrentCUDAStream(d.index()).stream());
}

// ---- per-device workspace ------------------------------------------------------------------
std::mutex g_ws_mu;
// Leaked on purpose: tensors must not be released after the CUDA context is torn down.
auto* g_ws = new std::map<int, at::Tensor>();
// Workspaces replaced by a larger one, kept alive for the life of the process: a graph
// captured earlier still replays into them.  Growth doubles the size, so what is kept here
// stays below the size of the current workspace.
auto* g_ws_retired = new std::vector<at::Tensor>();
auto* g_ws_need = new std::map<std::tuple<int, int64_t, int, int, int>, size_t>();

at::Tensor ensure_workspace(const at::Device& dev, int64_t tokens, int heads, int kv_heads,
                            int head_dim) {
  const int idx = dev.index();
  std::lock_guard<std::mutex> lock(g_ws_mu);
  const auto key = std::make_tuple(idx, tokens, heads, kv_heads, head_dim);
  auto nit = g_ws_need->find(key);
  size_t need = 0;
  if (nit != g_ws_need->end()) {
    need = nit->second;
  } else {
    check_rc(p_ws_bytes(idx, tokens, heads, kv_heads, head_dim, &need),
             "ss_attention_workspace_bytes");
    if (g_ws_need->size() > 4096) g_ws_need->clear();
    (*g_ws_need)[key] = need;
  }
  auto it = g_ws->find(idx);
  if (it != g_ws->end() && static_cast<size_t>(it->second.numel()) >= need) return it->second;
  cudaStreamCaptureStatus status = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(at::cuda::getCurrentCUDAStream(idx).stream(), &status) ==
          cudaSuccess &&
      status != cudaStreamCaptureStatusNone)
    throw std::runtime_error(
        "ragged_attention_direct: workspace must grow during CUDA graph capture; run the same "
        "shapes once before capturing");
  const int64_t old = it != g_ws->end() ? it->second.numel() : 0;
  const int64_t size = std::max<int64_t>({static_cast<int64_t>(need), 2 * old, int64_t{1} << 20});
  at::Tensor ws = at::zeros({size}, at::TensorOptions().dtype(at::kByte).device(dev));
  if (it != g_ws->end()) g_ws_retired->push_back(it->second);
  (*g_ws)[idx] = ws;
  return ws;
}

py::object workspace_for(int device_index) {
  std::lock_guard<std::mutex> lock(g_ws_mu);
  auto it = g_ws->find(device_index);
  if (it == g_ws->end()) return py::none();
  return py::cast(it->second);
}

void* err_word(const at::Device& dev) {
  std::lock_guard<std::mutex> lock(g_ws_mu);
  auto it = g_ws->find(dev.index());
  return it == g_ws->end() ? nullptr : it->second.data_ptr();
}

// The step's new K/V rows of kv_append_attention (nullptr: plain attention).
struct NewRows {
  const at::Tensor* k;
  const at::Tensor* v;
  const at::Tensor* slots;
};

void check_kv(const at::Tensor& k, const at::Tensor& v, int64_t kv_heads, int64_t head_dim);

// ---- ragged_attention_direct (reference shardserve/kernel.py:11-82) -------------------------
at::Tensor attention_call(const at::Tensor& q, const at::Tensor& k_pool, const at::Tensor& v_pool,
                          const at::Tensor& block_tables, const at::Tensor& query_seq_ids,
                          const at::Tensor& positions, double sm_scale, const NewRows* rows) {
  require_bound();
  // Checks and messages of the reference wrapper, kernel.py:28-49.
  if (!q.is_cuda() || q.scalar_type() != at::kBFloat16)
    unsupported("ragged kernel requires BF16 CUDA queries");
  if (q.dim() != 3 || (q.size(-1) != 64 && q.size(-1) != 128))
    unsupported("ragged q must be [tokens, heads, 64|128], got " + shape_str(q));
  if (k_pool.sizes() != v_pool.sizes() || k_pool.dim() != 4)
    unsupported("ragged K/V pools must have identical rank-4 shapes");
  if (k_pool.scalar_type() != at::kBFloat16 || k_pool.size(1) != kBlockSize)
    unsupported("ragged KV pools must be BF16 with block_size=16");
  if (k_pool.size(-1) != q.size(-1)) unsupported("query and KV head dimensions differ");
  if (block_tables.device() != q.device() || block_tables.dim() != 2)
    unsupported("block_tables must be a device-resident rank-2 tensor");
  if (query_seq_ids.numel() != q.size(0) || positions.numel() != q.size(0))
    unsupported("one sequence id and absolute position are required per query");
  if (q.size(0) < 1) unsupported("ragged batch cannot be empty");
  const int64_t tokens = q.size(0);
  const int heads = static_cast<int>(q.size(1)), head_dim = static_cast<int>(q.size(2));
  const int kv_heads = static_cast<int>(k_pool.size(2));
  if (kv_heads < 1 || heads % kv_heads) unsupported("query heads must be divisible by KV heads");
  const std::pair<const char*, const at::Tensor*> same_device[] = {
      {"k_pool_layer", &k_pool}, {"v_pool_layer", &v_pool},
      {"query_seq_ids", &query_seq_ids}, {"positions", &positions}};
  for (const auto& nt : same_device)
    if (nt.second->device() != q.device())
      unsupported(std::string(nt.first) + " must be on " + q.device().str());
  if (v_pool.scalar_type() != at::kBFloat16)
    unsupported("ragged KV pools must be BF16 with block_size=16");
  const int bt64 = index_flag(block_tables, "block_tables");
  const int seq64 = index_flag(query_seq_ids, "query_seq_ids");
  const int pos64 = index_flag(positions, "positions");
  const at::Tensor seqs = flat_index(query_seq_ids);
  const at::Tensor pos = flat_index(positions);

  const c10::cuda::OptionalCUDAGuard guard(q.device());
  at::Tensor out = at::empty_like(q);
  const at::Tensor ws = ensure_workspace(q.device(), tokens, heads, kv_heads, head_dim);
  const Strides<3> qs(q), os(out);
  const Strides<4> ks(k_pool), vs(v_pool);
  const Strides<2> bs(block_tables);
  if (rows == nullptr) {
    check_rc(p_attention(q.data_ptr(), qs.v, k_pool.data_ptr(), ks.v, v_pool.data_ptr(), vs.v,
                         block_tables.data_ptr(), bs.v, block_tables.size(0),
                         block_tables.size(1), bt64, seqs.data_ptr(), seq64, pos.data_ptr(),
                         pos64, out.data_ptr(), os.v, tokens, heads, kv_heads, head_dim,
                         k_pool.size(0), static_cast<float>(sm_scale), ws.data_ptr(),
                         static_cast<size_t>(ws.numel()), stream_of(q.device())),
             "ss_ragged_paged_attention");
    return out;
  }
  // kv_append's checks (same messages as kv_append), then the fused call.
  const at::Tensor& k = *rows->k;
  const at::Tensor& v = *rows->v;
  check_kv(k, v, kv_heads, head_dim);
  if (k.size(0) != tokens) unsupported("k/v must hold one row per query token");
  const std::pair<const char*, const at::Tensor*> row_devices[] = {
      {"k", &k}, {"v", &v}, {"slots", rows->slots}};
  for (const auto& nt : row_devices)
    if (nt.second->device() != q.device())
      unsupported(std::string(nt.first) + " must be on " + q.device().str());
  if (rows->slots->numel() != tokens) unsupported("one slot is required per appended token");
  const int s64 = index_flag(*rows->slots, "slots");
  const at::Tensor sl = flat_index(*rows->slots);
  const Strides<3> kst(k), vst(v);
  check_rc(p_append_attention(k.data_ptr(), kst.v, v.data_ptr(), vst.v, sl.data_ptr(), s64,
                              q.data_ptr(), qs.v, k_pool.data_ptr(), ks.v, v_pool.data_ptr(),
                              vs.v, block_tables.data_ptr(), bs.v, block_tables.size(0),
                              block_tables.size(1), bt64, seqs.data_ptr(), seq64,
                              pos.data_ptr(), pos64, out.data_ptr(), os.v, tokens, heads,
                              kv_heads, head_dim, k_pool.size(0), static_cast<float>(sm_scale),
                              ws.data_ptr(), static_cast<size_t>(ws.numel()),
                              stream_of(q.device())),
           "ss_append_ragged_paged_attention");
  return out;
}

at::Tensor ragged_attention_direct(const at::Tensor& q, const at::Tensor& k_pool,
                                   const at::Tensor& v_pool, const at::Tensor& block_tables,
                                   const at::Tensor& query_seq_ids, const at::Tensor& positions,
                                   double sm_scale) {
  return attention_call(q, k_pool, v_pool, block_tables, query_seq_ids, positions, sm_scale,
                        nullptr);
}

// Cache.write + ragged_attention_direct in one call (reference model.py:32-37).
at::Tensor kv_append_attention(const at::Tensor& k_pool, const at::Tensor& v_pool,
                               const at::Tensor& k, const at::Tensor& v, const at::Tensor& slots,
                               const at::Tensor& q, const at::Tensor& block_tables,
                               const at::Tensor& query_seq_ids, const at::Tensor& positions,
                               double sm_scale) {
  const NewRows rows{&k, &v, &slots};
  return attention_call(q, k_pool, v_pool, block_tables, query_seq_ids, positions, sm_scale,
                        &rows);
}

// Pool checks shared by kv_append and rope_kv_append.
void check_pools(const at::Tensor& k_pool, const at::Tensor& v_pool, const char* not_cuda) {
  if (!k_pool.is_cuda()) unsupported(not_cuda);
  if (k_pool.scalar_type() != at::kBFloat16 || v_pool.scalar_type() != at::kBFloat16)
    unsupported("KV pools must be BF16");
  if (k_pool.sizes() != v_pool.sizes() || k_pool.dim() != 4 || k_pool.size(1) != kBlockSize)
    unsupported("ragged K/V pools must have identical rank-4 shapes");
}

void check_kv(const at::Tensor& k, const at::Tensor& v, int64_t kv_heads, int64_t head_dim) {
  if (k.dim() != 3 || k.size(1) != kv_heads || k.size(2) != head_dim || k.sizes() != v.sizes()) {
    unsupported("k/v must be [tokens, " + std::to_string(kv_heads) + ", " +
                std::to_string(head_dim) + "], got " + shape_str(k) + "/" + shape_str(v));
  }
  if (k.scalar_type() != at::kBFloat16 || v.scalar_type() != at::kBFloat16)
    unsupported("k/v must be BF16");
}

// ---- kv_append: the device half of Cache.write (reference shardserve/cache.py:47-49) -------
void kv_append(const at::Tensor& k_pool, const at::Tensor& v_pool, const at::Tensor& k,
               const at::Tensor& v, const at::Tensor& slots) {
  require_bound();
  check_pools(k_pool, v_pool, "KV append requires CUDA pools");
  const int64_t kv_heads = k_pool.size(2), head_dim = k_pool.size(3);
  check_kv(k, v, kv_heads, head_dim);
  const std::pair<const char*, const at::Tensor*> same_device[] = {
      {"v_pool_layer", &v_pool}, {"k", &k}, {"v", &v}, {"slots", &slots}};
  for (const auto& nt : same_device)
    if (nt.second->device() != k_pool.device())
      unsupported(std::string(nt.first) + " must be on " + k_pool.device().str());
  if (slots.numel() != k.size(0)) unsupported("one slot is required per appended token");
  const int s64 = index_flag(slots, "slots");
  const at::Tensor sl = flat_index(slots);
  const c10::cuda::OptionalCUDAGuard guard(k_pool.device());
  const Strides<3> kst(k), vst(v);
  const Strides<4> kps(k_pool), vps(v_pool);
  check_rc(p_append(k.data_ptr(), kst.v, v.data_ptr(), vst.v, k_pool.data_ptr(), kps.v,
                    v_pool.data_ptr(), vps.v, sl.data_ptr(), s64, k.size(0), k_pool.size(0),
                    static_cast<int>(kv_heads), static_cast<int>(head_dim),
                    err_word(k_pool.device()), stream_of(k_pool.device())),
           "ss_kv_append");
}

// ---- rope_kv_append: apply_rope (reference shardserve/math.py:28-38) + Cache.write ---------
at::Tensor rope_kv_append(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                          const at::Tensor& cos, const at::Tensor& sin,
                          const at::Tensor& positions, const at::Tensor& k_pool,
                          const at::Tensor& v_pool, const at::Tensor& slots,
                          c10::optional<at::Tensor> out_opt) {
  require_bound();
  check_pools(k_pool, v_pool, "RoPE + KV append requires CUDA pools");
  const int64_t kv_heads = k_pool.size(2), head_dim = k_pool.size(3);
  if (q.dim() != 3 || q.size(2) != head_dim || q.scalar_type() != at::kBFloat16)
    unsupported("q must be BF16 [tokens, heads, " + std::to_string(head_dim) + "]");
  check_kv(k, v, kv_heads, head_dim);
  if (q.size(0) != k.size(0) || kv_heads < 1 || q.size(1) % kv_heads)
    unsupported("q and k/v must have the same tokens and a whole GQA group");
  if (head_dim % 2) unsupported("RoPE needs an even head_dim");
  const std::pair<const char*, const at::Tensor*> tables[] = {{"cos", &cos}, {"sin", &sin}};
  for (const auto& nt : tables) {
    const at::Tensor& t = *nt.second;
    if (t.scalar_type() != at::kFloat || t.dim() != 2 || t.size(1) != head_dim)
      unsupported(std::string(nt.first) + " must be float32 [rows, " + std::to_string(head_dim) +
                  "]");
  }
  if (cos.sizes() != sin.sizes()) unsupported("cos and sin tables must have the same shape");
  const std::pair<const char*, const at::Tensor*> same_device[] = {
      {"v_pool_layer", &v_pool}, {"q", &q},   {"k", &k},
      {"v", &v},                 {"cos", &cos}, {"sin", &sin},
      {"positions", &positions}, {"slots", &slots}};
  for (const auto& nt : same_device)
    if (nt.second->device() != k_pool.device())
      unsupported(std::string(nt.first) + " must be on " + k_pool.device().str());
  const int64_t tokens = q.size(0);
  if (slots.numel() != tokens || positions.numel() != tokens)
    unsupported("one position and one slot are required per token");
  const int p64 = index_flag(positions, "positions");
  const int s64 = index_flag(slots, "slots");
  const at::Tensor pos = flat_index(positions);
  const at::Tensor sl = flat_index(slots);
  const c10::cuda::OptionalCUDAGuard guard(k_pool.device());
  at::Tensor out;
  if (!out_opt.has_value() || !out_opt->defined()) {
    out = at::empty_like(q);
  } else {
    out = *out_opt;
    if (out.sizes() != q.sizes() || out.scalar_type() != at::kBFloat16 || out.device() != q.device())
      unsupported("out must be a BF16 tensor shaped like q on q's device");
  }
  const Strides<3> qs(q), os(out), kst(k), vst(v);
  const Strides<2> cs(cos), ss(sin);
  const Strides<4> kps(k_pool), vps(v_pool);
  check_rc(p_rope(q.data_ptr(), qs.v, out.data_ptr(), os.v, k.data_ptr(), kst.v, v.data_ptr(),
                  vst.v, static_cast<const float*>(cos.data_ptr()), cs.v,
                  static_cast<const float*>(sin.data_ptr()), ss.v, cos.size(0), pos.data_ptr(), p64,
                  k_pool.data_ptr(), kps.v, v_pool.data_ptr(), vps.v, sl.data_ptr(), s64, tokens,
                  static_cast<int>(q.size(1)), static_cast<int>(kv_heads),
                  static_cast<int>(head_dim), k_pool.size(0), err_word(k_pool.device()),
                  stream_of(k_pool.device())),
           "ss_rope_kv_append");
  return out;
}

template <typename F>
void take(const py::dict& addrs, const char* name, F*& slot) {
  slot = reinterpret_cast<F*>(static_cast<uintptr_t>(addrs[name].cast<uint64_t>()));
  if (!slot) throw std::runtime_error(std::string("bind(): null address for ") + name);
}

void bind(const py::dict& addrs, const py::object& unsupported_cls) {
  take(addrs, "ss_ragged_paged_attention", p_attention);
  take(addrs, "ss_append_ragged_paged_attention", p_append_attention);
  take(addrs, "ss_kv_append", p_append);
  take(addrs, "ss_rope_kv_append", p_rope);
  take(addrs, "ss_attention_workspace_bytes", p_ws_bytes);
  take(addrs, "ss_last_error_message", p_last_error);
  PyObject* cls = unsupported_cls.ptr();
  Py_INCREF(cls);
  Py_XDECREF(g_unsupported);
  g_unsupported = cls;
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "torch-tensor binding of the shardserve_b200 attention hot path";
  m.def("bind", &bind, py::arg("addresses"), py::arg("unsupported"));
  m.def("ragged_attention_direct", &ragged_attention_direct, py::arg("q"),
        py::arg("k_pool_layer"), py::arg("v_pool_layer"), py::arg("block_tables"),
        py::arg("query_seq_ids"), py::arg("positions"), py::arg("sm_scale"));
  m.def("kv_append", &kv_append, py::arg("k_pool_layer"), py::arg("v_pool_layer"), py::arg("k"),
        py::arg("v"), py::arg("slots"));
  m.def("kv_append_attention", &kv_append_attention, py::arg("k_pool_layer"),
        py::arg("v_pool_layer"), py::arg("k"), py::arg("v"), py::arg("slots"), py::arg("q"),
        py::arg("block_tables"), py::arg("query_seq_ids"), py::arg("positions"),
        py::arg("sm_scale"));
  m.def("rope_kv_append", &rope_kv_append, py::arg("q"), py::arg("k"), py::arg("v"),
        py::arg("cos"), py::arg("sin"), py::arg("positions"), py::arg("k_pool_layer"),
        py::arg("v_pool_layer"), py::arg("slots"), py::arg("out") = py::none());
  m.def("ensure_workspace",
        [](int device_index, int64_t tokens, int heads, int kv_heads, int head_dim) {
          require_bound();
          return ensure_workspace(at::Device(at::kCUDA, static_cast<c10::DeviceIndex>(device_index)),
                                  tokens, heads, kv_heads, head_dim);
        });
  m.def("workspace_for", &workspace_for);
}
