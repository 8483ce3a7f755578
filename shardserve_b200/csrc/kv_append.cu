// Slot-mapped KV append into the paged pool (reference: shardserve/cache.py:47-49,
// `pool.flatten(0, 1).index_copy_(0, slots, k)`).
//
// Slot s addresses row s % 16 of page s / 16.  One thread moves one 16-byte vector (8 bf16)
// when both sides are 16-byte addressable along head_dim, else one element.  The copy is
// bit-exact.
//
// Programmatic dependent launch: the kernel is launched so that it may start while the
// preceding kernel on the stream finishes (it then waits, griddepcontrol.wait, before it
// reads k / v or writes the pool).  It does not release the kernel after it early.
#include <cuda_bf16.h>

#include "attention.cuh"
#include "ptx.cuh"

namespace ss {

namespace {

template <bool VEC>
__global__ void __launch_bounds__(256) kv_append_kernel(const AppendArgs a) {
  // The attention kernel after this one is not released early (the kernel ends first): an
  // SM that still held one of these CTAs when the attention grid was placed was seen to take
  // only two of the three attention CTAs it can hold until it drained, which holds up the
  // attention kernel's grid barrier.
  griddep_wait();  // k / v may come from the preceding kernel, which may still read the pool
  constexpr int E = VEC ? 8 : 1;  // elements per thread
  const long long per_row = static_cast<long long>(a.KVH) * a.D / E;
  const long long total = a.T * per_row;
  const long long step = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < 2 * total;
       i += step) {
    const bool is_v = i >= total;
    const long long j = is_v ? i - total : i;
    const long long t = j / per_row;
    const long long e = (j % per_row) * E;
    const int h = static_cast<int>(e / a.D);
    const int dd = static_cast<int>(e % a.D);
    const long long slot = ld_index(a.slots, a.slots64, t);
    if (slot < 0 || slot >= a.N * kPage) {
      if (a.err && e == 0 && !is_v) atomicOr(a.err, SS_DEVERR_SLOT);
      continue;
    }
    const long long page = slot / kPage, row = slot % kPage;
    const __nv_bfloat16* src;
    __nv_bfloat16* dst;
    if (!is_v) {
      src = a.k + t * a.k_st + h * a.k_sh + dd * a.k_sd;
      dst = a.kp + page * a.kp_sn + row * a.kp_ss + h * a.kp_sh + dd * a.kp_sd;
    } else {
      src = a.v + t * a.v_st + h * a.v_sh + dd * a.v_sd;
      dst = a.vp + page * a.vp_sn + row * a.vp_ss + h * a.vp_sh + dd * a.vp_sd;
    }
    if (VEC) {
      *reinterpret_cast<uint4*>(dst) = __ldg(reinterpret_cast<const uint4*>(src));
    } else {
      *dst = *src;
    }
  }
}

}  // namespace

cudaError_t launch_kv_append(const AppendArgs& a, bool vectorised, cudaStream_t stream) {
  const long long per = static_cast<long long>(a.KVH) * a.D / (vectorised ? 8 : 1);
  const long long work = 2 * a.T * per;
  long long blocks = (work + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  if (blocks < 1) blocks = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(blocks));
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return vectorised ? cudaLaunchKernelEx(&cfg, kv_append_kernel<true>, a)
                    : cudaLaunchKernelEx(&cfg, kv_append_kernel<false>, a);
}

}  // namespace ss
