// Generic strided ragged paged attention: one warp per (query token, head).
//
// Used only for layouts the TMA kernel cannot describe (non-unit head_dim stride, strides
// or base addresses that are not 16-byte multiples, more than 16 query heads per KV head).
// It follows shardserve/kernel.py:115-166 literally: walk pages through the block table,
// fp32 dot products, online softmax, fp32 P.V, bf16 store.  Correct for every stride the
// reference accepts; not tuned.
#include <cuda_bf16.h>
#include <math_constants.h>

#include "attention.cuh"
#include "ptx.cuh"

namespace ss {

namespace {

constexpr int kWarpsPerBlock = 4;

__global__ void __launch_bounds__(32 * kWarpsPerBlock) generic_attention_kernel(const AttnArgs a) {
  const long long w = static_cast<long long>(blockIdx.x) * kWarpsPerBlock + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w >= a.T * a.H) return;
  const long long t = w / a.H;
  const int h = static_cast<int>(w % a.H);
  const int kvh = h / a.group;  // kernel.py:120
  const TokInfo ti = token_info(a, t, h == 0 && lane == 0);
  constexpr int kMaxPer = 4;  // head_dim <= 128 -> at most 4 dims per lane
  const int per = a.D / 32;
  float qv[kMaxPer], acc[kMaxPer];
  const __nv_bfloat16* qp = a.q + t * a.q_st + static_cast<long long>(h) * a.q_sh;
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    qv[i] = i < per ? __bfloat162float(qp[static_cast<long long>(lane + 32 * i) * a.q_sd]) : 0.f;
    acc[i] = 0.f;
  }
  float m = -CUDART_INF_F, l = 0.f;
  for (int pg = 0; pg < ti.npages; ++pg) {
    const long long pid = ld_index(a.bt, a.bt64, ti.seq * a.bt_sb + pg * a.bt_sn);
    const bool valid_page = pid >= 0 && pid < a.N;
    if (!valid_page && lane == 0) atomicOr(a.err, SS_DEVERR_PAGE);
    const int nk = min(kPage, ti.L - pg * kPage);
    for (int s = 0; s < nk; ++s) {
      float part = 0.f, vv[kMaxPer];
      const long long kb = pid * a.k_sn + s * a.k_ss + static_cast<long long>(kvh) * a.k_sh;
      const long long vb = pid * a.v_sn + s * a.v_ss + static_cast<long long>(kvh) * a.v_sh;
#pragma unroll
      for (int i = 0; i < kMaxPer; ++i) {
        vv[i] = 0.f;
        if (i < per && valid_page) {
          const long long dd = lane + 32 * i;
          part += qv[i] * __bfloat162float(a.kp[kb + dd * a.k_sd]);
          vv[i] = __bfloat162float(a.vp[vb + dd * a.v_sd]);
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
      const float x = part * a.scale_log2;
      const float mn = fmaxf(m, x);
      const float alpha = ex2(m - mn);
      const float p = ex2(x - mn);
      l = l * alpha + p;
#pragma unroll
      for (int i = 0; i < kMaxPer; ++i) acc[i] = acc[i] * alpha + p * vv[i];
      m = mn;
    }
  }
  const float inv = l > 0.f ? 1.f / l : 0.f;
  __nv_bfloat16* op = a.out + t * a.o_st + static_cast<long long>(h) * a.o_sh;
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i)
    if (i < per) op[static_cast<long long>(lane + 32 * i) * a.o_sd] = __float2bfloat16(acc[i] * inv);
}

}  // namespace

cudaError_t launch_generic_attention(const AttnArgs& a, cudaStream_t stream) {
  const long long warps = a.T * a.H;
  const long long blocks = (warps + kWarpsPerBlock - 1) / kWarpsPerBlock;
  if (blocks > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  generic_attention_kernel<<<static_cast<unsigned>(blocks), 32 * kWarpsPerBlock, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace ss
