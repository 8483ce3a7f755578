// Rotary position embedding of q and k fused with the slot-mapped K/V append.
//
// Replaces, in one launch, the reference's
//     q, k = apply_rope(q, k, cos, sin, positions)      (shardserve/math.py:28-38, model.py:25)
//     cache.write(layer, k, v, slots)                    (shardserve/cache.py:47-49, model.py:32)
// with the same bf16 arithmetic as torch on bf16 tensors, so the result is bit-exact:
//     c = bf16(cos[pos][i]), s = bf16(sin[pos][i])
//     out[i]       = bf16( bf16(x[i] * c) + bf16(-x[i + D/2] * s) )        i <  D/2
//     out[i + D/2] = bf16( bf16(x[i + D/2] * c') + bf16(x[i] * s') )        (c', s' at i + D/2)
// Products and sums use __fmul_rn / __fadd_rn (never contracted into an fma) and every
// rounding is round-to-nearest-even, without flushing subnormals, as torch does.
//
// Work item = (token, job): one job rotates 8 elements of the first half and the 8 matching
// elements of the second half of one q or k head (one element pair in the scalar form), or
// copies 16 bytes (one element) of one v head into its slot.  Each item reads both halves
// before writing, so q may be rotated in place.  A token whose position lies outside the
// table is skipped entirely (SS_DEVERR_POS); a slot outside the pool skips that token's
// append (SS_DEVERR_SLOT) but its queries are still rotated.
#include <cuda_bf16.h>

#include "attention.cuh"
#include "ptx.cuh"

namespace ss {

namespace {

__device__ __forceinline__ float rope_mul(float x, float c) {
  return __bfloat162float(__float2bfloat16_rn(__fmul_rn(x, c)));
}
__device__ __forceinline__ __nv_bfloat16 rope_add(float a, float b) {
  return __float2bfloat16_rn(__fadd_rn(a, b));
}
__device__ __forceinline__ float bf16r(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

template <bool VEC>
__global__ void __launch_bounds__(256) rope_append_kernel(const RopeArgs r) {
  // Programmatic dependent launch (as kv_append_kernel): may start while the preceding
  // kernel finishes and waits for it before reading q / k / v; releases nothing early.
  griddep_wait();
  const AppendArgs& a = r.app;
  constexpr int E = VEC ? 8 : 1;  // elements per half (rotation) or per copy (v)
  const int half = a.D / 2;
  const int jq = r.H * (half / E), jk = a.KVH * (half / E), jv = a.KVH * (a.D / E);
  const long long per_tok = jq + jk + jv;
  const long long total = a.T * per_tok;
  const long long step = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += step) {
    const long long t = i / per_tok;
    int j = static_cast<int>(i % per_tok);
    const long long pos = ld_index(r.pos, r.pos64, t);
    if (pos < 0 || pos >= r.rows) {
      if (a.err && j == 0) atomicOr(a.err, SS_DEVERR_POS);
      continue;
    }
    const long long slot = ld_index(a.slots, a.slots64, t);
    const bool slot_ok = slot >= 0 && slot < a.N * kPage;
    if (!slot_ok && a.err && j == 0) atomicOr(a.err, SS_DEVERR_SLOT);
    const long long page = slot / kPage, prow = slot % kPage;
    if (j >= jq + jk) {  // ---- v: plain copy into the slot
      if (!slot_ok) continue;
      j -= jq + jk;
      const int h = j / (a.D / E), d = (j % (a.D / E)) * E;
      const __nv_bfloat16* src = a.v + t * a.v_st + h * a.v_sh + d * a.v_sd;
      __nv_bfloat16* dst = a.vp + page * a.vp_sn + prow * a.vp_ss + h * a.vp_sh + d * a.vp_sd;
      if (VEC) *reinterpret_cast<uint4*>(dst) = __ldg(reinterpret_cast<const uint4*>(src));
      else *dst = *src;
      continue;
    }
    // ---- q or k: rotate E elements of each half
    const bool is_k = j >= jq;
    if (is_k && !slot_ok) continue;
    if (is_k) j -= jq;
    const int h = j / (half / E), d = (j % (half / E)) * E;
    const __nv_bfloat16* src;
    long long s_d;
    __nv_bfloat16* dst;
    long long d_d;
    if (is_k) {
      src = a.k + t * a.k_st + h * a.k_sh;
      s_d = a.k_sd;
      dst = a.kp + page * a.kp_sn + prow * a.kp_ss + h * a.kp_sh;
      d_d = a.kp_sd;
    } else {
      src = r.q + t * r.q_st + h * r.q_sh;
      s_d = r.q_sd;
      dst = r.qo + t * r.qo_st + h * r.qo_sh;
      d_d = r.qo_sd;
    }
    const float* cr = r.cos + pos * r.cos_sr;
    const float* sr = r.sin + pos * r.sin_sr;
    float x1[E], x2[E], c1[E], s1[E], c2[E], s2[E];
    if (VEC) {
      const uint4 u1 = *reinterpret_cast<const uint4*>(src + d);
      const uint4 u2 = *reinterpret_cast<const uint4*>(src + d + half);
      const uint32_t w1[4] = {u1.x, u1.y, u1.z, u1.w}, w2[4] = {u2.x, u2.y, u2.z, u2.w};
#pragma unroll
      for (int e = 0; e < E; ++e) {  // bf16 -> fp32 is a 16-bit shift, exact
        x1[e] = __uint_as_float(((w1[e >> 1] >> (16 * (e & 1))) & 0xFFFFu) << 16);
        x2[e] = __uint_as_float(((w2[e >> 1] >> (16 * (e & 1))) & 0xFFFFu) << 16);
      }
#pragma unroll
      for (int e = 0; e < E; e += 4) {
        const float4 fc1 = __ldg(reinterpret_cast<const float4*>(cr + d + e));
        const float4 fs1 = __ldg(reinterpret_cast<const float4*>(sr + d + e));
        const float4 fc2 = __ldg(reinterpret_cast<const float4*>(cr + d + half + e));
        const float4 fs2 = __ldg(reinterpret_cast<const float4*>(sr + d + half + e));
        c1[e] = fc1.x; c1[e + 1] = fc1.y; c1[e + 2] = fc1.z; c1[e + 3] = fc1.w;
        s1[e] = fs1.x; s1[e + 1] = fs1.y; s1[e + 2] = fs1.z; s1[e + 3] = fs1.w;
        c2[e] = fc2.x; c2[e + 1] = fc2.y; c2[e + 2] = fc2.z; c2[e + 3] = fc2.w;
        s2[e] = fs2.x; s2[e + 1] = fs2.y; s2[e + 2] = fs2.z; s2[e + 3] = fs2.w;
      }
    } else {
      x1[0] = __bfloat162float(src[d * s_d]);
      x2[0] = __bfloat162float(src[(d + half) * s_d]);
      c1[0] = __ldg(cr + d * r.cos_sd);
      s1[0] = __ldg(sr + d * r.sin_sd);
      c2[0] = __ldg(cr + (d + half) * r.cos_sd);
      s2[0] = __ldg(sr + (d + half) * r.sin_sd);
    }
    __nv_bfloat16 o1[E], o2[E];
#pragma unroll
    for (int e = 0; e < E; ++e) {
      o1[e] = rope_add(rope_mul(x1[e], bf16r(c1[e])), rope_mul(-x2[e], bf16r(s1[e])));
      o2[e] = rope_add(rope_mul(x2[e], bf16r(c2[e])), rope_mul(x1[e], bf16r(s2[e])));
    }
    if (VEC) {
      uint32_t p1[4], p2[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        p1[e] = static_cast<uint32_t>(__bfloat16_as_ushort(o1[2 * e])) |
                (static_cast<uint32_t>(__bfloat16_as_ushort(o1[2 * e + 1])) << 16);
        p2[e] = static_cast<uint32_t>(__bfloat16_as_ushort(o2[2 * e])) |
                (static_cast<uint32_t>(__bfloat16_as_ushort(o2[2 * e + 1])) << 16);
      }
      *reinterpret_cast<uint4*>(dst + d) = make_uint4(p1[0], p1[1], p1[2], p1[3]);
      *reinterpret_cast<uint4*>(dst + d + half) = make_uint4(p2[0], p2[1], p2[2], p2[3]);
    } else {
      dst[d * d_d] = o1[0];
      dst[(d + half) * d_d] = o2[0];
    }
  }
}

}  // namespace

cudaError_t launch_rope_append(const RopeArgs& r, bool vectorised, cudaStream_t stream) {
  const int E = vectorised ? 8 : 1;
  const long long per_tok = static_cast<long long>(r.H + r.app.KVH) * (r.app.D / 2 / E) +
                            static_cast<long long>(r.app.KVH) * (r.app.D / E);
  long long blocks = (r.app.T * per_tok + 255) / 256;
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
  return vectorised ? cudaLaunchKernelEx(&cfg, rope_append_kernel<true>, r)
                    : cudaLaunchKernelEx(&cfg, rope_append_kernel<false>, r);
}

}  // namespace ss
