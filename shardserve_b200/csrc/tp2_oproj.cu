// TP2 attention output projection fused with its all-reduce over NVLink (two ranks).
//
// Replaces, per layer and rank, the reference's
//     hidden = hidden + reduce(F.linear(attention, w_o))          (shardserve/model.py:40)
//     reduce = dist.all_reduce over the two TP ranks (sum)         (shardserve/runtime.py:17-24)
// for its projection + reduction part: out = bf16(P_0 + P_1), P_r = bf16(A_r W_rᵀ), where
// A_r [T, K] is rank r's attention output (its heads) and W_r [N, K] its column shard of
// o_proj.  Every rank computes the same out (the sum of two bf16 values is formed in fp32,
// so both ranks round the same number).
//
// One CTA = 128 tokens x 32 output features, full K.  Warp 0 (one thread) loads A and W
// tiles by TMA (128-byte swizzle, 4-stage ring; local memory only), warp 1 (one thread)
// issues tcgen05.mma M128 N32 K16 into 32 TMEM columns, then all four warps read their
// 32-token TMEM quadrant, round P_r to bf16 and store it straight into the PEER's inbox
// (plain 16-byte stores over NVLink), publish a flag in the peer's memory (release,
// system scope), wait (bounded) for the peer's flag for the same tile, and add the peer's
// partial from the local inbox.  The inbox and flags alternate between two halves by call
// parity and flags carry the call's epoch, so nothing is ever cleared and a rank cannot
// overwrite a partial the other rank has not consumed.  A CTA never waits for another CTA
// of its own GPU; it waits only for its counterpart on the other GPU, which stores its
// partial before it waits.  The grid is at most one wave, so both counterparts are
// resident.  TMA reads only this GPU's memory; no library kernel touches peer memory.
#include <cuda_bf16.h>

#include "attention.cuh"
#include "ptx.cuh"

namespace ss {

namespace {

constexpr int kTM = 128;   // tokens per tile (MMA M)
constexpr int kTN = 32;    // features per tile (MMA N)
constexpr int kTK = 64;    // K per stage (one 128-byte swizzle atom of bf16)
constexpr int kStagesO = 4;
constexpr int kABytes = kTM * kTK * 2;  // 16 KiB
constexpr int kWBytes = kTN * kTK * 2;  // 4 KiB
constexpr int kStageBytes = kABytes + kWBytes;
constexpr int kSmemO = kStagesO * kStageBytes + 256 + 1024;

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(128, 1)
    tp2_oproj_kernel(const __grid_constant__ CUtensorMap tmA,
                     const __grid_constant__ CUtensorMap tmW, const OprojArgs o) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sb = smem_u32(smem);
  const uint32_t bars = sb + kStagesO * kStageBytes;  // full[4], empty[4], done
  auto full = [&](int s) { return bars + 8 * s; };
  auto empty = [&](int s) { return bars + 8 * (kStagesO + s); };
  const uint32_t done = bars + 8 * (2 * kStagesO);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kStagesO * kStageBytes + 128);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n0 = blockIdx.x * kTN;
  const long long m0 = static_cast<long long>(blockIdx.y) * kTM;
  const int kblocks = o.K / kTK;

  if (tid == 0) {
    for (int s = 0; s < kStagesO; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);
    }
    mbar_init(done, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(tmem_slot), 32);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  if (warp == 0 && lane == 0) {  // ---- TMA producer
    prefetch_tensormap(&tmA);
    prefetch_tensormap(&tmW);
    for (int kb = 0; kb < kblocks && ok; ++kb) {
      const int s = kb % kStagesO;
      ok = mbar_wait(empty(s), ((kb / kStagesO) & 1) ^ 1);
      if (!ok) break;
      const uint32_t dst = sb + s * kStageBytes;
      mbar_arrive_expect_tx(full(s), kStageBytes);
      tma_load_2d(dst, &tmA, full(s), kb * kTK, static_cast<int>(m0));
      tma_load_2d(dst + kABytes, &tmW, full(s), kb * kTK, n0);
    }
  } else if (warp == 1 && lane == 0) {  // ---- MMA issuer
    constexpr uint32_t idesc = idesc_bf16_f32(kTM, kTN, 0, 0);
    for (int kb = 0; kb < kblocks && ok; ++kb) {
      const int s = kb % kStagesO;
      ok = mbar_wait(full(s), (kb / kStagesO) & 1);
      if (!ok) break;
      tc_fence_after();
      const uint32_t a = sb + s * kStageBytes, w = a + kABytes;
#pragma unroll
      for (int kk = 0; kk < kTK / 16; ++kk)
        tc_mma_f16(tmem, smem_desc_sw128(a + kk * 32, 16, 1024),
                   smem_desc_sw128(w + kk * 32, 16, 1024), idesc, (kb > 0 || kk > 0) ? 1u : 0u);
      tc_commit(empty(s));
    }
    tc_commit(done);
  }
  __syncwarp();
  if (!ok) atomicOr(o.err, SS_DEVERR_TIMEOUT);

  // ---- epilogue: every warp owns 32 tokens (its TMEM lane quadrant) x 32 features
  const bool mma_ok = __all_sync(0xffffffffu, mbar_wait(done, 0));
  const int parity = static_cast<int>(o.epoch & 1u);
  const long long row = m0 + (warp & 3) * 32 + lane;
  const bool live = mma_ok && row < o.T;
  uint32_t acc[32];
  if (mma_ok) {
    tc_fence_after();
    tmem_ld32(tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16), acc);
    tmem_wait_ld();
  }
  float mine[32];
  uint32_t packed[16];
#pragma unroll
  for (int i = 0; i < 32; i += 2) {
    const __nv_bfloat162 p = __floats2bfloat162_rn(__uint_as_float(acc[i]), __uint_as_float(acc[i + 1]));
    packed[i / 2] = *reinterpret_cast<const uint32_t*>(&p);
    mine[i] = __low2float(p);
    mine[i + 1] = __high2float(p);
  }
  const long long inbox_off = (static_cast<long long>(parity) * o.T_max + row) * o.N + n0;
  if (live) {  // this rank's partial into the peer's inbox (16-byte stores over NVLink)
    uint4* dst = reinterpret_cast<uint4*>(o.peer_inbox + inbox_off);
#pragma unroll
    for (int q = 0; q < 4; ++q)
      dst[q] = make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
  }
  __syncthreads();
  const int tile = blockIdx.y * gridDim.x + blockIdx.x;
  if (tid == 0) {
    __threadfence_system();
    st_release_sys(o.peer_flags + parity * o.tiles_max + tile, o.epoch);
    // Wait (bounded) for the other rank's partial of this tile in the local inbox.
    const unsigned* f = o.local_flags + parity * o.tiles_max + tile;
    const long long start = clock64();
    bool arrived = ld_acquire_sys(f) == o.epoch;
    while (!arrived && clock64() - start < kWaitLimitCycles) arrived = ld_acquire_sys(f) == o.epoch;
    if (!arrived) atomicOr(o.err, SS_DEVERR_TIMEOUT);
    *reinterpret_cast<volatile int*>(smem + kStagesO * kStageBytes + 132) = arrived ? 1 : 0;
  }
  __syncthreads();
  const bool arrived = *reinterpret_cast<volatile int*>(smem + kStagesO * kStageBytes + 132) != 0;
  if (live && arrived) {
    const uint4* src = reinterpret_cast<const uint4*>(o.local_inbox + inbox_off);
    __nv_bfloat16* out = o.out + row * o.out_rs + n0;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint4 v = __ldcv(src + q);  // the peer wrote it: bypass L1
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
      uint32_t r[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float lo = __uint_as_float(w[e] << 16), hi = __uint_as_float(w[e] & 0xFFFF0000u);
        const __nv_bfloat162 s = __floats2bfloat162_rn(__fadd_rn(mine[8 * q + 2 * e], lo),
                                                       __fadd_rn(mine[8 * q + 2 * e + 1], hi));
        r[e] = *reinterpret_cast<const uint32_t*>(&s);
      }
      reinterpret_cast<uint4*>(out)[q] = make_uint4(r[0], r[1], r[2], r[3]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 32);
  }
}

}  // namespace

int oproj_tile_features() { return kTN; }
int oproj_tile_tokens() { return kTM; }

cudaError_t launch_tp2_oproj(const CUtensorMap& tmA, const CUtensorMap& tmW, const OprojArgs& o,
                             cudaStream_t stream) {
  static bool attr_done = false;
  if (!attr_done) {
    const cudaError_t e = cudaFuncSetAttribute(tp2_oproj_kernel,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemO);
    if (e != cudaSuccess) return e;
    attr_done = true;
  }
  const dim3 grid(static_cast<unsigned>(o.N / kTN), static_cast<unsigned>((o.T + kTM - 1) / kTM));
  tp2_oproj_kernel<<<grid, 128, kSmemO, stream>>>(tmA, tmW, o);
  return cudaGetLastError();
}

}  // namespace ss
