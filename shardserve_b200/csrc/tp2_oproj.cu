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
// One CTA = 128 tokens x 32 output features (the kernel also takes 64 or 128), full K.
// Warp 0 (one thread) loads A and W by TMA with 3-D boxes that each carry two or four
// 64-column K chunks (128-byte swizzle), so a call with K = 1024 needs 8-16 copies per CTA;
// warp 1 (one thread) issues tcgen05.mma M128 N(tile) K16 into TMEM.  All four warps then
// read their 32-token TMEM quadrant 32 features at a time and round P_r to bf16.  The
// exchange uses flag-carrying vectors: every 16-byte vector holds six bf16 partials (three
// feature pairs) and the call's epoch, so a token's 32 features take six vectors, 96 bytes
// for 64 bytes of payload.  A warp stores each of its six vectors for its 32 tokens as one
// contiguous 512-byte run (vector-major inbox layout) straight into the other rank's inbox
// over NVLink; the other rank polls its own inbox, with the same coalesced 16-byte loads,
// until every vector carries the current epoch (bounded), so no fence or separate flag is
// needed, and adds the pairs to its own partial.  A vector is written and read whole
// (st / ld .v4.b32 of one aligned 16-byte vector).  Inbox halves alternate by call parity,
// so a rank never overwrites vectors the other rank has not read.  The epoch lives in device memory: every
// CTA reads the last completed call number at its start and the last CTA to finish
// advances it, so calls can be replayed from a CUDA graph.  A CTA waits only for its
// counterpart on the other GPU, which writes before it waits; the grid is at most one wave,
// so both are resident.  TMA reads only this GPU's memory; no library kernel touches peer
// memory.
#include <cuda_bf16.h>

#include "attention.cuh"
#include "ptx.cuh"

namespace ss {

namespace {

constexpr int kTM = 128;    // tokens per tile (MMA M)
constexpr int kTNMax = 128; // features per tile (MMA N): 32, 64 or 128 by call size
constexpr int kTK = 64;     // K columns per swizzle atom
constexpr int kMaxStagesO = 8;
constexpr int kVecPerGroup = 6;  // inbox vectors per (token, 32 features): 3 bf16 pairs each
constexpr int kRingBytes = 200 * 1024;
constexpr int kSmemO = kRingBytes + 512 + 1024;

__device__ __forceinline__ void st_volatile_v4(void* p, uint4 v) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ uint4 ld_volatile_v4(const void* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

__global__ void __launch_bounds__(128, 1)
    tp2_oproj_kernel(const __grid_constant__ CUtensorMap tmA,
                     const __grid_constant__ CUtensorMap tmW, const OprojArgs o) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sb = smem_u32(smem);
  const int nst = o.stages, kc = o.atoms, tn = o.tile_n;
  const int a_chunk = o.a_rows * kTK * 2;              // one 64-column atom of A rows
  const int w_chunk = tn * kTK * 2;
  const int a_stage = kc * a_chunk, stage_bytes = a_stage + kc * w_chunk;
  const uint32_t bars = sb + kRingBytes;               // full[8], empty[8], done
  auto full = [&](int s) { return bars + 8 * s; };
  auto empty = [&](int s) { return bars + 8 * (kMaxStagesO + s); };
  const uint32_t done = bars + 8 * (2 * kMaxStagesO);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kRingBytes + 320);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n0 = blockIdx.x * tn;
  const long long m0 = static_cast<long long>(blockIdx.y) * kTM;
  const int nload = o.K / (kTK * kc);                  // ring stages of this call
  const unsigned epoch = *reinterpret_cast<volatile const unsigned*>(o.epoch_ctr) + 1u;

  if (tid == 0) {
    for (int s = 0; s < nst; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);
    }
    mbar_init(done, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(tmem_slot), kTNMax);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  if (warp == 0 && lane == 0) {  // ---- TMA producer: 3-D boxes of kc atoms
    prefetch_tensormap(&tmA);
    prefetch_tensormap(&tmW);
    for (int i = 0; i < nload && ok; ++i) {
      const int s = i % nst;
      ok = mbar_wait(empty(s), ((i / nst) & 1) ^ 1);
      if (!ok) break;
      const uint32_t dst = sb + s * stage_bytes;
      mbar_arrive_expect_tx(full(s), stage_bytes);
      tma_load_3d(dst, &tmA, full(s), 0, static_cast<int>(m0), i * kc);
      tma_load_3d(dst + a_stage, &tmW, full(s), 0, n0, i * kc);
    }
  } else if (warp == 1 && lane == 0) {  // ---- MMA issuer
    const uint32_t idesc = idesc_bf16_f32(kTM, tn, 0, 0);
    for (int i = 0; i < nload && ok; ++i) {
      const int s = i % nst;
      ok = mbar_wait(full(s), (i / nst) & 1);
      if (!ok) break;
      tc_fence_after();
      const uint32_t a = sb + s * stage_bytes, w = a + a_stage;
      for (int c = 0; c < kc; ++c)
#pragma unroll
        for (int kk = 0; kk < kTK / 16; ++kk)
          tc_mma_f16(tmem, smem_desc_sw128(a + c * a_chunk + kk * 32, 16, 1024),
                     smem_desc_sw128(w + c * w_chunk + kk * 32, 16, 1024), idesc,
                     (i > 0 || c > 0 || kk > 0) ? 1u : 0u);
      tc_commit(empty(s));
    }
    tc_commit(done);
  }
  __syncwarp();
  if (!ok) atomicOr(o.err, SS_DEVERR_TIMEOUT);

  // ---- epilogue: every warp owns 32 tokens (its TMEM lane quadrant); groups of 32
  // features are rounded, exchanged and summed one after another.
  const bool mma_ok = __all_sync(0xffffffffu, mbar_wait(done, 0));
  const long long row = m0 + (warp & 3) * 32 + lane;
  const bool live = mma_ok && row < o.T;
  if (mma_ok) tc_fence_after();
  bool timed_out = false;
  for (int g = 0; g < tn / 32; ++g) {
    const int f0 = n0 + 32 * g;
    uint32_t acc[32];
    if (mma_ok) {
      tmem_ld32(tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16) + 32 * g, acc);
      tmem_wait_ld();
    }
    uint32_t pk[16];  // this rank's partial: bf16 pairs (features 2i, 2i + 1)
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const __nv_bfloat162 p = __floats2bfloat162_rn(__uint_as_float(acc[2 * i]),
                                                     __uint_as_float(acc[2 * i + 1]));
      pk[i] = *reinterpret_cast<const uint32_t*>(&p);
    }
    // Inbox vector v (0..5) of (token row, 32-feature group): {pairs 3v .. 3v + 2, epoch},
    // laid out [parity][32-row block][feature group][v][row % 32] so that a warp's store of
    // one vector is 512 contiguous bytes.
    const long long rb = row >> 5, nfg = o.N / 32;
    const long long vec0 =
        (((static_cast<long long>(epoch & 1u) * ((o.T_max + 31) / 32) + rb) * nfg + f0 / 32) *
         kVecPerGroup) * 32 + (row & 31);
    if (live) {
      uint4* dst = reinterpret_cast<uint4*>(o.peer_inbox) + vec0;
#pragma unroll
      for (int v = 0; v < kVecPerGroup; ++v) {
        const uint32_t p0 = pk[3 * v], p1 = 3 * v + 1 < 16 ? pk[3 * v + 1] : 0u;
        const uint32_t p2 = 3 * v + 2 < 16 ? pk[3 * v + 2] : 0u;
        st_volatile_v4(dst + 32 * v, make_uint4(p0, p1, p2, epoch));
      }
    }
    if (live && !timed_out) {  // the other rank's partial: poll until every vector is current
      const uint4* src = reinterpret_cast<const uint4*>(o.local_inbox) + vec0;
      uint32_t theirs[3 * kVecPerGroup];
      unsigned pending = (1u << kVecPerGroup) - 1;  // one bit per vector
      const long long start = clock64();
      while (pending) {
#pragma unroll
        for (int v = 0; v < kVecPerGroup; ++v) {
          if (pending & (1u << v)) {
            const uint4 x = ld_volatile_v4(src + 32 * v);
            if (x.w == epoch) {
              theirs[3 * v] = x.x;
              theirs[3 * v + 1] = x.y;
              theirs[3 * v + 2] = x.z;
              pending &= ~(1u << v);
            }
          }
        }
        if (pending && clock64() - start > kWaitLimitCycles) break;
      }
      if (pending) {
        atomicOr(o.err, SS_DEVERR_TIMEOUT);
        timed_out = true;
      } else {
        uint32_t r[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float a0 = __uint_as_float(pk[i] << 16), a1 = __uint_as_float(pk[i] & 0xFFFF0000u);
          const float b0 = __uint_as_float(theirs[i] << 16);
          const float b1 = __uint_as_float(theirs[i] & 0xFFFF0000u);
          const __nv_bfloat162 s2 = __floats2bfloat162_rn(__fadd_rn(a0, b0), __fadd_rn(a1, b1));
          r[i] = *reinterpret_cast<const uint32_t*>(&s2);
        }
        uint4* out = reinterpret_cast<uint4*>(o.out + row * o.out_rs + f0);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          out[q] = make_uint4(r[4 * q], r[4 * q + 1], r[4 * q + 2], r[4 * q + 3]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTNMax);
  }
  if (tid == 0) {  // the last CTA out records this call as complete
    __threadfence();
    if (atomicAdd(o.epoch_ctr + 1, 1u) == gridDim.x * gridDim.y - 1) {
      atomicExch(o.epoch_ctr, epoch);
      atomicExch(o.epoch_ctr + 1, 0u);
    }
  }
}

}  // namespace

int oproj_tile_tokens() { return kTM; }
int oproj_min_k_step() { return kTK * 2; }
// Features per tile.  The kernel handles 32, 64 and 128; 32 measured fastest at 32 and 256
// tokens per pair (more CTAs share the loads of W; wider tiles halve the re-reads of A but
// leave too few CTAs issuing copies).
int oproj_tile_n(long long) { return 32; }
// Atoms per stage and ring depth: the largest stage (4, then 2 atoms) that still leaves two
// stages in the ring, and as many stages as fit (at most one per load).
void oproj_ring(int a_rows, int tn, int k, int* atoms, int* stages) {
  int kc = 4;
  while (kc > 2 && 2 * kc * (a_rows + tn) * kTK * 2 > kRingBytes) kc /= 2;
  if ((k / kTK) % kc) kc = 2;
  const int stage = kc * (a_rows + tn) * kTK * 2;
  int n = kRingBytes / stage;
  if (n > kMaxStagesO) n = kMaxStagesO;
  const int loads = k / (kTK * kc);
  *atoms = kc;
  *stages = n < loads ? n : loads;
}

cudaError_t launch_tp2_oproj(const CUtensorMap& tmA, const CUtensorMap& tmW, const OprojArgs& o,
                             cudaStream_t stream) {
  static bool attr_done = false;
  if (!attr_done) {
    const cudaError_t e = cudaFuncSetAttribute(tp2_oproj_kernel,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemO);
    if (e != cudaSuccess) return e;
    attr_done = true;
  }
  if (o.stages < 1 || o.stages > kMaxStagesO || o.tile_n % 32 || o.tile_n > kTNMax ||
      o.stages * o.atoms * (o.a_rows + o.tile_n) * kTK * 2 > kRingBytes)
    return cudaErrorInvalidValue;
  const dim3 grid(static_cast<unsigned>(o.N / o.tile_n),
                  static_cast<unsigned>((o.T + kTM - 1) / kTM));
  tp2_oproj_kernel<<<grid, 128, kSmemO, stream>>>(tmA, tmW, o);
  return cudaGetLastError();
}

}  // namespace ss
