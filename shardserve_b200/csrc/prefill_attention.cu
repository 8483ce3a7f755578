// Chunked-prefill tiles of ragged paged attention on B200 tensor cores (tcgen05 + TMEM).
//
// Reference semantics: shardserve/kernel.py:85-166 (each query token attends to keys
// 0..position of its sequence row).  Tokens that belong to a run of >= 2 consecutive query
// tokens of one sequence (a chunked-prefill chunk; token_in_long_run with min_run 2) are
// computed here as dense tiles; isolated tokens (decode rows) by the split-K decode kernel.
//
// Tile: 16 consecutive query tokens x the 8 query heads of one KV head = 128 rows (M), head
// dim 128 (K), keys in blocks of 128 (N).  Per key block:
//   S  = Q.K^T       tcgen05.mma kind::f16, A = Q (smem, K-major), B = K (smem, K-major)
//                    -> 128 x 128 fp32 in TMEM columns [0, 128)
//   softmax          one thread per TMEM lane (= tile row): causal mask from the token's
//                    position, base-2 online softmax; O is rescaled in TMEM only when the
//                    row max grows by more than 2^8 (the reference max is otherwise kept,
//                    which is exact: O and l use the same reference)
//   O += P.V         tcgen05.mma, A = P (bf16 in smem, K-major over keys), B = V (smem,
//                    MN-major: head_dim contiguous) -> 128 x 128 fp32 in TMEM [128, 256)
// K/V pages come by TMA (one 2 KiB box per page and 64-dim half, 128-byte swizzle, no
// multicast) through a 2-stage ring; Q by two 4-D TMA boxes.  Warp roles: warp 0 TMA
// producer, warp 1 MMA issuer (one elected thread), warps 4-7 softmax / epilogue.
#include <cuda_bf16.h>
#include <math_constants.h>

#include <mutex>

#include "attention.cuh"
#include "ptx.cuh"

namespace ss {

namespace {

constexpr int kTQ = 16;                        // query tokens per tile
constexpr int kGroup = 8;                      // query heads per KV head (this kernel)
constexpr int kRowsT = kTQ * kGroup;           // 128 tile rows (M)
constexpr int kHDp = 128;                      // head dim (K of S, N of O)
constexpr int kNB = 128;                       // keys per block (N of S, K of O)
constexpr int kPgPerBlk = kNB / kPage;         // 8 pages per block
constexpr int kStagesP = 2;
constexpr int kThreadsP = 256;
constexpr int kMinRunP = 2;                    // tokens of runs >= 2 are prefill tokens
constexpr uint32_t kTmemCols = 256;            // S [0,128) + O [128,256)

// Shared memory (1024-aligned base).  Every operand tile is [2 halves of 64][rows][128 B].
constexpr int kQBytes = 2 * kRowsT * 128;      // 32 KiB
constexpr int kKVBytes = 2 * kNB * 128;        // 32 KiB for K (or V) of one block
constexpr int kOffQ = 0;
constexpr int kOffK = kOffQ + kQBytes;                       // + s * 2 * kKVBytes
constexpr int kOffP = kOffK + kStagesP * 2 * kKVBytes;       // 32 KiB
constexpr int kOffBarP = kOffP + 2 * kRowsT * 128;
// barriers: q_full, s_full, s_free, p_full, o_done, kv_full[2], kv_empty[2]
constexpr int kNumBars = 5 + 2 * kStagesP;
constexpr int kOffCtlP = kOffBarP + 8 * kNumBars;
constexpr int kMaxSeg = kTQ;

struct CtlP {
  uint32_t tmem_base;
  int nseg;
  int seg_first[kMaxSeg];  // window-relative first token of each segment
  int seg_last[kMaxSeg];
  long long seg_seq[kMaxSeg];
  int seg_keys[kMaxSeg];   // keys the segment's last row attends (max position + 1, clamped)
};
constexpr int kSmemP = kOffCtlP + static_cast<int>(sizeof(CtlP)) + 1024;

__device__ __forceinline__ uint32_t bar_addr(uint32_t base, int i) { return base + 8 * i; }

template <int D>
__global__ void __launch_bounds__(kThreadsP, 1)
    prefill_attention_kernel(const __grid_constant__ CUtensorMap tmQ,
                             const __grid_constant__ CUtensorMap tmK,
                             const __grid_constant__ CUtensorMap tmV, const AttnArgs a) {
  static_assert(D == kHDp, "prefill tiles are built for head_dim 128");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sb = smem_u32(smem);
  const uint32_t sQ = sb + kOffQ, sK0 = sb + kOffK, sP = sb + kOffP;
  const uint32_t bars = sb + kOffBarP;
  const uint32_t q_full = bar_addr(bars, 0), s_full = bar_addr(bars, 1), s_free = bar_addr(bars, 2);
  const uint32_t p_full = bar_addr(bars, 3), o_done = bar_addr(bars, 4);
  auto kv_full = [&](int s) { return bar_addr(bars, 5 + s); };
  auto kv_empty = [&](int s) { return bar_addr(bars, 5 + kStagesP + s); };
  CtlP* ctl = reinterpret_cast<CtlP*>(smem + kOffCtlP);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const long long t0 = static_cast<long long>(blockIdx.x) * kTQ;
  const int kvh = blockIdx.y;

  if (tid == 0) {
    mbar_init(q_full, 1);
    mbar_init(s_full, 1);
    mbar_init(s_free, 128);
    mbar_init(p_full, 128);
    mbar_init(o_done, 1);
    for (int s = 0; s < kStagesP; ++s) {
      mbar_init(kv_full(s), 1);
      mbar_init(kv_empty(s), 1);
    }
    fence_mbar_init();
  }
  // Segments of this 16-token window: maximal runs of prefill tokens of one sequence.
  if (warp == 2) {
    const long long t = t0 + lane;
    long long seq = -1;
    int pre = 0, pos = 0;
    if (lane < kTQ && t < a.T) {
      // Same predicate as the decode kernel: every token of a multi-token run is ours.
      const TokInfo ti = token_info(a, t, false);
      seq = ti.seq;
      pre = token_in_long_run(a, kMinRunP, t, ti.seq) ? 1 : 0;
      pos = ti.L;  // keys of this row (0 for invalid metadata: the row is written as zeros)
    }
    const unsigned pm = __ballot_sync(0xffffffffu, pre);
    const long long prev_seq = __shfl_up_sync(0xffffffffu, seq, 1);
    const long long next_seq = __shfl_down_sync(0xffffffffu, seq, 1);
    const int starts = pre && (lane == 0 || !((pm >> (lane - 1)) & 1) || prev_seq != seq);
    const unsigned sm = __ballot_sync(0xffffffffu, starts);
    if (pre) {
      const int idx = __popc(sm & ((2u << lane) - 1)) - 1;  // segment of this token
      if (starts) {
        ctl->seg_first[idx] = lane;
        ctl->seg_seq[idx] = seq;
      }
      const int ends = (lane == 31) || !((pm >> (lane + 1)) & 1) || next_seq != seq;
      if (ends) ctl->seg_last[idx] = lane;
    }
    // Keys of a segment = max over its tokens (positions grow inside a chunk, but do not
    // rely on it): reduce per segment with a simple loop in lane 0.
    __syncwarp();
    const int nseg = __popc(sm);
    int keys_of_lane = pos;
    for (int sgi = 0; sgi < nseg; ++sgi) {
      const int f = ctl->seg_first[sgi], l = ctl->seg_last[sgi];
      int v = (lane >= f && lane <= l) ? keys_of_lane : 0;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
      if (lane == 0) ctl->seg_keys[sgi] = v;
    }
    if (lane == 0) ctl->nseg = nseg;
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(&ctl->tmem_base), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const int nseg = ctl->nseg;
  const uint32_t tmem = ctl->tmem_base;
  const uint32_t tS = tmem, tO = tmem + kNB;

  if (nseg > 0) {
    if (warp == 0) {
      // ============================== TMA producer ==============================
      if (lane == 0) {
        prefetch_tensormap(&tmQ);
        prefetch_tensormap(&tmK);
        prefetch_tensormap(&tmV);
        mbar_arrive_expect_tx(q_full, kQBytes);
        tma_load_4d(sQ, &tmQ, q_full, 0, 0, kvh * kGroup, static_cast<int>(t0));
        tma_load_4d(sQ + kQBytes / 2, &tmQ, q_full, 0, 1, kvh * kGroup, static_cast<int>(t0));
      }
      int st = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int sgi = 0; sgi < nseg && ok; ++sgi) {
        const long long seq = ctl->seg_seq[sgi];
        const int keys = ctl->seg_keys[sgi];
        const int npages = (keys + kPage - 1) / kPage;
        const int nblk = (keys + kNB - 1) / kNB;
        for (int j = 0; j < nblk && ok; ++j) {
          int pg = -1;
          if (lane < kPgPerBlk) {
            const int pi = j * kPgPerBlk + lane;
            if (pi < npages) {
              const long long pid = ld_index(a.bt, a.bt64, seq * a.bt_sb + pi * a.bt_sn);
              if (pid < 0 || pid >= a.N) atomicOr(a.err, SS_DEVERR_PAGE);
              else pg = static_cast<int>(pid);
            }
          }
          int pgs[kPgPerBlk];
#pragma unroll
          for (int p = 0; p < kPgPerBlk; ++p) pgs[p] = __shfl_sync(0xffffffffu, pg, p);
          if (lane == 0) {
            if (!mbar_wait(kv_empty(st), ph ^ 1)) {
              ok = false;
            } else {
              const uint32_t kdst = sK0 + st * 2 * kKVBytes, vdst = kdst + kKVBytes;
              mbar_arrive_expect_tx(kv_full(st), 2 * kKVBytes);
#pragma unroll
              for (int p = 0; p < kPgPerBlk; ++p) {
#pragma unroll
                for (int dh = 0; dh < 2; ++dh) {
                  const uint32_t off = dh * (kKVBytes / 2) + p * (kPage * 128);
                  tma_load_5d_nohint(kdst + off, &tmK, kv_full(st), 0, 0, dh, kvh, pgs[p]);
                  tma_load_5d_nohint(vdst + off, &tmV, kv_full(st), 0, 0, dh, kvh, pgs[p]);
                }
              }
            }
          }
          ok = __shfl_sync(0xffffffffu, ok, 0);
          if (++st == kStagesP) {
            st = 0;
            ph ^= 1;
          }
        }
      }
      if (!ok && lane == 0) atomicOr(a.err, SS_DEVERR_TIMEOUT);
    } else if (warp == 1) {
      // ============================== MMA issuer ================================
      if (lane == 0) {
        constexpr uint32_t idesc_qk = idesc_bf16_f32(128, kNB, 0, 0);
        constexpr uint32_t idesc_pv = idesc_bf16_f32(128, kHDp, 0, 1);
        int st = 0;
        uint32_t ph = 0;
        int jg = 0;
        bool ok = mbar_wait(q_full, 0);
        for (int sgi = 0; sgi < nseg && ok; ++sgi) {
          const int nblk = (ctl->seg_keys[sgi] + kNB - 1) / kNB;
          for (int j = 0; j < nblk && ok; ++j, ++jg) {
            const uint32_t kst = sK0 + st * 2 * kKVBytes, vst = kst + kKVBytes;
            ok = mbar_wait(kv_full(st), ph);
            if (ok && jg > 0) ok = mbar_wait(s_free, (jg - 1) & 1);
            if (!ok) break;
            tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < kHDp / 16; ++kk) {
              const uint32_t koff = (kk >> 2) * (kKVBytes / 2) + (kk & 3) * 32;
              const uint64_t ad = smem_desc_sw128(sQ + (kk >> 2) * (kQBytes / 2) + (kk & 3) * 32, 16, 1024);
              const uint64_t bd = smem_desc_sw128(kst + koff, 16, 1024);
              tc_mma_f16(tS, ad, bd, idesc_qk, kk > 0 ? 1u : 0u);
            }
            tc_commit(s_full);
            ok = mbar_wait(p_full, jg & 1);
            if (!ok) break;
            tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < kNB / 16; ++kk) {
              const uint64_t ad = smem_desc_sw128(sP + (kk >> 2) * (kRowsT * 128) + (kk & 3) * 32, 16, 1024);
              const uint64_t bd = smem_desc_sw128(vst + kk * 16 * 128, kKVBytes / 2, 1024);
              tc_mma_f16(tO, ad, bd, idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
            }
            tc_commit(o_done);
            tc_commit(kv_empty(st));
            if (++st == kStagesP) {
              st = 0;
              ph ^= 1;
            }
          }
        }
        if (!ok) atomicOr(a.err, SS_DEVERR_TIMEOUT);
      }
      __syncwarp();
    } else if (warp >= 4) {
      // ========================= softmax + epilogue (1 row per thread) ==========
      const int wq = warp - 4;            // TMEM lane quadrant of this warp
      const int row = wq * 32 + lane;     // tile row = token * 8 + head
      const int rt = row / kGroup, rh = row % kGroup;
      const long long t = t0 + rt;
      const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
      const float sc = a.scale_log2;
      int jg = 0;
      bool ok = true;
      for (int sgi = 0; sgi < nseg && ok; ++sgi) {
        const int f = ctl->seg_first[sgi], l = ctl->seg_last[sgi];
        const bool mine = rt >= f && rt <= l && t < a.T;
        const int keys = mine ? token_info(a, t, false).L : 0;
        const int nblk = (ctl->seg_keys[sgi] + kNB - 1) / kNB;
        if (nblk == 0) {  // no row of the segment has keys: zero output rows
          if (mine)
            for (int dd = 0; dd < kHDp; ++dd)
              a.out[t * a.o_st + static_cast<long long>(kvh * kGroup + rh) * a.o_sh + dd * a.o_sd] =
                  __float2bfloat16(0.f);
          continue;
        }
        float m_ref = -CUDART_INF_F, lsum = 0.f;
        for (int j = 0; j < nblk; ++j, ++jg) {
          ok = mbar_wait(s_full, jg & 1);
          if (!ok) break;
          tc_fence_after();
          uint32_t sr[4][32];
#pragma unroll
          for (int c = 0; c < 4; ++c) tmem_ld32(tS + lane_off + c * 32, sr[c]);
          tmem_wait_ld();
          tc_fence_before();
          mbar_arrive(s_free);
          const int kbase = j * kNB;
          float mblk = -CUDART_INF_F;
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const float x = (kbase + c * 32 + i < keys) ? __uint_as_float(sr[c][i]) * sc : -CUDART_INF_F;
              sr[c][i] = __float_as_uint(x);
              mblk = fmaxf(mblk, x);
            }
          // Keep the reference max unless this block raises it by more than 8 (2^8 in p).
          const bool raise = mblk > m_ref + 8.f;
          const float m_new = raise ? mblk : m_ref;
          const float alpha = (raise && m_ref != -CUDART_INF_F) ? ex2(m_ref - m_new) : (raise ? 0.f : 1.f);
          if (j > 0) {  // PV of the previous block must be done: O stable, P buffer free
            ok = mbar_wait(o_done, (jg - 1) & 1);
            if (!ok) break;
            tc_fence_after();
            if (__any_sync(0xffffffffu, raise)) {
#pragma unroll
              for (int c = 0; c < 4; ++c) {
                uint32_t orow[32];
                tmem_ld32(tO + lane_off + c * 32, orow);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; ++i) orow[i] = __float_as_uint(__uint_as_float(orow[i]) * alpha);
                tmem_st32(tO + lane_off + c * 32, orow);
              }
              tmem_wait_st();
            }
          }
          lsum *= alpha;
          m_ref = m_new;
          const float ms = m_ref == -CUDART_INF_F ? 0.f : m_ref;
          // P row -> shared memory, bf16, 128-byte swizzled K-major tile [2][128 rows][128 B].
#pragma unroll
          for (int c = 0; c < 4; ++c) {
#pragma unroll
            for (int q8 = 0; q8 < 4; ++q8) {
              float pv[8];
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                pv[e] = ex2(__uint_as_float(sr[c][q8 * 8 + e]) - ms);
                lsum += pv[e];
              }
              const int key = c * 32 + q8 * 8;  // first key of this 16-byte chunk
              const int kh = key >> 6, chunk = (key & 63) >> 3;
              const uint32_t addr = sP + kh * (kRowsT * 128) + row * 128 + ((chunk ^ (row & 7)) << 4);
              asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr),
                           "r"(pack_bf16(pv[0], pv[1])), "r"(pack_bf16(pv[2], pv[3])),
                           "r"(pack_bf16(pv[4], pv[5])), "r"(pack_bf16(pv[6], pv[7]))
                           : "memory");
            }
          }
          fence_proxy_async_smem();
          tc_fence_before();
          mbar_arrive(p_full);
        }
        if (!ok) break;
        // ---- epilogue: O / l -> bf16 ---------------------------------------------------
        ok = mbar_wait(o_done, (jg - 1) & 1);
        if (!ok) break;
        tc_fence_after();
        const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
        __nv_bfloat16* op = a.out + t * a.o_st + static_cast<long long>(kvh * kGroup + rh) * a.o_sh;
        const bool vec = mine && a.o_sd == 1 && ((reinterpret_cast<uintptr_t>(op) & 15) == 0);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t orow[32];
          tmem_ld32(tO + lane_off + c * 32, orow);
          tmem_wait_ld();
          if (mine) {
            if (vec) {
#pragma unroll
              for (int q8 = 0; q8 < 4; ++q8) {
                uint4 v;
                v.x = pack_bf16(__uint_as_float(orow[q8 * 8 + 0]) * inv, __uint_as_float(orow[q8 * 8 + 1]) * inv);
                v.y = pack_bf16(__uint_as_float(orow[q8 * 8 + 2]) * inv, __uint_as_float(orow[q8 * 8 + 3]) * inv);
                v.z = pack_bf16(__uint_as_float(orow[q8 * 8 + 4]) * inv, __uint_as_float(orow[q8 * 8 + 5]) * inv);
                v.w = pack_bf16(__uint_as_float(orow[q8 * 8 + 6]) * inv, __uint_as_float(orow[q8 * 8 + 7]) * inv);
                *reinterpret_cast<uint4*>(op + c * 32 + q8 * 8) = v;
              }
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i)
                op[static_cast<long long>(c * 32 + i) * a.o_sd] = __float2bfloat16(__uint_as_float(orow[i]) * inv);
            }
          }
        }
        tc_fence_before();  // O reads complete before the next segment's P.V overwrites O
      }
      if (!ok && lane == 0) atomicOr(a.err, SS_DEVERR_TIMEOUT);
    }
  }
  // ---- teardown ------------------------------------------------------------------------
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
  // This grid completes only after the decode grid before it (programmatic launch chain),
  // so the merge kernel that waits on this grid also waits on the decode grid.
  griddep_wait();
}

}  // namespace

bool prefill_supported(const AttnArgs& a) {
  return a.D == kHDp && a.group == kGroup && a.q_sd == 1 && (a.q_sh % 8) == 0 &&
         (a.q_st % 8) == 0 && (reinterpret_cast<uintptr_t>(a.q) & 15) == 0;
}

int prefill_min_run() { return kMinRunP; }

cudaError_t launch_prefill(const CUtensorMap& tmQ, const CUtensorMap& tmK, const CUtensorMap& tmV,
                           const AttnArgs& a, cudaStream_t stream) {
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [] {
    attr_err = cudaFuncSetAttribute(prefill_attention_kernel<kHDp>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemP);
  });
  if (attr_err != cudaSuccess) return attr_err;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>((a.T + kTQ - 1) / kTQ), a.KVH);
  cfg.blockDim = dim3(kThreadsP);
  cfg.dynamicSmemBytes = kSmemP;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, prefill_attention_kernel<kHDp>, tmQ, tmK, tmV, a);
}

}  // namespace ss
