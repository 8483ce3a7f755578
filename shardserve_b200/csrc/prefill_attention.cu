// Chunked-prefill tiles of ragged paged attention on B200 tensor cores (tcgen05 + TMEM).
//
// Reference semantics: shardserve/kernel.py:85-166 (each query token attends to keys
// 0..position of its sequence row).  Tokens that belong to a run of >= 2 consecutive query
// tokens of one sequence (a chunked-prefill chunk; token_in_long_run with min_run 2) are
// computed here as dense tiles; isolated tokens (decode rows) by the split-K decode kernel.
//
// One CTA = a window of 32 consecutive query tokens x one KV head, as two tiles of 16
// tokens x the KV head's 8 query heads (128 rows = TMEM lanes each).  Both tiles use every
// K/V block the CTA loads, which halves the shared-memory fill traffic per FLOP against one
// tile per CTA (the per-SM TMA fill rate, not HBM, bounds a single 128-row tile).  Per key
// block j of 128 keys and tile t:
//   S_t  = Q_t.K_j^T  tcgen05.mma kind::f16, A = Q_t (smem, K-major), B = K_j (smem,
//                     K-major), fp32 128 x 128 in TMEM columns [128 t, 128 t + 128)
//   softmax           one thread per TMEM lane (= tile row): causal mask from the token's
//                     position, base-2 online softmax; P (bf16 pairs) is written back over
//                     the first 64 columns of S_t; O_t is rescaled in TMEM only when the row
//                     max grows by more than 2^8 (the old reference max is otherwise kept,
//                     which is exact because O_t and the row sum share the reference)
//   O_t += P_t.V_j    tcgen05.mma with A = P_t read from TMEM, B = V_j (smem, MN-major),
//                     fp32 in TMEM columns [256 + 128 t, 384 + 128 t)
// MMA issue order per block: S_0(j), O_1 += P_1 V(j-1), S_1(j), O_0 += P_0 V(j).  Each
// softmax thus has two MMAs' time for its block, the two softmax warpgroups run on
// alternate halves of the period, and the tensor pipe is never left empty.  tcgen05.mma
// operations of one thread execute in issue order, so S_t(j+1) may be issued right after
// the P_t.V(j) that reads P_t from the same columns; every other hand-off goes through an
// mbarrier.  K and V pages come by TMA (one 2 KiB box per page and 64-dim half, 128-byte
// swizzle, this CTA's own boxes) through two-stage rings filled by three producer warps, because
// one thread issues its TMA copies one after another.
//
// Scheduling: the grid is persistent (one CTA per SM, at most one per work item).  A work
// item is (32-token window, KV head); every CTA ranks the windows by an estimate of the key
// blocks their segments walk and takes items longest first from an atomic counter in the
// workspace header, so the wave tail is made of the shortest items.  The last CTA to
// finish returns the counter to zero for the next launch.  P.V of keys 0-63 starts once
// that half of P is written.
//
// Warps: 0 producer (Q, K d 0-63), 1 MMA issuer (one elected lane), 2 segment scan then producer
// (K d 64-127), 3 producer (V), 4-7 softmax / epilogue of tile 0, 8-11 of tile 1 (TMEM lane
// quadrant = warp % 4).  Registers are moved from the producer warpgroup to the softmax
// warpgroups with setmaxnreg: 384 threads launch with 168 registers each (64,512) and end
// with 72 (warps 0-3) + 2 x 216 (warps 4-11) per thread, 64,512 in total.
#include <cuda_bf16.h>
#include <math_constants.h>

#include <algorithm>
#include <climits>
#include <mutex>

#include "attention.cuh"
#include "ptx.cuh"

namespace ss {

namespace {

constexpr int kTiles = 2;
constexpr int kTQT = 16;                       // query tokens per tile
constexpr int kTQ = kTiles * kTQT;             // query tokens per CTA window
constexpr int kGroup = 8;                      // query heads per KV head (this kernel)
constexpr int kRowsT = kTQT * kGroup;          // 128 tile rows (M)
constexpr int kHDp = 128;                      // head dim (K of S, N of O)
constexpr int kNB = 128;                       // keys per block (N of S, K of O)
constexpr int kPgPerBlk = kNB / kPage;         // 8 pages per block
constexpr int kStages = 2;                     // K and V ring depth
constexpr int kThreadsP = 384;
constexpr int kLaunchRegs = 168;               // 65,536 / 384, rounded down to 8
constexpr int kRegsProducer = 72, kRegsSoftmax = 216;
static_assert(128 * kRegsProducer + 256 * kRegsSoftmax <= kThreadsP * kLaunchRegs,
              "setmaxnreg split exceeds the launch register pool");
constexpr int kMinRunP = 2;                    // tokens of runs >= 2 are prefill tokens
// One exponential pair in 3 on the FMA pipe.  The row sum accumulates pair i into acc[i % 4],
// so with 3 the slow polynomial results spread over all four partial sums; with 4 they all
// fell into one and formed a serial chain (the prefill-only step was 72.4 us against 67.9).
constexpr int kPolyEvery = 3;
constexpr uint32_t kTmemCols = 512;            // S_0 S_1 [0,256), O_0 O_1 [256,512)
constexpr uint32_t kColO = 256;

// Shared memory (1024-aligned base).  Every operand tile is [2 halves of 64][rows][128 B].
constexpr int kQBytes = 2 * kRowsT * 128;      // 32 KiB per tile
constexpr int kKVBytes = 2 * kNB * 128;        // 32 KiB: K (or V) of one key block
constexpr int kOffQ = 0;
constexpr int kOffK = kOffQ + kTiles * kQBytes;
constexpr int kOffV = kOffK + kStages * kKVBytes;
constexpr int kOffBarP = kOffV + kStages * kKVBytes;
// barriers: q_full, s_full[tile], p_full[tile], pv_done[tile], p_half[tile] (P of keys
// 0-63 written), k_full/k_empty[stage], v_full/v_empty[stage]
constexpr int kBarQ = 0, kBarS = 1, kBarP = 3, kBarPV = 5, kBarPH = 7, kBarKF = 9;
constexpr int kBarKE = kBarKF + kStages, kBarVF = kBarKE + kStages, kBarVE = kBarVF + kStages;
constexpr int kNumBars = kBarVE + kStages;
constexpr int kOffCtlP = kOffBarP + 8 * kNumBars;
constexpr int kMaxSeg = kTQ;
constexpr int kMaxWinSort = 1024;              // windows ranked longest first (else in order)
constexpr int kSchedWord = 16;                 // workspace header words: next item, CTAs done

struct CtlP {
  uint32_t tmem_base;
  int item[2];             // work item of even / odd iterations (from the atomic counter)
  int abort;               // set when a bounded wait timed out: stop after this item
  int nsub;                // ranked entries present (split ranking)
  int nseg;
  int seg_first[kMaxSeg];  // window-relative first token of each segment
  int seg_last[kMaxSeg];
  long long seg_seq[kMaxSeg];
  int seg_keys[kMaxSeg];   // keys the segment's last row attends (max position + 1, clamped)
};
constexpr int kOffSort = (kOffCtlP + static_cast<int>(sizeof(CtlP)) + 15) / 16 * 16;
constexpr int kCostBins = 1024;                // counting-sort bins (cost -1 .. 1022, clamped)
constexpr int kOffHist = kOffSort + 2 * 4 * kMaxWinSort;  // after the window cost and order
constexpr int kSmemP = kOffHist + 4 * kCostBins + 1024;

// 2^x for a pair of fp32 values on the FMA pipe, offloading the MUFU unit (which computes
// 16 exponentials per clock per SM, as many as the tensor core needs here at full rate).
// Method: Cody-Waite range reduction 2^x = 2^n * 2^f with n = rint(x) (the 1.5 * 2^23
// addition trick, round-to-nearest), f in [-1/2, 1/2], and a cubic for 2^f whose
// coefficients are a minimax fit for relative error made for this kernel by iteratively
// reweighted least squares (Lawson's algorithm) on 4001 Chebyshev nodes: fit error
// 7.5e-5, measured 1.3e-4 in fp32 evaluation (bf16 P keeps 2^-9 = 2.0e-3).  Inputs are
// clamped to >= -126 so 2^n stays a normal power of two; the result for x < -126 is
// below 1.2e-38 instead of 0, which no sum of P notices.  2^n is applied by adding
// n << 23 to the exponent field: the low 9 bits of rint's float pattern hold n mod 512.
__device__ __forceinline__ uint64_t exp2_poly2(uint64_t x2) {
  float x0, x1;
  f2unpack(x2, x0, x1);
  x2 = f2pack(fmaxf(x0, -126.f), fmaxf(x1, -126.f));
  const uint64_t magic = f2pack(12582912.f, 12582912.f), nmagic = f2pack(-12582912.f, -12582912.f);
  const uint64_t j2 = add2(x2, magic);
  const uint64_t r2 = add2(j2, nmagic);                       // rint(x), exact
  const uint64_t f2 = fma2(r2, f2pack(-1.f, -1.f), x2);       // x - rint(x), exact
  uint64_t p2 = fma2(f2pack(0x1.c3f76p-5f, 0x1.c3f76p-5f), f2, f2pack(0x1.f0de1cp-3f, 0x1.f0de1cp-3f));
  p2 = fma2(p2, f2, f2pack(0x1.62f31ap-1f, 0x1.62f31ap-1f));
  p2 = fma2(p2, f2, f2pack(0x1.fff692p-1f, 0x1.fff692p-1f));
  float p0, p1, j0, j1;
  f2unpack(p2, p0, p1);
  f2unpack(j2, j0, j1);
  return f2pack(__int_as_float(__float_as_int(p0) + (__float_as_int(j0) << 23)),
                __int_as_float(__float_as_int(p1) + (__float_as_int(j1) << 23)));
}

// Bounded wait whose outcome every lane of the warp shares (a lane that timed out makes
// the whole warp leave together, so no later warp-wide operation waits on a missing lane).
__device__ __forceinline__ bool wait_warp(uint32_t bar, uint32_t parity) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity));
}

__device__ __forceinline__ int seg_blocks(const CtlP* ctl, int s) {
  return (ctl->seg_keys[s] + kNB - 1) / kNB;
}

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
  const uint32_t sQ = sb + kOffQ, sK0 = sb + kOffK, sV0 = sb + kOffV;
  const uint32_t bars = sb + kOffBarP;
  auto bar = [&](int i) { return bars + 8 * i; };
  CtlP* ctl = reinterpret_cast<CtlP*>(smem + kOffCtlP);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  int* wcost = reinterpret_cast<int*>(smem + kOffSort);
  int* worder = wcost + kMaxWinSort;
  int* hist = reinterpret_cast<int*>(smem + kOffHist);
  unsigned* sched = a.err + kSchedWord;
  const int nwin = static_cast<int>((a.T + kTQ - 1) / kTQ);
  const bool ranked = nwin <= kMaxWinSort;
  // Split ranking: a window whose first and last tokens start different prefill runs is two
  // entries, its last segment and the rest, so the two halves of a window that straddles
  // chunks run on different SMs (otherwise it walks the key blocks of both and is the
  // longest item of the launch).  Entry 2w: the whole window w, or its segments but the last
  // one; entry 2w + 1: the last segment, or absent (cost -1).
  const bool split = 2 * nwin <= kMaxWinSort;
  const int nent = split ? 2 * nwin : nwin;
  // This CTA's first work item is taken from the counter now; its round trip overlaps the
  // set-up and ranking below (CTAs that start earlier still take earlier, longer items).
  const int first_item = tid == 0 ? static_cast<int>(atomicAdd(sched, 1u)) : 0;

  if (tid == 0) {
    mbar_init(bar(kBarQ), 1);
    for (int t = 0; t < kTiles; ++t) {
      mbar_init(bar(kBarS + t), 1);
      mbar_init(bar(kBarP + t), 128);
      mbar_init(bar(kBarPV + t), 1);
      mbar_init(bar(kBarPH + t), 128);
    }
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar(kBarKF + s), 2);  // two producer warps per K block
      mbar_init(bar(kBarKE + s), 1);
      mbar_init(bar(kBarVF + s), 1);
      mbar_init(bar(kBarVE + s), 1);
    }
    fence_mbar_init();
    ctl->abort = 0;
    ctl->nsub = 0;
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(&ctl->tmem_base), kTmemCols);
    tmem_relinquish();
  }
  // Longest first: a window's cost estimates the key blocks its segments walk from its
  // first and last tokens only (eight independent loads): the last token's segment walks
  // ceil(keys / 128) blocks, and a different first segment at most ceil((pos + 32) / 128).
  // Windows are ranked by cost, ties by window index, so every CTA builds the same order.
  if (ranked) {
    auto seq_at = [&](long long t) {
      return t >= 0 && t < a.T ? ld_index(a.seq, a.seq64, t) : -2 - t;  // matches no row
    };
    auto blocks_of = [&](long long keys) {
      return static_cast<int>((min(max(keys, 0ll), a.W * kPage) + kNB - 1) / kNB);
    };
    for (int b = tid; b < kCostBins; b += kThreadsP) hist[b] = 0;
    for (int w = tid; w < nwin; w += kThreadsP) {
      const long long ts = static_cast<long long>(w) * kTQ, te = min(ts + kTQ - 1, a.T - 1);
      const long long s0 = seq_at(ts - 1), s1 = seq_at(ts), s2 = seq_at(ts + 1);
      const long long e0 = seq_at(te - 1), e1 = seq_at(te), e2 = seq_at(te + 1);
      const long long ps = ld_index(a.pos, a.pos64, ts), pe = ld_index(a.pos, a.pos64, te);
      const int c_last = (e1 == e0 || e1 == e2) ? blocks_of(pe + 1) : 0;  // last segment
      const int c_first =
          (s1 != e1 && (s1 == s0 || s1 == s2)) ? blocks_of(ps + kTQ) : 0;   // first segment
      if (split) {
        const bool two = c_first > 0 && c_last > 0;
        wcost[2 * w] = two ? c_first : c_first + c_last;
        wcost[2 * w + 1] = two ? c_last : -1;
      } else {
        wcost[w] = c_first + c_last;
      }
    }
    // Rank = entries of higher cost + entries of equal cost and lower index (highest cost
    // first, ties by index), by a stable counting sort in linear work: a histogram of the
    // costs (bin = cost + 1, so absent entries fall in bin 0 and rank last; costs above 1022
    // share the top bin), an exclusive scan from the top bin down, then one warp places the
    // entries in index order, 32 at a time.  (Counting each entry's rank over all entries
    // costs ~5 instructions per pair: ~7 us per CTA at 1,024 entries.)
    __syncthreads();
    {
      auto bin_of = [&](int c) { return min(c, kCostBins - 2) + 1; };
      for (int e = tid; e < nent; e += kThreadsP) atomicAdd(&hist[bin_of(wcost[e])], 1);
      __syncthreads();
      if (warp == 0) {
        int local = 0;  // lane l scans bins 1023 - 32 l down to 992 - 32 l
#pragma unroll 8
        for (int i = 0; i < 32; ++i) local += hist[kCostBins - 1 - (lane * 32 + i)];
        int incl = local;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int y = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += y;
        }
        int run = incl - local;
#pragma unroll 8
        for (int i = 0; i < 32; ++i) {
          const int b = kCostBins - 1 - (lane * 32 + i);
          const int h = hist[b];
          hist[b] = run;
          run += h;
        }
        __syncwarp();
        if (lane == 0) ctl->nsub = hist[0];  // entries above bin 0: the present ones
        __syncwarp();
        for (int base = 0; base < nent; base += 32) {
          const int e = base + lane;
          const int b = e < nent ? bin_of(wcost[e]) : -1;
          const unsigned same = __match_any_sync(0xffffffffu, b);
          if (e < nent) worder[hist[b] + __popc(same & ((1u << lane) - 1u))] = e;
          __syncwarp();
          if (e < nent && lane == __ffs(same) - 1) hist[b] += __popc(same);
          __syncwarp();
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;
  const int nitems = (ranked && split ? ctl->nsub : nwin) * a.KVH;

  // Per-role running counters: block barriers keep their phases across work items.
  int jg = 0;      // key blocks processed so far by this CTA
  int qn = 0;      // Q tiles loaded so far (q_full phases)
  bool ok = true;
  struct ItemInfo {
    bool live;
    long long t0;
    int kvh, nseg, nblk_total;
  };
  // Takes the next work item and scans its window's segments (warp 2).  The item slot
  // alternates between iterations: thread 0 may write the next item before a thread that
  // has passed the barrier has read this one.  Nothing else is written between the two
  // barriers, so every thread takes the same decisions.
  int iter = 0;
  auto item_head = [&]() -> ItemInfo {
    if (tid == 0) ctl->item[iter & 1] = iter == 0 ? first_item : static_cast<int>(atomicAdd(sched, 1u));
    named_bar_sync(1, kThreadsP);
    const int item = ctl->item[iter & 1];
    ++iter;
    if (item >= nitems || ctl->abort) return ItemInfo{false, 0, 0, 0, 0};
    const int wi = item / a.KVH;
    const int ent = ranked ? worder[wi] : wi;
    int w = ent, part = 0;  // part 0: every segment, 1: all but the last, 2: the last only
    if (ranked && split) {
      w = ent >> 1;
      part = (ent & 1) ? 2 : (wcost[ent | 1] >= 0 ? 1 : 0);
    }
    const long long t0 = static_cast<long long>(w) * kTQ;
    const int kvh = item % a.KVH;
    // Segments of this 32-token window: maximal runs of prefill tokens of one sequence.
    if (warp == 2) {
      const long long t = t0 + lane;
      long long seq = -1;
      int pre = 0, pos = 0;
      if (t < a.T) {
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
      __syncwarp();
      const int nseg = __popc(sm);
      for (int sgi = 0; sgi < nseg; ++sgi) {  // keys of a segment = max over its rows
        const int f = ctl->seg_first[sgi], l = ctl->seg_last[sgi];
        int v = (lane >= f && lane <= l) ? pos : 0;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
        if (lane == 0) ctl->seg_keys[sgi] = v;
      }
      if (lane == 0) {  // keep the segments of this item's part
        int n = nseg;
        if (part == 2 && n > 1) {
          ctl->seg_first[0] = ctl->seg_first[n - 1];
          ctl->seg_last[0] = ctl->seg_last[n - 1];
          ctl->seg_seq[0] = ctl->seg_seq[n - 1];
          ctl->seg_keys[0] = ctl->seg_keys[n - 1];
          n = 1;
        } else if (part == 1) {
          n = n > 0 ? n - 1 : 0;
        }
        ctl->nseg = n;
      }
    }
    named_bar_sync(1, kThreadsP);
    const int nseg = ctl->nseg;
    int nblk_total = 0;
    for (int s = 0; s < nseg; ++s) nblk_total += seg_blocks(ctl, s);
    return ItemInfo{true, t0, kvh, nseg, nblk_total};
  };

  // The work-item loop is written once per register class so that each keeps its
  // setmaxnreg budget; both pass named barrier 1 the same number of times.
  if (warp < 4) {
    setmaxnreg_dec<kRegsProducer>();
    for (;;) {
      const ItemInfo it = item_head();
      if (!it.live) break;
      const long long t0 = it.t0;
      const int kvh = it.kvh, nseg = it.nseg, nblk_total = it.nblk_total;
      if (nblk_total > 0 && warp != 1) {
        // ============================ TMA producers (3 warps) ============================
        // One thread issues TMA copies one after another, so three warps share each block's
        // 32 page boxes: warp 0 K d 0-63, warp 2 K d 64-127, warp 3 all of V.
        const int r = warp == 0 ? 0 : warp - 1;
        const bool is_v = r == 2;
        const int ndh = is_v ? 2 : 1, dh0 = is_v ? 0 : r;
        const CUtensorMap* tm = is_v ? &tmV : &tmK;
        const uint32_t base0 = is_v ? sV0 : sK0 + dh0 * (kKVBytes / 2);
        const int full0 = is_v ? kBarVF : kBarKF, empty0 = is_v ? kBarVE : kBarKE;
        if (lane == 0) {
          prefetch_tensormap(tm);
          if (r == 0) {
            prefetch_tensormap(&tmQ);
            mbar_arrive_expect_tx(bar(kBarQ), kTiles * kQBytes);  // Q is free: the last item's
                                                                   // MMAs completed before its end
            for (int t = 0; t < kTiles; ++t)
              for (int dh = 0; dh < 2; ++dh)
                tma_load_4d(sQ + t * kQBytes + dh * (kQBytes / 2), &tmQ, bar(kBarQ), 0, dh,
                            kvh * kGroup, static_cast<int>(t0) + t * kTQT);
          }
        }
        // Page ids of block (sgi, j): lanes 0-7, -1 past the segment's pages or out of range.
        auto page_of = [&](int sgi, int j) -> int {
          if (sgi >= nseg || lane >= kPgPerBlk) return -1;
          const int pi = j * kPgPerBlk + lane;
          if (pi >= (ctl->seg_keys[sgi] + kPage - 1) / kPage) return -1;
          const long long pid = ld_index(a.bt, a.bt64, ctl->seg_seq[sgi] * a.bt_sb + pi * a.bt_sn);
          if (pid < 0 || pid >= a.N) {
            atomicOr(a.err, SS_DEVERR_PAGE);
            return -1;
          }
          return static_cast<int>(pid);
        };
        auto advance = [&](int& sgi, int& j) {
          ++j;
          while (sgi < nseg && j >= seg_blocks(ctl, sgi)) {
            ++sgi;
            j = 0;
          }
        };
        int sgi = 0, j = -1;
        advance(sgi, j);
        int pg = page_of(sgi, j);
        for (; sgi < nseg && ok; ++jg) {
          int nsgi = sgi, nj = j;
          advance(nsgi, nj);
          const int pg_next = page_of(nsgi, nj);  // block-table load overlaps this block's copies
          int pgs[kPgPerBlk];
#pragma unroll
          for (int p = 0; p < kPgPerBlk; ++p) pgs[p] = __shfl_sync(0xffffffffu, pg, p);
          if (lane == 0) {
            const int st = jg % kStages;
            ok = mbar_wait(bar(empty0 + st), ((jg / kStages) & 1) ^ 1);
            if (ok) {
              const uint32_t dst = base0 + st * kKVBytes;
              mbar_arrive_expect_tx(bar(full0 + st), ndh * (kKVBytes / 2));
              for (int h = 0; h < ndh; ++h)
#pragma unroll
                for (int p = 0; p < kPgPerBlk; ++p)
                  tma_load_5d_nohint(dst + h * (kKVBytes / 2) + p * (kPage * 128), tm, bar(full0 + st),
                                     0, 0, dh0 + h, kvh, pgs[p]);
            }
          }
          ok = __shfl_sync(0xffffffffu, ok, 0);
          sgi = nsgi;
          j = nj;
          pg = pg_next;
        }
        if (!ok && lane == 0) {
          atomicOr(a.err, SS_DEVERR_TIMEOUT);
          ctl->abort = 1;
        }
      } else if (nblk_total > 0) {
        // ================================ MMA issuer ==================================
        // The whole warp walks the schedule and waits; one elected lane issues.  Descriptors
        // are per-operand bases plus compile-time offsets (the start-address field holds
        // address / 16 in bits 0-13, and no offset here carries out of it).
        constexpr uint32_t idesc_qk = idesc_bf16_f32(128, kNB, 0, 0);
        constexpr uint32_t idesc_pv = idesc_bf16_f32(128, kHDp, 0, 1);
        const bool leader = elect_one();
        uint64_t dq[kTiles], dk[kStages], dv[kStages];
#pragma unroll
        for (int t = 0; t < kTiles; ++t) dq[t] = smem_desc_sw128(sQ + t * kQBytes, 16, 1024);
#pragma unroll
        for (int st = 0; st < kStages; ++st) {
          dk[st] = smem_desc_sw128(sK0 + st * kKVBytes, 16, 1024);
          dv[st] = smem_desc_sw128(sV0 + st * kKVBytes, kKVBytes / 2, 1024);
        }
        ok = wait_warp(bar(kBarQ), qn & 1);
        ++qn;
        // S_t(jg) = Q_t K(jg)^T into columns [128 t, 128 t + 128).
        auto issue_qk = [&](int t, int jg) {
          if (leader) {
            const uint64_t kd = dk[jg % kStages];
#pragma unroll
            for (int kk = 0; kk < kHDp / 16; ++kk) {
              const uint32_t off = ((kk >> 2) * (kKVBytes / 2) + (kk & 3) * 32) >> 4;
              const uint32_t qoff = ((kk >> 2) * (kQBytes / 2) + (kk & 3) * 32) >> 4;
              tc_mma_f16(tmem + t * kNB, dq[t] + qoff, kd + off, idesc_qk, kk > 0 ? 1u : 0u);
            }
            tc_commit(bar(kBarS + t));
          }
          __syncwarp();
        };
        // O_t (+)= P_t(jg) V(jg); P_t sits in the first 64 columns of S_t (16 keys = 8
        // columns per k-step).
        // The first four k-steps (keys 0-63) start as soon as that half of P is written.
        auto issue_pv = [&](int t, int jg, bool first_of_seg) -> bool {
          const uint64_t vd = dv[jg % kStages];
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            if (!wait_warp(bar((half ? kBarP : kBarPH) + t), jg & 1)) return false;
            tc_fence_after();
            if (leader) {
#pragma unroll
              for (int kk = half * 4; kk < half * 4 + 4; ++kk)
                tc_mma_f16_ts(tmem + kColO + t * kHDp, tmem + t * kNB + kk * 8,
                              vd + ((kk * 16 * 128) >> 4), idesc_pv,
                              (!first_of_seg || kk > 0) ? 1u : 0u);
            }
            __syncwarp();
          }
          if (leader) tc_commit(bar(kBarPV + t));
          __syncwarp();
          return true;
        };
        auto commit = [&](int b) {
          if (leader) tc_commit(bar(b));
          __syncwarp();
        };
        int jl = 0;  // blocks of this item
        bool prev_first = false;
        for (int sgi = 0; sgi < nseg && ok; ++sgi) {
          const int nblk = seg_blocks(ctl, sgi);
          for (int j = 0; j < nblk && ok; ++j, ++jg, ++jl) {
            const int st = jg % kStages;
            ok = wait_warp(bar(kBarKF + st), (jg / kStages) & 1);
            if (!ok) break;
            tc_fence_after();
            issue_qk(0, jg);
            if (jl > 0) {
              ok = issue_pv(1, jg - 1, prev_first);
              if (!ok) break;
              commit(kBarVE + (jg - 1) % kStages);  // both tiles have read V(jg - 1)
            }
            issue_qk(1, jg);
            commit(kBarKE + st);                     // both tiles have read K(jg)
            ok = wait_warp(bar(kBarVF + st), (jg / kStages) & 1);
            if (ok) ok = issue_pv(0, jg, j == 0);
            prev_first = (j == 0);
          }
        }
        if (ok) {
          ok = issue_pv(1, jg - 1, prev_first);
          if (ok) commit(kBarVE + (jg - 1) % kStages);
        }
        if (!ok && lane == 0) {
          atomicOr(a.err, SS_DEVERR_TIMEOUT);
          ctl->abort = 1;
        }
      }
      tc_fence_before();
    }
  } else {
    setmaxnreg_inc<kRegsSoftmax>();
    for (;;) {
      const ItemInfo it = item_head();
      if (!it.live) break;
      const long long t0 = it.t0;
      const int kvh = it.kvh, nseg = it.nseg;
      {
        // ============== softmax + epilogue (1 row per thread, one tile per warpgroup) ===========
        const int tt = (warp - 4) >> 2;      // tile of this warpgroup
        const int wq = warp & 3;             // TMEM lane quadrant of this warp
        const int row = wq * 32 + lane;      // tile row = token * 8 + head
        const int rt = tt * kTQT + row / kGroup, rh = row % kGroup;  // window token, head
        const long long t = t0 + rt;
        const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
        const uint32_t tS = tmem + tt * kNB + lane_off, tO = tmem + kColO + tt * kHDp + lane_off;
        const float sc = a.scale_log2;
        for (int sgi = 0; sgi < nseg && ok; ++sgi) {
          const int f = ctl->seg_first[sgi], l = ctl->seg_last[sgi];
          const bool mine = rt >= f && rt <= l && t < a.T;
          const int keys = mine ? token_info(a, t, false).L : 0;
          const int nblk = seg_blocks(ctl, sgi);
          __nv_bfloat16* op = a.out + t * a.o_st + static_cast<long long>(kvh * kGroup + rh) * a.o_sh;
          if (nblk == 0) {  // no row of the segment has keys: zero output rows
            if (mine)
              for (int dd = 0; dd < kHDp; ++dd) op[dd * a.o_sd] = __float2bfloat16(0.f);
            continue;
          }
          // Rows outside the segment compute on whatever their Q row holds and are discarded,
          // so they are never masked (this keeps full blocks mask-free for the whole warp).
          const int lim = mine ? keys : INT_MAX;
          float m_ref = -CUDART_INF_F, lsum = 0.f;
          for (int j = 0; j < nblk; ++j, ++jg) {
            ok = wait_warp(bar(kBarS + tt), jg & 1);
            if (!ok) break;
            tc_fence_after();
            uint32_t sr[4][32];
#pragma unroll
            for (int c = 0; c < 4; ++c) tmem_ld32(tS + c * 32, sr[c]);
            tmem_wait_ld();
            const int nv = lim - j * kNB;  // valid columns of this row in this block
            if (!__all_sync(0xffffffffu, nv >= kNB)) {
#pragma unroll
              for (int c = 0; c < 4; ++c)
#pragma unroll
                for (int i = 0; i < 32; ++i)
                  if (c * 32 + i >= nv) sr[c][i] = __float_as_uint(-CUDART_INF_F);
            }
            // Row max of the raw scores: four independent chains of three-input maxima.
            float mc[4];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              float m = fmaxf(__uint_as_float(sr[c][0]), __uint_as_float(sr[c][1]));
#pragma unroll
              for (int i = 2; i < 32; i += 2)
                m = max3(m, __uint_as_float(sr[c][i]), __uint_as_float(sr[c][i + 1]));
              mc[c] = m;
            }
            const float mblk = max3(mc[0], mc[1], fmaxf(mc[2], mc[3])) * sc;  // sc > 0
            // Keep the reference max unless this block raises it by more than 8 (2^8 in p).
            const bool raise = mblk > m_ref + 8.f;
            const float m_new = raise ? mblk : m_ref;
            const float alpha = raise ? (m_ref == -CUDART_INF_F ? 0.f : ex2(m_ref - m_new)) : 1.f;
            if (j > 0 && __any_sync(0xffffffffu, raise)) {
              // Rescale O_t in place.  S_t(jg) completing implies P_t.V(jg - 1) completed (the
              // MMA thread issued it earlier); the wait below returns at once.
              ok = wait_warp(bar(kBarPV + tt), (jg - 1) & 1);
              if (!ok) break;
              tc_fence_after();
#pragma unroll
              for (int c = 0; c < 4; ++c) {
                uint32_t orow[32];
                tmem_ld32(tO + c * 32, orow);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; ++i) orow[i] = __float_as_uint(__uint_as_float(orow[i]) * alpha);
                tmem_st32(tO + c * 32, orow);
              }
            }
            m_ref = m_new;
            const float ms = m_ref == -CUDART_INF_F ? 0.f : m_ref;
            const uint64_t sc2 = f2pack(sc, sc), nms2 = f2pack(-ms, -ms);
            uint64_t acc[4] = {0, 0, 0, 0};  // four independent packed partial row sums
            // p = 2^(s sc - m): paired fma, then the hardware exponential for most pairs and the
            // polynomial on the FMA pipe for one pair in kPolyEvery; P as bf16 pairs over the
            // first 64 columns of S_t (column c holds keys 2c, 2c + 1).
#pragma unroll
            for (int h2 = 0; h2 < 2; ++h2) {
              uint32_t pk[32];
#pragma unroll
              for (int i = 0; i < 32; ++i) {
                const int k0 = h2 * 64 + 2 * i;
                const uint64_t x2 = fma2(f2pack(__uint_as_float(sr[k0 >> 5][k0 & 31]),
                                                __uint_as_float(sr[(k0 + 1) >> 5][(k0 + 1) & 31])),
                                         sc2, nms2);
                uint64_t p2;
                if ((i % kPolyEvery) == kPolyEvery - 1) {
                  p2 = exp2_poly2(x2);
                } else {
                  float x0, x1;
                  f2unpack(x2, x0, x1);
                  p2 = f2pack(ex2(x0), ex2(x1));
                }
                acc[i & 3] = add2(acc[i & 3], p2);
                float p0, p1;
                f2unpack(p2, p0, p1);
                pk[i] = pack_bf16(p0, p1);
              }
              tmem_st32(tS + h2 * 32, pk);
              tmem_wait_st();  // (also orders a rescale of O_t before the P.V that reads it)
              tc_fence_before();
              mbar_arrive(bar((h2 ? kBarP : kBarPH) + tt));
            }
            float s0, s1;
            f2unpack(add2(add2(acc[0], acc[1]), add2(acc[2], acc[3])), s0, s1);
            lsum = lsum * alpha + (s0 + s1);
          }
          if (!ok) break;
          // ---- epilogue: O_t / l -> bf16 ---------------------------------------------------
          ok = wait_warp(bar(kBarPV + tt), (jg - 1) & 1);
          if (!ok) break;
          tc_fence_after();
          const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
          // Output rows are 16-byte addressable (prefill_supported): 16-byte stores.
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t orow[32];
            tmem_ld32(tO + c * 32, orow);
            tmem_wait_ld();
            if (mine) {
#pragma unroll
              for (int q8 = 0; q8 < 4; ++q8) {
                uint4 v;
                v.x = pack_bf16(__uint_as_float(orow[q8 * 8 + 0]) * inv, __uint_as_float(orow[q8 * 8 + 1]) * inv);
                v.y = pack_bf16(__uint_as_float(orow[q8 * 8 + 2]) * inv, __uint_as_float(orow[q8 * 8 + 3]) * inv);
                v.z = pack_bf16(__uint_as_float(orow[q8 * 8 + 4]) * inv, __uint_as_float(orow[q8 * 8 + 5]) * inv);
                v.w = pack_bf16(__uint_as_float(orow[q8 * 8 + 6]) * inv, __uint_as_float(orow[q8 * 8 + 7]) * inv);
                *reinterpret_cast<uint4*>(op + c * 32 + q8 * 8) = v;
              }
            }
          }
          tc_fence_before();  // O_t reads complete before the next segment's P.V overwrites O_t
        }
        if (!ok && lane == 0) {
          atomicOr(a.err, SS_DEVERR_TIMEOUT);
          ctl->abort = 1;
        }
      }
      tc_fence_before();  // this item's TMEM accesses are ordered before the next item's
    }
  }
  // ---- teardown ------------------------------------------------------------------------
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
  if (tid == 0) {  // the last CTA out returns the work counter to zero for the next launch
    __threadfence();
    if (atomicAdd(sched + 1, 1u) == gridDim.x - 1) {
      atomicExch(sched, 0u);
      atomicExch(sched + 1, 0u);
    }
  }
  // This grid completes only after the decode grid before it (programmatic launch chain,
  // the decode grid's split-K merge included), so a kernel that waits on this grid also
  // waits for every output row of the call.
  griddep_wait();
}

// SMs of the current device (the persistent grid has one CTA per SM).
int sm_count() {
  static std::mutex mu;
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev] == 0 &&
      cudaDeviceGetAttribute(&cache[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    cache[dev] = 148;
  return cache[dev];
}

// The setmaxnreg split needs the kernel to launch with kLaunchRegs registers per thread.
bool launch_regs_ok() {
  static std::once_flag once;
  static bool ok = false;
  std::call_once(once, [] {
    cudaFuncAttributes fa;
    ok = cudaFuncGetAttributes(&fa, prefill_attention_kernel<kHDp>) == cudaSuccess &&
         fa.numRegs == kLaunchRegs;
  });
  return ok;
}

}  // namespace

bool prefill_supported(const AttnArgs& a) {
  // scale_log2 > 0: the row max is taken over the unscaled scores.
  return a.D == kHDp && a.group == kGroup && a.q_sd == 1 && (a.q_sh % 8) == 0 &&
         (a.q_st % 8) == 0 && (reinterpret_cast<uintptr_t>(a.q) & 15) == 0 &&
         a.o_sd == 1 && (a.o_sh % 8) == 0 && (a.o_st % 8) == 0 &&
         (reinterpret_cast<uintptr_t>(a.out) & 15) == 0 && a.scale_log2 > 0.f &&
         launch_regs_ok();
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
  const long long items = (a.T + kTQ - 1) / kTQ * a.KVH;
  cfg.gridDim = dim3(static_cast<unsigned>(std::min<long long>(items, sm_count())));
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
