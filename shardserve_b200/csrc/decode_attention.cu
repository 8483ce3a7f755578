// Split-K ragged paged attention for decode-style query tokens on B200 (sm_100a).
//
// Reference semantics: shardserve/kernel.py:85-166.  For query token t and head h the
// reference walks the pages of sequence row seq[t] through the block table, masks keys at
// positions >= positions[t] + 1, and runs an fp32 online softmax over q.k * sm_scale.
//
// B200 design (one persistent wave, balanced by KV bytes, not by tokens):
//  * Work unit = one 16-token page of one (token, KV-head block).  A prologue scan over
//    the query tokens gives the total U; CTA c owns units [c*chunk, (c+1)*chunk), so every
//    CTA streams the same number of pages regardless of how ragged the contexts are.
//  * A producer warp gathers pages through the block table and moves each page of K and V
//    with ONE 5-D TMA box each (128-byte swizzled, no multicast) into a multi-stage ring
//    guarded by mbarriers.  Every byte of K/V is read from HBM exactly once per call: the
//    GROUP query heads that share a KV head all consume the same shared-memory page.
//  * Consumer warps (2 per KV head, 8 keys each) compute S = Q.K^T and O += P.V with
//    mma.sync bf16 tensor-core tiles (fp32 accumulate); the 16-row M dimension holds the
//    GROUP query heads of the KV head.  Softmax max/sum use quad shuffles, base-2 exponent.
//  * A token whose pages span several CTAs leaves fp32 partial (m, l, acc) states; the
//    last CTA to finish it (atomic ticket, never a spin) merges them and writes bf16.
#include <cuda_bf16.h>
#include <math_constants.h>

#include <algorithm>
#include <mutex>

#include "attention.cuh"
#include "ptx.cuh"

namespace ss {

namespace {

constexpr int kMinChunk = 4;  // pages: lower bound on a CTA's share (limits tiny splits)

enum : int { kFirst = 1, kLast = 2, kWhole = 4, kDone = 8, kFirstPartLate = 16 };

struct StageMeta {
  int t;       // query token
  int b;       // KV-head block
  int page;    // page index inside the token's context
  int L;       // keys attended by the token
  int flags;   // kFirst/kLast/kWhole/kDone/kFirstPartLate
  int slot;    // partial slot written by this CTA (split rows)
  int nparts;  // CTAs sharing this row (split rows)
  int cfirst;  // first CTA of this row (split rows)
};
static_assert(sizeof(StageMeta) == 32, "StageMeta layout");

struct Ctl {
  long long U;       // total units of this launch
  long long chunk;   // units per CTA
  long long u0;      // first unit of this CTA
  long long r0;      // first row (token * nkvblk + block)
  int off0;          // first page inside r0
  int n_units;       // units owned by this CTA
  int last;          // broadcast: this CTA merges the current split row
  int found;
  long long red[32];
};

template <int HD, int KVB>
struct Traits {
  static constexpr int kNCW = 2 * KVB;  // consumer warps: (kv head, key half)
  static constexpr int kThreads = 32 * (kNCW + 1);
  static constexpr int kSlab = kPage * KVB * HD * 2;  // one page of K (or V), KVB heads
  static constexpr int kStages = KVB == 2 ? 3 : 6;
  static constexpr int kStageBytes = 2 * kSlab;
  static constexpr int kRows = 16 * KVB;  // padded query rows per CTA
  static constexpr int kSlotFloats = kRows * (HD + 2);
  static constexpr int kMergeFloats = KVB * 16 * (HD + 2);
  static constexpr int kOffMerge = kStages * kStageBytes;
  static constexpr int kOffMeta = kOffMerge + kMergeFloats * 4;
  static constexpr int kOffBar = kOffMeta + kStages * (int)sizeof(StageMeta);
  static constexpr int kOffCtl = kOffBar + 2 * kStages * 8;
  static constexpr int kSmemBytes = kOffCtl + (int)sizeof(Ctl) + 1024;  // +1024: base alignment
  static_assert(kSlab % 1024 == 0, "128B-swizzled TMA destinations must be 1024-aligned");
};

// ---- block-wide reductions over all kThreads threads ---------------------------------
template <int NT>
__device__ __forceinline__ long long block_sum(long long v, Ctl* ctl) {
  constexpr int NW = NT / 32;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) ctl->red[w] = v;
  __syncthreads();
  long long s = 0;
#pragma unroll
  for (int i = 0; i < NW; ++i) s += ctl->red[i];
  return s;
}

// Exclusive scan; returns this thread's prefix and sets `total`.
template <int NT>
__device__ __forceinline__ long long block_excl_scan(long long v, Ctl* ctl, long long& total) {
  constexpr int NW = NT / 32;
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  long long inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const long long n = __shfl_up_sync(0xffffffffu, inc, o);
    if (l >= o) inc += n;
  }
  __syncthreads();
  if (l == 31) ctl->red[w] = inc;
  __syncthreads();
  long long before = 0;
  total = 0;
#pragma unroll
  for (int i = 0; i < NW; ++i) {
    const long long s = ctl->red[i];
    if (i < w) before += s;
    total += s;
  }
  return before + inc - v;
}

// Units (pages x KV blocks) a token contributes to this launch.
__device__ __forceinline__ long long token_units(const DecodeArgs& d, long long t, bool report,
                                                 int* npages_out) {
  const TokInfo ti = token_info(d.a, t, report);
  const bool mine = !token_in_long_run(d.a, d.min_run, t, ti.seq);
  const int np = mine ? ti.npages : 0;
  if (npages_out) *npages_out = np;
  // A token of this launch with no keys still needs an output row (zeros): flag it with -1.
  if (mine && np == 0) return -1;
  return static_cast<long long>(np) * d.nkvblk;
}

__device__ void write_zero_token(const AttnArgs& a, long long t, int lane, int nlanes) {
  const __nv_bfloat16 z = __float2bfloat16(0.f);
  for (int e = lane; e < a.H * a.D; e += nlanes) {
    const int h = e / a.D, dd = e % a.D;
    a.out[t * a.o_st + h * a.o_sh + dd * a.o_sd] = z;
  }
}

template <int HD, int KVB>
__device__ __forceinline__ void load_q_frags(const AttnArgs& a, long long t, int h0, int group,
                                             int lane, uint32_t (&qa)[HD / 16][4]) {
  const int r = lane >> 2, qd = lane & 3;
  const __nv_bfloat16* qt = a.q + t * a.q_st;
  const bool pair = (a.q_sd == 1) && ((a.q_sh & 1) == 0) && ((a.q_st & 1) == 0) &&
                    ((reinterpret_cast<uintptr_t>(a.q) & 3) == 0);
  auto ld2 = [&](int row, int dd) -> uint32_t {
    if (row >= group) return 0u;
    const __nv_bfloat16* p = qt + static_cast<long long>(h0 + row) * a.q_sh;
    if (pair) return __ldg(reinterpret_cast<const unsigned int*>(p + dd));
    const unsigned short lo = __bfloat16_as_ushort(p[dd * a.q_sd]);
    const unsigned short hi = __bfloat16_as_ushort(p[(dd + 1) * a.q_sd]);
    return static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
  };
#pragma unroll
  for (int kk = 0; kk < HD / 16; ++kk) {
    const int d0 = kk * 16 + 2 * qd;
    qa[kk][0] = ld2(r, d0);
    qa[kk][1] = ld2(r + 8, d0);
    qa[kk][2] = ld2(r, d0 + 8);
    qa[kk][3] = ld2(r + 8, d0 + 8);
  }
}

template <int HD, int KVB>
__global__ void __launch_bounds__(Traits<HD, KVB>::kThreads)
    decode_attention_kernel(const __grid_constant__ CUtensorMap tmK,
                            const __grid_constant__ CUtensorMap tmV, const DecodeArgs d) {
  using Tr = Traits<HD, KVB>;
  constexpr int NT = Tr::kThreads;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_u32(smem);
  StageMeta* meta = reinterpret_cast<StageMeta*>(smem + Tr::kOffMeta);
  float* merge = reinterpret_cast<float*>(smem + Tr::kOffMerge);
  const uint32_t bar_full = sbase + Tr::kOffBar;
  const uint32_t bar_empty = bar_full + 8 * Tr::kStages;
  Ctl* ctl = reinterpret_cast<Ctl*>(smem + Tr::kOffCtl);
  const AttnArgs& a = d.a;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int s = 0; s < Tr::kStages; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, Tr::kNCW);
    }
    fence_mbar_init();
  }
  if (warp == Tr::kNCW && lane == 0) {
    prefetch_tensormap(&tmK);
    prefetch_tensormap(&tmV);
  }

  // ---- prologue: total units, this CTA's range, and its first (row, page) ------------
  constexpr int ITEMS = 4;
  constexpr int CH = NT * ITEMS;
  long long U = 0;
  for (long long base = 0; base < a.T; base += CH) {
    long long s = 0;
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) {
      const long long t = base + static_cast<long long>(tid) * ITEMS + i;
      if (t < a.T) {
        const long long u = token_units(d, t, blockIdx.x == 0, nullptr);
        if (u < 0) {
          if (t % d.G == blockIdx.x) write_zero_token(a, t, 0, 1);
        } else {
          s += u;
        }
      }
    }
    U += block_sum<NT>(s, ctl);
  }
  const long long chunk = max((U + d.G - 1) / d.G, static_cast<long long>(kMinChunk));
  const long long u0 = static_cast<long long>(blockIdx.x) * chunk;
  if (u0 >= U) return;  // uniform across the CTA
  const int n_units = static_cast<int>(min(chunk, U - u0));
  if (tid == 0) ctl->found = 0;
  __syncthreads();
  long long run = 0;
  for (long long base = 0; base < a.T; base += CH) {
    long long us[ITEMS];
    int nps[ITEMS];
    long long s = 0;
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) {
      const long long t = base + static_cast<long long>(tid) * ITEMS + i;
      us[i] = 0;
      nps[i] = 0;
      if (t < a.T) {
        const long long u = token_units(d, t, false, &nps[i]);
        us[i] = u < 0 ? 0 : u;
      }
      s += us[i];
    }
    long long total;
    long long start = run + block_excl_scan<NT>(s, ctl, total);
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) {
      if (us[i] > 0 && start <= u0 && u0 < start + us[i]) {
        const long long t = base + static_cast<long long>(tid) * ITEMS + i;
        const long long off = u0 - start;
        ctl->r0 = t * d.nkvblk + off / nps[i];
        ctl->off0 = static_cast<int>(off % nps[i]);
        ctl->found = 1;
      }
      start += us[i];
    }
    run += total;
    __syncthreads();
    if (ctl->found) break;
  }
  __syncthreads();
  if (!ctl->found) return;  // cannot happen when u0 < U; uniform across the CTA
  // Everything above only read metadata the preceding kernel does not write.  From here on
  // the pool pages (appended by the preceding kernel) and the workspace are touched.
  griddep_wait();

  if (warp == Tr::kNCW) {
    // ============================ producer warp ====================================
    const uint64_t policy = l2_policy_evict_first();
    long long r = ctl->r0;
    int p = ctl->off0;
    long long u = u0;
    int remaining = n_units;
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    while (remaining > 0 && ok) {
      const long long t = r / d.nkvblk;
      const int b = static_cast<int>(r % d.nkvblk);
      if (t >= a.T) {  // the walk and the prologue scan disagree: never expected
        atomicOr(a.err, SS_DEVERR_TIMEOUT);
        break;
      }
      int np = 0;
      token_units(d, t, false, &np);
      const TokInfo ti = token_info(a, t, false);
      if (p >= np) {
        ++r;
        p = 0;
        continue;
      }
      const int seg_end = min(np, p + remaining);
      const bool whole = (p == 0 && seg_end == np);
      const long long row_start = u - p;
      int nparts = 1, slot = 0, cfirst = 0, late = 0;
      if (!whole) {
        const long long cf = row_start / chunk;
        const long long cl = (row_start + np - 1) / chunk;
        nparts = static_cast<int>(cl - cf + 1);
        cfirst = static_cast<int>(cf);
        late = (row_start != cf * chunk) ? kFirstPartLate : 0;
        slot = 2 * blockIdx.x + (u == u0 ? 0 : 1);
      }
      const long long bt_row = ti.seq * a.bt_sb;
      for (int pb = p; pb < seg_end && ok; pb += 32) {
        const int idx = pb + lane;
        int page_id = -1;
        if (idx < seg_end) {
          const long long pid = ld_index(a.bt, a.bt64, bt_row + idx * a.bt_sn);
          if (pid < 0 || pid >= a.N) {
            atomicOr(a.err, SS_DEVERR_PAGE);  // TMA reads zeros for the out-of-range box
          } else {
            page_id = static_cast<int>(pid);
          }
        }
        const int cnt = min(32, seg_end - pb);
        for (int k = 0; k < cnt; ++k) {
          const int pg = __shfl_sync(0xffffffffu, page_id, k);
          if (lane == 0) {
            if (!mbar_wait(bar_empty + 8 * stage, phase ^ 1)) {
              ok = false;
            } else {
              StageMeta m;
              m.t = static_cast<int>(t);
              m.b = b;
              m.page = pb + k;
              m.L = ti.L;
              m.flags = (pb + k == p ? kFirst : 0) | (pb + k == seg_end - 1 ? kLast : 0) |
                        (whole ? kWhole : 0) | late;
              m.slot = slot;
              m.nparts = nparts;
              m.cfirst = cfirst;
              meta[stage] = m;
              const uint32_t dst = sbase + stage * Tr::kStageBytes;
              mbar_arrive_expect_tx(bar_full + 8 * stage, Tr::kStageBytes);
              tma_load_5d(dst, &tmK, bar_full + 8 * stage, 0, 0, 0, b * KVB, pg, policy);
              tma_load_5d(dst + Tr::kSlab, &tmV, bar_full + 8 * stage, 0, 0, 0, b * KVB, pg,
                          policy);
            }
          }
          ok = __shfl_sync(0xffffffffu, ok, 0);
          if (!ok) break;
          if (++stage == Tr::kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      remaining -= seg_end - p;
      u += seg_end - p;
      ++r;
      p = 0;
    }
    if (lane == 0) {
      if (ok && mbar_wait(bar_empty + 8 * stage, phase ^ 1)) {
        meta[stage].flags = kDone;
        mbar_arrive(bar_full + 8 * stage);
      } else {
        atomicOr(a.err, SS_DEVERR_TIMEOUT);
        // Let in-flight copies land before the CTA's shared memory is released.
        for (int s = 0; s < Tr::kStages; ++s) mbar_wait(bar_full + 8 * s, phase);
      }
    }
    return;
  }

  // ============================== consumer warps ======================================
  const int g = warp >> 1;   // KV head inside the block
  const int hk = warp & 1;   // key half: keys 8*hk .. 8*hk+7 of every page
  const int r = lane >> 2, qd = lane & 3;
  const int group = a.group;
  const int key_in = hk * 8 + (lane & 7);
  const float sc = a.scale_log2;

  uint32_t qa[HD / 16][4];
  float acc[HD / 8][4];
  float m0 = -CUDART_INF_F, m1 = -CUDART_INF_F, l0 = 0.f, l1 = 0.f;
#pragma unroll
  for (int nt = 0; nt < HD / 8; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
#pragma unroll
  for (int kk = 0; kk < HD / 16; ++kk) qa[kk][0] = qa[kk][1] = qa[kk][2] = qa[kk][3] = 0u;

  int stage = 0;
  uint32_t phase = 0;
  while (true) {
    if (!mbar_wait(bar_full + 8 * stage, phase)) {
      atomicOr(a.err, SS_DEVERR_TIMEOUT);
      break;
    }
    const StageMeta m = meta[stage];
    if (m.flags & kDone) break;
    const int h0 = (m.b * KVB + g) * group;
    if (m.flags & kFirst) {
      load_q_frags<HD, KVB>(a, m.t, h0, group, lane, qa);
      m0 = m1 = -CUDART_INF_F;
      l0 = l1 = 0.f;
#pragma unroll
      for (int nt = 0; nt < HD / 8; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
    }
    const uint32_t ks = sbase + stage * Tr::kStageBytes;
    const uint32_t vs = ks + Tr::kSlab;

    // ---- S = Q K^T for this warp's 8 keys (M = 16 query-head rows, N = 8 keys) -------
    float s[4] = {0.f, 0.f, 0.f, 0.f}, s2[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int j = 0; j < HD / 32; ++j) {
      const int row = (g * (HD / 64) + (j >> 1)) * kPage + key_in;
      const int chunk16 = ((j & 1) << 2) + (lane >> 3);
      const uint32_t addr = ks + row * 128 + ((chunk16 ^ (key_in & 7)) << 4);
      uint32_t b0, b1, b2, b3;
      ldsm_x4(addr, b0, b1, b2, b3);
      mma_16816(s, qa[2 * j], b0, b1);
      mma_16816(s2, qa[2 * j + 1], b2, b3);
    }
    // ---- online softmax (base 2), rows r and r+8 ---------------------------------------
    const int kpos = m.page * kPage + hk * 8 + 2 * qd;
    float x0 = (s[0] + s2[0]) * sc, x1 = (s[1] + s2[1]) * sc;
    float x2 = (s[2] + s2[2]) * sc, x3 = (s[3] + s2[3]) * sc;
    if (kpos >= m.L) x0 = x2 = -CUDART_INF_F;
    if (kpos + 1 >= m.L) x1 = x3 = -CUDART_INF_F;
    float mx0 = fmaxf(x0, x1), mx1 = fmaxf(x2, x3);
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float ms0 = mn0 == -CUDART_INF_F ? 0.f : mn0;
    const float ms1 = mn1 == -CUDART_INF_F ? 0.f : mn1;
    const float al0 = ex2(m0 - ms0), al1 = ex2(m1 - ms1);
    const float p0 = ex2(x0 - ms0), p1 = ex2(x1 - ms0);
    const float p2 = ex2(x2 - ms1), p3 = ex2(x3 - ms1);
    l0 = l0 * al0 + p0 + p1;
    l1 = l1 * al1 + p2 + p3;
    m0 = mn0;
    m1 = mn1;
#pragma unroll
    for (int nt = 0; nt < HD / 8; ++nt) {
      acc[nt][0] *= al0;
      acc[nt][1] *= al0;
      acc[nt][2] *= al1;
      acc[nt][3] *= al1;
    }
    const uint32_t pa0 = pack_bf16(p0, p1), pa1 = pack_bf16(p2, p3);
    // ---- O += P V (K = this warp's 8 keys, N = head_dim in tiles of 8) ---------------
#pragma unroll
    for (int j = 0; j < HD / 32; ++j) {
      const int row = (g * (HD / 64) + (j >> 1)) * kPage + key_in;
      const int chunk16 = ((j & 1) << 2) + (lane >> 3);
      const uint32_t addr = vs + row * 128 + ((chunk16 ^ (key_in & 7)) << 4);
      uint32_t v0, v1, v2, v3;
      ldsm_x4_trans(addr, v0, v1, v2, v3);
      mma_1688(acc[4 * j + 0], pa0, pa1, v0);
      mma_1688(acc[4 * j + 1], pa0, pa1, v1);
      mma_1688(acc[4 * j + 2], pa0, pa1, v2);
      mma_1688(acc[4 * j + 3], pa0, pa1, v3);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(bar_empty + 8 * stage);
    if (++stage == Tr::kStages) {
      stage = 0;
      phase ^= 1;
    }
    if (!(m.flags & kLast)) continue;

    // ---- end of this CTA's segment of a (token, KV block) row --------------------------
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    float* mg = merge + g * 16 * (HD + 2);
    float* mg_m = mg + 16 * HD;
    float* mg_l = mg_m + 16;
    if (hk == 1) {
#pragma unroll
      for (int nt = 0; nt < HD / 8; ++nt) {
        *reinterpret_cast<float2*>(mg + r * HD + nt * 8 + 2 * qd) = make_float2(acc[nt][0], acc[nt][1]);
        *reinterpret_cast<float2*>(mg + (r + 8) * HD + nt * 8 + 2 * qd) =
            make_float2(acc[nt][2], acc[nt][3]);
      }
      if (qd == 0) {
        mg_m[r] = m0;
        mg_m[r + 8] = m1;
        mg_l[r] = l0;
        mg_l[r + 8] = l1;
      }
    }
    named_bar_sync(1, Tr::kNCW * 32);
    const bool whole = (m.flags & kWhole) != 0;
    if (hk == 0) {
      const float mo0 = mg_m[r], mo1 = mg_m[r + 8];
      const float M0 = fmaxf(m0, mo0), M1 = fmaxf(m1, mo1);
      const float Ms0 = M0 == -CUDART_INF_F ? 0.f : M0, Ms1 = M1 == -CUDART_INF_F ? 0.f : M1;
      const float e0 = ex2(m0 - Ms0), eo0 = ex2(mo0 - Ms0);
      const float e1 = ex2(m1 - Ms1), eo1 = ex2(mo1 - Ms1);
      const float L0 = l0 * e0 + mg_l[r] * eo0, L1 = l1 * e1 + mg_l[r + 8] * eo1;
#pragma unroll
      for (int nt = 0; nt < HD / 8; ++nt) {
        const float2 o0 = *reinterpret_cast<const float2*>(mg + r * HD + nt * 8 + 2 * qd);
        const float2 o1 = *reinterpret_cast<const float2*>(mg + (r + 8) * HD + nt * 8 + 2 * qd);
        acc[nt][0] = acc[nt][0] * e0 + o0.x * eo0;
        acc[nt][1] = acc[nt][1] * e0 + o0.y * eo0;
        acc[nt][2] = acc[nt][2] * e1 + o1.x * eo1;
        acc[nt][3] = acc[nt][3] * e1 + o1.y * eo1;
      }
      if (whole) {
        const float i0 = L0 > 0.f ? 1.f / L0 : 0.f, i1 = L1 > 0.f ? 1.f / L1 : 0.f;
        __nv_bfloat16* ot = a.out + static_cast<long long>(m.t) * a.o_st;
#pragma unroll
        for (int nt = 0; nt < HD / 8; ++nt) {
          const int dd = nt * 8 + 2 * qd;
          if (r < group) {
            __nv_bfloat16* o = ot + static_cast<long long>(h0 + r) * a.o_sh;
            o[dd * a.o_sd] = __float2bfloat16(acc[nt][0] * i0);
            o[(dd + 1) * a.o_sd] = __float2bfloat16(acc[nt][1] * i0);
          }
          if (r + 8 < group) {
            __nv_bfloat16* o = ot + static_cast<long long>(h0 + r + 8) * a.o_sh;
            o[dd * a.o_sd] = __float2bfloat16(acc[nt][2] * i1);
            o[(dd + 1) * a.o_sd] = __float2bfloat16(acc[nt][3] * i1);
          }
        }
      } else {
        float* ps = d.part + static_cast<long long>(m.slot) * Tr::kSlotFloats;
#pragma unroll
        for (int nt = 0; nt < HD / 8; ++nt) {
          const int dd = nt * 8 + 2 * qd;
          *reinterpret_cast<float2*>(ps + (g * 16 + r) * HD + dd) = make_float2(acc[nt][0], acc[nt][1]);
          *reinterpret_cast<float2*>(ps + (g * 16 + r + 8) * HD + dd) =
              make_float2(acc[nt][2], acc[nt][3]);
        }
        if (qd == 0) {
          ps[Tr::kRows * HD + g * 16 + r] = M0;
          ps[Tr::kRows * HD + g * 16 + r + 8] = M1;
          ps[Tr::kRows * HD + Tr::kRows + g * 16 + r] = L0;
          ps[Tr::kRows * HD + Tr::kRows + g * 16 + r + 8] = L1;
        }
      }
    }
    if (!whole) {
      // Publish the partial, take a ticket; the last of the row's CTAs merges.  No CTA
      // ever waits for another: whoever arrives last does the work.
      __threadfence();
      named_bar_sync(1, Tr::kNCW * 32);
      const long long row = static_cast<long long>(m.t) * d.nkvblk + m.b;
      if (tid == 0) {
        const int old = atomicAdd(d.tickets + row, 1);
        const int last = (old == m.nparts - 1);
        if (last) d.tickets[row] = 0;  // ready for the next call
        ctl->last = last;
      }
      named_bar_sync(1, Tr::kNCW * 32);
      if (ctl->last) {
        __threadfence();
        const int rows = KVB * group;
        __nv_bfloat16* ot = a.out + static_cast<long long>(m.t) * a.o_st;
        for (int e = tid; e < rows * (HD / 4); e += Tr::kNCW * 32) {
          const int rr = e / (HD / 4);
          const int d4 = (e % (HD / 4)) * 4;
          const int gg = rr / group, i = rr % group;
          const int prow = gg * 16 + i;
          float M = -CUDART_INF_F;
          for (int pi = 0; pi < m.nparts; ++pi) {
            const int c = m.cfirst + pi;
            const int sl = 2 * c + ((pi == 0 && (m.flags & kFirstPartLate)) ? 1 : 0);
            M = fmaxf(M, __ldcg(d.part + static_cast<long long>(sl) * Tr::kSlotFloats + Tr::kRows * HD + prow));
          }
          const float Ms = M == -CUDART_INF_F ? 0.f : M;
          float Lsum = 0.f;
          float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
          for (int pi = 0; pi < m.nparts; ++pi) {
            const int c = m.cfirst + pi;
            const int sl = 2 * c + ((pi == 0 && (m.flags & kFirstPartLate)) ? 1 : 0);
            const float* ps = d.part + static_cast<long long>(sl) * Tr::kSlotFloats;
            const float w = ex2(__ldcg(ps + Tr::kRows * HD + prow) - Ms);
            Lsum += __ldcg(ps + Tr::kRows * HD + Tr::kRows + prow) * w;
            const float4 v = __ldcg(reinterpret_cast<const float4*>(ps + prow * HD + d4));
            o.x += v.x * w;
            o.y += v.y * w;
            o.z += v.z * w;
            o.w += v.w * w;
          }
          const float inv = Lsum > 0.f ? 1.f / Lsum : 0.f;
          __nv_bfloat16* op = ot + static_cast<long long>((m.b * KVB + gg) * group + i) * a.o_sh;
          op[d4 * a.o_sd] = __float2bfloat16(o.x * inv);
          op[(d4 + 1) * a.o_sd] = __float2bfloat16(o.y * inv);
          op[(d4 + 2) * a.o_sd] = __float2bfloat16(o.z * inv);
          op[(d4 + 3) * a.o_sd] = __float2bfloat16(o.w * inv);
        }
      }
    }
    named_bar_sync(1, Tr::kNCW * 32);  // merge scratch is reused by the next segment
  }
}

template <int HD, int KVB>
struct Instance {
  static void* fn() { return reinterpret_cast<void*>(&decode_attention_kernel<HD, KVB>); }
};

struct CachedOcc {
  int device = -1;
  int blocks = 0;
};

template <int HD, int KVB>
int occupancy(int device, const char** why) {
  using Tr = Traits<HD, KVB>;
  static std::mutex mu;
  static CachedOcc cache[16];
  std::lock_guard<std::mutex> lock(mu);
  if (device < 0 || device >= 16) {
    *why = "device index out of range";
    return 0;
  }
  if (cache[device].device == device) return cache[device].blocks;
  int prev = 0;
  cudaGetDevice(&prev);
  if (prev != device) cudaSetDevice(device);
  cudaError_t e = cudaFuncSetAttribute(decode_attention_kernel<HD, KVB>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, Tr::kSmemBytes);
  int blocks = 0;
  if (e == cudaSuccess)
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, decode_attention_kernel<HD, KVB>,
                                                      Tr::kThreads, Tr::kSmemBytes);
  if (prev != device) cudaSetDevice(prev);
  if (e != cudaSuccess || blocks <= 0) {
    *why = "decode kernel does not fit on this device";
    return 0;
  }
  cache[device].device = device;
  cache[device].blocks = blocks;
  return blocks;
}

int sm_count(int device) {
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return 0;
  return sms;
}

template <int HD, int KVB>
size_t partial_bytes_of(int device, const char** why) {
  return static_cast<size_t>(2) * sm_count(device) * occupancy<HD, KVB>(device, why) *
         Traits<HD, KVB>::kSlotFloats * sizeof(float);
}

// The partial-state region is sized for the largest kernel instance, so its size and the
// offset of the ticket region behind it are the same for every call on a device: tickets
// of one call can never alias partial states another call wrote (tickets must read zero).
size_t partial_region_bytes(int device, const char** why) {
  size_t m = partial_bytes_of<128, 2>(device, why);
  m = std::max(m, partial_bytes_of<128, 1>(device, why));
  m = std::max(m, partial_bytes_of<64, 2>(device, why));
  m = std::max(m, partial_bytes_of<64, 1>(device, why));
  return align_up(m, 256);
}

template <int HD, int KVB>
bool geometry_for(int device, long long tokens, int kv_heads, DecodeGeometry* g, const char** why) {
  using Tr = Traits<HD, KVB>;
  const int per_sm = occupancy<HD, KVB>(device, why);
  if (per_sm <= 0) return false;
  const int sms = sm_count(device);
  if (sms <= 0) {
    *why = "cannot query SM count";
    return false;
  }
  g->kvb = KVB;
  g->nkvblk = kv_heads / KVB;
  g->G = sms * per_sm;
  g->threads = Tr::kThreads;
  g->smem = Tr::kSmemBytes;
  g->part_bytes = partial_region_bytes(device, why);
  g->tickets_bytes = align_up(static_cast<size_t>(tokens) * g->nkvblk * sizeof(int), 256);
  return true;
}

}  // namespace

bool decode_geometry(int device, long long tokens, int heads, int kv_heads, int head_dim,
                     DecodeGeometry* g, const char** why) {
  const int group = heads / kv_heads;
  if (group > 16) {
    *why = "more than 16 query heads per KV head";
    return false;
  }
  const bool pair = (kv_heads % 2) == 0;
  if (head_dim == 128) {
    return pair ? geometry_for<128, 2>(device, tokens, kv_heads, g, why)
                : geometry_for<128, 1>(device, tokens, kv_heads, g, why);
  }
  if (head_dim == 64) {
    return pair ? geometry_for<64, 2>(device, tokens, kv_heads, g, why)
                : geometry_for<64, 1>(device, tokens, kv_heads, g, why);
  }
  *why = "head_dim must be 64 or 128";
  return false;
}

cudaError_t launch_decode(const DecodeGeometry& g, const CUtensorMap& tmK, const CUtensorMap& tmV,
                          const DecodeArgs& d, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(g.G);
  cfg.blockDim = dim3(g.threads);
  cfg.dynamicSmemBytes = g.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const int hd = d.a.D;
  if (hd == 128 && g.kvb == 2) return cudaLaunchKernelEx(&cfg, decode_attention_kernel<128, 2>, tmK, tmV, d);
  if (hd == 128 && g.kvb == 1) return cudaLaunchKernelEx(&cfg, decode_attention_kernel<128, 1>, tmK, tmV, d);
  if (hd == 64 && g.kvb == 2) return cudaLaunchKernelEx(&cfg, decode_attention_kernel<64, 2>, tmK, tmV, d);
  if (hd == 64 && g.kvb == 1) return cudaLaunchKernelEx(&cfg, decode_attention_kernel<64, 1>, tmK, tmV, d);
  return cudaErrorInvalidValue;
}

}  // namespace ss
