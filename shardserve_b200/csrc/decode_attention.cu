// Split-K ragged paged attention for decode-style query tokens on B200 (sm_100a).
//
// Reference semantics: shardserve/kernel.py:85-166.  For query token t and head h the
// reference walks the pages of sequence row seq[t] through the block table, masks keys at
// positions >= positions[t] + 1, and runs an fp32 online softmax over q.k * sm_scale.
//
// B200 design (one wave of CTAs, balanced by KV bytes, not by tokens):
//  * Work unit = one 16-token page of one (token, KV-head block).  A prologue scan over
//    the query tokens gives the total U; CTA c owns units [c*chunk, (c+1)*chunk), so every
//    CTA streams the same number of pages however ragged the contexts are.
//  * A producer warp gathers pages through the block table and moves each page of K and of
//    V with ONE 5-D TMA box (128-byte swizzle, loaded by this CTA alone) into a multi-stage ring guarded
//    by mbarriers.  Every byte of K/V is read from HBM once per call: the GROUP query heads
//    sharing a KV head consume the same shared-memory page.
//  * Two consumer warps per KV head take alternate pages.  Per page a warp computes
//    S = Q.K^T (mma.sync m16n8k16, M = query heads of the group, N = 16 keys), an fp32
//    base-2 online softmax with quad shuffles, and O^T += V^T.P^T (M = head_dim, N = heads,
//    K = 16 keys): P goes from the S accumulators straight into the B operand, so the P.V
//    product wastes no padded rows and the accumulator is head_dim x 8 per warp.
//  * A token whose pages span several CTAs leaves fp32 partial (m, l, acc) states.  When
//    every active CTA has streamed its share (a grid-wide barrier: one arrival per CTA; a
//    waiter gives up after ~0.5 ms, since a CTA of the grid may not be resident, and the
//    call's last arrival then merges for it), the same CTAs fold those states into bf16
//    outputs, each taking (split row, 32- or 64-dim slice) items.  Folding inside
//    the grid saves a second kernel's launch and CTA dispatch on every call.
//  * Two CTA shapes.  Decode-only launches: two consumer warps per KV head, 3-4 CTAs per SM
//    on every SM.  Launches followed by chunked-prefill tiles: the wide CTA (five consumer
//    warps per KV head, a 9-18 stage ring, one CTA per SM) on only as many SMs as the decode
//    rows need (~1.3 MB of K/V each, a quarter to three quarters of the SMs); the others
//    exit after the prologue, so the prefill tiles, which fill a whole SM per CTA, start on
//    them while the decode rows stream.
#include <cuda_bf16.h>
#include <math_constants.h>

#include <algorithm>
#include <cmath>
#include <mutex>

#include "attention.cuh"
#include "ptx.cuh"

namespace ss {

namespace {

constexpr int kMinChunk = 4;  // pages: lower bound on a CTA's share (limits tiny splits)
// Pages of its first row a CTA prefetches into L2 before it waits for the preceding grid
// (its block-table entries are read before that wait): the prefetches stream while the
// preceding kernels finish, and the first TMA loads after the wait hit L2.  Measured on the
// batch-64 workload (graph-replayed steps): 0 pages 32.9 us, 4 pages 30.5 us, 8 pages 31.4.
#ifndef SS_DECODE_L2_PREFETCH_PAGES
#define SS_DECODE_L2_PREFETCH_PAGES 4
#endif
constexpr int kPrefetchPages = SS_DECODE_L2_PREFETCH_PAGES;
// Decode-only shape with two KV heads per CTA: depth of each CTA's stage ring, and the CTAs
// per SM its launch bounds assume (its register cap); shared memory sets the actual count.
#ifndef SS_DECODE_NARROW_STAGES
#define SS_DECODE_NARROW_STAGES 3
#endif
#ifndef SS_DECODE_NARROW_REG_CTAS
#define SS_DECODE_NARROW_REG_CTAS 3
#endif
// Consumer warps per KV head of the wide configuration.  A warp holds its stage while it
// computes the page, so the ring keeps (stages - warps per head) pages in flight: 5 warps
// with 9 stages measured best (6 with 8: a decode-heavy mixed step 146.9 us against 140.0;
// 4 with 10: 147.6).
constexpr int kWidePR = 5;
// Bytes of K/V a wide CTA streams beside at most kWideBaseTokens prefill tokens: the active
// wide CTAs are sized so (between a quarter and three quarters of the SMs; the rest exit at
// once and leave their SMs to the prefill tiles).  ~90 CTAs saturate HBM.  With more prefill
// tokens the tiles need more of the SMs, and the share grows as (tokens / 1024)^0.4.
// Measured (graph-replayed steps, 56 decode rows + 512-token chunks, fixed 1.3 / 1.7 / 2.2 /
// 3.0 MB per CTA): 2 chunks 53.5 / 61.8 / 71.3 / 86.3 us, 4 chunks 73.1 / 68.1 / 76.6 / 92.0,
// 8 chunks 105.6 / 100.2 / 101.3 / 107.2, 16 chunks 170.9 / 165.6 / 165.7 / 158.9.
constexpr long long kWideBytesPerCta = 1344LL << 10;
constexpr double kWideBaseTokens = 1024.0;
constexpr double kWideTokenExp = 0.4;

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
  int next_row;  // row of this CTA's next segment (-1: none); lets consumers prefetch its q
  int pad[3];
};
static_assert(sizeof(StageMeta) == 48, "StageMeta layout");

struct Ctl {
  long long r0;  // first row (token * nkvblk + block)
  int off0;      // first page inside r0
  int found;
  int merge_mask;  // grid_barrier's answer: 0 leave, 1 merge own items, 2 merge every item
  int nactive;     // CTAs with units (their merge items), set by the prologue
  int m_np;        // pages of this CTA's merge row (first item), -1: not found by the scan
  long long m_start;  // first unit of that row
  long long chunk;    // units per CTA
  unsigned long long stage_bar;  // mbarrier of the staged index arrays (wide shape)
  long long red[32];
};

// PR = consumer warps per KV head, which take the pages of a segment round robin.  PR = 2
// (two warps per head, 3-4 CTAs per SM) is the configuration for decode-only launches;
// PR = 6 is the wide CTA (one per SM, as many bytes in flight and consumer warps as three
// narrow CTAs) that the chunked-prefill path uses on half of the SMs, so that the prefill
// tiles run on the other half at the same time.
template <int HD, int KVB, int NG, int PR>
struct Traits {
  static constexpr int kNCW = PR * KVB;  // consumer warps: (KV head, page parity)
  static constexpr int kThreads = 32 * (kNCW + 1);
  // CTAs per SM the register cap assumes (shared memory sets the resident count).
  static constexpr int kRegBlocks = PR > 2 ? 1 : (KVB == 2 ? SS_DECODE_NARROW_REG_CTAS : 4);
  static constexpr int kSlab = kPage * KVB * HD * 2;   // one page of K (or V), KVB heads
  static constexpr int kStages = PR > 2 ? (KVB == 2 ? 9 : 18) : (KVB == 2 ? SS_DECODE_NARROW_STAGES : 5);
  static constexpr int kStageBytes = 2 * kSlab;
  static constexpr int kRows = 16 * KVB;  // query-head rows per partial slot
  static constexpr int kSlotFloats = kRows * (HD + 2);
  static constexpr int kAccPerThread = NG * (HD / 16) * 4;  // O^T fragment floats per lane
  static constexpr int kMergePerHead = 32 * kAccPerThread + 32;  // acc + m[16] + l[16]
  static constexpr int kQRows = 8 * NG;  // query-head rows a consumer warp prefetches
  static constexpr int kQBufBytes = kQRows * HD * 2;  // one row block of q, bf16
  static constexpr int kOffMerge = kStages * kStageBytes;
  static constexpr int kOffQ = kOffMerge + KVB * (PR - 1) * kMergePerHead * 4;  // [warp][2][kQBufBytes]
  static constexpr int kOffMeta = kOffQ + kNCW * 2 * kQBufBytes;
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

// Units (pages x KV blocks) a token contributes to this launch; -1 marks a token of this
// launch without keys (its output row is zeros).
// kRuns: the launch may hold chunked-prefill runs (the wide shape only); the narrow shape
// never evaluates the run predicate, which keeps its scan loops out of that kernel's code.
template <bool kRuns>
__device__ __forceinline__ long long token_units(const DecodeArgs& d, long long t, bool report,
                                                 int* npages_out) {
  const TokInfo ti = token_info(d.a, t, report);
  const bool mine = !kRuns || !token_in_long_run(d.a, d.min_run, t, ti.seq);
  const int np = mine ? ti.npages : 0;
  if (npages_out) *npages_out = np;
  if (mine && np == 0) return -1;
  return static_cast<long long>(np) * d.nkvblk;
}

// Out of line (it runs only for tokens without keys) and with plain-value arguments (a
// reference to the kernel's argument block would put a copy of it on the stack).
__device__ __noinline__ void write_zero_token(__nv_bfloat16* out, long long o_st, long long o_sh,
                                              long long o_sd, int H, int D, long long t) {
  const __nv_bfloat16 z = __float2bfloat16(0.f);
  for (int h = 0; h < H; ++h)
    for (int dd = 0; dd < D; ++dd) out[t * o_st + h * o_sh + dd * o_sd] = z;
}

// A token without units in this launch: clear its split descriptors and, for a decode token
// without keys, write its zero output row.  Out of line: it runs only for such tokens.
__device__ __noinline__ void clear_empty_token(int4* desc, int nkvblk, long long t, bool zero,
                                               __nv_bfloat16* out, long long o_st, long long o_sh,
                                               long long o_sd, int H, int D) {
  // The preceding grids (the append, and before it the previous call's merge, which reads
  // the descriptors) may still run: wait for them before writing.
  griddep_wait();
  for (int b = 0; b < nkvblk; ++b) desc[t * nkvblk + b] = make_int4(0, 0, 0, 0);
  if (zero) write_zero_token(out, o_st, o_sh, o_sd, H, D, t);
}

// A CTA leaving before the streaming phase (no units, or a failed staging copy) still
// arrives at the grid barrier, after its descriptor writes, without waiting at it.  Out of
// line, called by every thread of the CTA; returns grid_barrier's answer (2: this arrival
// completed a call in which CTAs gave up, so this CTA merges every item), shared through
// `code` in shared memory.
__device__ int grid_barrier(unsigned* bar, unsigned n, bool wait);
__device__ __noinline__ int arrive_and_leave(unsigned* gbar, unsigned n, int* code) {
  griddep_wait();
  __syncthreads();
  if (threadIdx.x == 0) *code = grid_barrier(gbar, n, false);
  __syncthreads();
  return *code;
}

// A-operand fragments of Q for S = Q.K^T: rows = query heads h0 .. h0+15 of token t.
// k-step kk holds {row r, d 16kk+2qd..+1}, {row r, d +8} and, when NG == 2, the same for
// row r + 8.  Rows >= group are zero.
template <int HD, int NG>
__device__ __forceinline__ void load_q_frags(const AttnArgs& a, long long t, int h0, int group,
                                             int lane, uint32_t (&qa)[HD / 16][2 * NG]) {
  const int r = lane >> 2, qd = lane & 3;
  // The host launches this kernel only for q rows that are 16-byte addressable (unit
  // head_dim stride, head and token strides multiples of 8, 16-byte aligned base).
  const __nv_bfloat16* qt = a.q + t * a.q_st;
  auto ld2 = [&](int row, int dd) -> uint32_t {
    if (row >= group) return 0u;
    const __nv_bfloat16* p = qt + static_cast<long long>(h0 + row) * a.q_sh;
    return __ldg(reinterpret_cast<const unsigned int*>(p + dd));
  };
#pragma unroll
  for (int kk = 0; kk < HD / 16; ++kk) {
    const int d0 = kk * 16 + 2 * qd;
    qa[kk][0] = ld2(r, d0);
    qa[kk][1] = ld2(r, d0 + 8);
    if (NG == 2) {
      qa[kk][2 % (2 * NG)] = ld2(r + 8, d0);
      qa[kk][3 % (2 * NG)] = ld2(r + 8, d0 + 8);
    }
  }
}

// Shared-memory address (swizzled) that lane `lane` supplies to an x4 ldmatrix reading the
// 16 keys x 16 d block starting at d = 16 * kk of KV head g inside a page slab.  Matrices:
// (keys 0-7, d +0..7), (keys 0-7, d +8..15), (keys 8-15, d +0..7), (keys 8-15, d +8..15).
template <int HD>
__device__ __forceinline__ uint32_t slab_addr(uint32_t slab, int g, int kk, int lane) {
  const int mi = lane >> 3;
  const int key = ((mi >> 1) << 3) + (lane & 7);
  const int chunk16 = ((kk * 2) & 7) + (mi & 1);
  const int row = (g * (HD / 64) + (kk >> 2)) * kPage + key;
  return slab + row * 128 + ((chunk16 ^ (key & 7)) << 4);
}

// Grid-wide barrier over n <= 2^16 arrivals, one per CTA, that never waits for a CTA that may
// not be resident.  Counter: one 64-bit word (workspace bytes 72..79, zero before the first
// call) changed only by atomic additions.  Bits 0..47 count arrivals: every call adds exactly
// 2^16 (CTA 0 adds 2^16 - (n - 1), every other CTA 1), so an arrival's old value names its
// call's start (a multiple of 2^16, modulo 2^48) and the call is complete when the field has
// grown by 2^16.  Bits 48..63 count give-ups of the current call.  Every arrival is an
// acq_rel addition by one thread after a CTA barrier (it releases the CTA's partial states and
// descriptors).  A waiter polls with acquire loads for about 0.5 ms; a CTA of the grid that is
// not yet resident (another kernel's CTAs can hold its slot) would otherwise keep it waiting
// for ever, so the waiter then gives up by adding 2^48: if the call completed first, its
// addition says so and it takes it back and merges as usual; otherwise it leaves, and the
// arrival that completes the call sees the give-ups in the value it returns, takes them back
// and merges every item of the call.  A merge writes the same bytes whoever makes it, so an
// item merged twice is harmless.  Returns 0: leave; 1: merge this CTA's own items; 2: merge
// every item of the call.
constexpr unsigned long long kBarrierQuantum = 1ull << 16;
constexpr unsigned long long kGiveUp = 1ull << 48;
constexpr unsigned long long kArrivalMask = kGiveUp - 1;
constexpr long long kGiveUpCycles = 1ll << 20;
__device__ int grid_barrier(unsigned* bar, unsigned n, bool wait) {
  unsigned long long* c = reinterpret_cast<unsigned long long*>(bar);
  const unsigned long long add = blockIdx.x == 0 ? kBarrierQuantum - (n - 1) : 1ull;
  const unsigned long long old = atom_add_acq_rel_gpu_u64(c, add);
  const unsigned long long start = old & kArrivalMask & ~(kBarrierQuantum - 1);
  auto done = [start](unsigned long long v) {
    return ((v - start) & kArrivalMask) >= kBarrierQuantum;
  };
  if (done(old + add)) {  // this arrival completed the call
    const unsigned long long g = old >> 48;
    if (g == 0) return wait ? 1 : 0;
    atom_add_acq_rel_gpu_u64(c, (0ull - g) << 48);
    return 2;
  }
  if (!wait) return 0;
  const long long t0 = clock64();
  while (!done(ld_acquire_gpu_u64(c))) {
    if (clock64() - t0 > kGiveUpCycles) {
      if (!done(atom_add_acq_rel_gpu_u64(c, kGiveUp))) return 0;
      atom_add_acq_rel_gpu_u64(c, 0ull - kGiveUp);
      return 1;
    }
    __nanosleep(64);
  }
  return 1;
}

// Split-K merge after the grid barrier.  Item = (row, SD-column slice of head_dim); active CTA
// c takes items c, c + nactive, ...  A row split over n CTAs left n fp32 partial states
// (unnormalised O, running max m, running sum l per query head, base 2) in slots 2 (cfirst +
// p) (+1 for part 0 when the row starts inside CTA cfirst's range).  Per round every thread
// reads one item's descriptor, the split items are compacted into shared memory, then each
// thread (valid query-head row, SD / 8 dims) folds up to 8 parts per L2 round trip.  Every read
// bypasses L1: the parts come from other SMs during this call.
struct MergeIn {  // what the merge reads and writes (plain values: no kernel-parameter pointer)
  const int4* desc;
  const float* part;
  __nv_bfloat16* out;
  long long o_st, o_sh, o_sd, T;
  int nkvblk, group;
};

template <int HD, int KVB, int NT, int SD>
__device__ __noinline__ void merge_split_rows(const MergeIn d, int cta, int nactive,
                                              uint8_t* scratch, bool known, int4 ds_known) {
  constexpr int R = 16 * KVB;       // query-head rows per partial slot
  constexpr int SF = R * (HD + 2);  // floats per slot
  constexpr int NSL = HD / SD;      // slices per row
  constexpr int kDirect = 8;        // parts folded from registers per round trip
  constexpr int RPP = NT / 8;       // rows per pass (8 threads cover a slice)
  constexpr int NV = SD / 32;       // float4 vectors per thread and part (4 or 8 dims)
  const MergeIn& a = d;
  const int tid = threadIdx.x;
  const int group = a.group;
  const int vrows = KVB * group;    // valid query-head rows of a slot
  long long* items = reinterpret_cast<long long*>(scratch);
  int4* descs = reinterpret_cast<int4*>(scratch + NT * sizeof(long long));
  int* nitems = reinterpret_cast<int*>(scratch + NT * (sizeof(long long) + sizeof(int4)));
  const long long npairs = a.T * d.nkvblk * NSL;
  const long long per_round = static_cast<long long>(nactive) * NT;
  for (long long base = cta; base < npairs; base += per_round) {
    if (tid == 0) *nitems = 0;
    named_bar_sync(1, NT);
    const long long w = base + static_cast<long long>(tid) * nactive;
    if (known) {  // one item, its descriptor computed by the prologue scan
      if (tid == 0) {
        items[0] = w;
        descs[0] = ds_known;
        *nitems = 1;
      }
    } else if (w < npairs) {
      const int4 ds = __ldcg(&d.desc[w / NSL]);
      if (ds.x >= 2) {
        const int k = atomicAdd(nitems, 1);
        items[k] = w;
        descs[k] = ds;
      }
    }
    named_bar_sync(1, NT);
    const int n = *nitems;
    for (int it = 0; it < n; ++it) {
      const long long rr = items[it] / NSL;
      const int sl = static_cast<int>(items[it] % NSL);
      const int4 ds = descs[it];
      const int nparts = ds.x, cfirst = ds.y, late = ds.z;
      const long long t = rr / d.nkvblk;
      const int b = static_cast<int>(rr % d.nkvblk);
      for (int v0 = 0; v0 < vrows; v0 += RPP) {
        const int vr = v0 + tid / 8;
        if (vr >= vrows) continue;
        const int srow = (vr / group) * 16 + vr % group;
        const int dcol = sl * SD + (tid % 8) * (4 * NV);
        float M = -CUDART_INF_F, L = 0.f;
        float4 o[NV];
#pragma unroll
        for (int k = 0; k < NV; ++k) o[k] = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int p0 = 0; p0 < nparts; p0 += kDirect) {
          float mv[kDirect], lv[kDirect];
          float4 vv[kDirect][NV];
#pragma unroll
          for (int u = 0; u < kDirect; ++u) {
            mv[u] = -CUDART_INF_F;
            lv[u] = 0.f;
#pragma unroll
            for (int k = 0; k < NV; ++k) vv[u][k] = make_float4(0.f, 0.f, 0.f, 0.f);
            const int pi = p0 + u;
            if (pi < nparts) {
              const float* ps =
                  d.part + static_cast<long long>(2 * (cfirst + pi) + ((pi == 0 && late) ? 1 : 0)) * SF;
              mv[u] = __ldcg(ps + R * HD + srow);
              lv[u] = __ldcg(ps + R * HD + R + srow);
#pragma unroll
              for (int k = 0; k < NV; ++k)
                vv[u][k] = __ldcg(reinterpret_cast<const float4*>(ps + srow * HD + dcol + 4 * k));
            }
          }
          float Mn = M;
#pragma unroll
          for (int u = 0; u < kDirect; ++u) Mn = fmaxf(Mn, mv[u]);
          const float ms = Mn == -CUDART_INF_F ? 0.f : Mn;
          const float sc = ex2(M - ms);
          L *= sc;
#pragma unroll
          for (int k = 0; k < NV; ++k) {
            o[k].x *= sc;
            o[k].y *= sc;
            o[k].z *= sc;
            o[k].w *= sc;
          }
#pragma unroll
          for (int u = 0; u < kDirect; ++u) {
            const float wgt = ex2(mv[u] - ms);
            L += lv[u] * wgt;
#pragma unroll
            for (int k = 0; k < NV; ++k) {
              o[k].x += vv[u][k].x * wgt;
              o[k].y += vv[u][k].y * wgt;
              o[k].z += vv[u][k].z * wgt;
              o[k].w += vv[u][k].w * wgt;
            }
          }
          M = Mn;
        }
        const float inv = L > 0.f ? 1.f / L : 0.f;
        __nv_bfloat16* op = a.out + t * a.o_st +
                            static_cast<long long>((b * KVB + vr / group) * group + vr % group) * a.o_sh;
        // Output rows are 16-byte addressable (checked by the host): 8-byte stores.
#pragma unroll
        for (int k = 0; k < NV; ++k)
          *reinterpret_cast<uint2*>(op + dcol + 4 * k) =
              make_uint2(pack_bf16(o[k].x * inv, o[k].y * inv), pack_bf16(o[k].z * inv, o[k].w * inv));
      }
    }
    named_bar_sync(1, NT);  // the compacted list is rebuilt next round
  }
}

template <int HD, int KVB, int NG, int PR>
__global__ void __launch_bounds__(Traits<HD, KVB, NG, PR>::kThreads, Traits<HD, KVB, NG, PR>::kRegBlocks)
    decode_attention_kernel(const __grid_constant__ CUtensorMap tmK,
                            const __grid_constant__ CUtensorMap tmV, const DecodeArgs d) {
  using Tr = Traits<HD, KVB, NG, PR>;
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
    ctl->found = 0;
    ctl->m_np = -1;
  }
  if (warp == Tr::kNCW && lane == 0) {
    prefetch_tensormap(&tmK);
    prefetch_tensormap(&tmV);
  }
  if constexpr (PR > 2) {
    // Wide shape: the prefill tiles launched after this grid need none of its results, only
    // the pool pages the preceding append writes.  Wait for the append here and let them
    // start at once (on the SMs this grid leaves free) instead of after the prologue.
    griddep_wait();
    griddep_launch_dependents();
  }

  // ---- prologue: total units, this CTA's range, and its first (row, page) ------------
  // Tokens without units in this launch get their split descriptor cleared (and, for
  // decode tokens without keys, a zero output row) by CTA t % G.
  auto note_empty = [&](long long t, long long u) {
    // t < 2^31 (token indices are int in the stage metadata): a 32-bit modulo
    if (static_cast<unsigned>(t) % static_cast<unsigned>(d.G) != blockIdx.x) return;
    clear_empty_token(d.desc, d.nkvblk, t, u < 0, a.out, a.o_st, a.o_sh, a.o_sd, a.H, a.D);
  };
  long long U = 0, chunk = 0, u0 = 0;
  // What the split-K merge reads and writes (plain values, no kernel-parameter pointer).
  auto merge_in = [&]() {
    MergeIn mi;
    mi.desc = d.desc;
    mi.part = d.part;
    mi.out = a.out;
    mi.o_st = a.o_st;
    mi.o_sh = a.o_sh;
    mi.o_sd = a.o_sd;
    mi.T = a.T;
    mi.nkvblk = d.nkvblk;
    mi.group = a.group;
    return mi;
  };
  // Every item of the call, by this CTA alone (items of 64 columns; descriptors from memory).
  auto merge_all = [&]() {
    merge_split_rows<HD, KVB, Tr::kNCW * 32, 64>(merge_in(), 0, 1, smem, false,
                                                 make_int4(0, 0, 0, 0));
  };
  auto leave_early = [&]() {
    if (arrive_and_leave(d.gbar, static_cast<unsigned>(d.G), &ctl->merge_mask) == 2 &&
        warp < Tr::kNCW)
      merge_all();
  };
  // Wide shape: the launch carries thousands of prefill tokens, and a scan that loads them
  // token by token (several dependent round trips per pass, several passes) kept the
  // tiles waiting ~13 us.  Instead the sequence-id and position arrays are copied whole into
  // the idle stage ring (one bulk copy each) and scanned from shared memory by rolled loops.
  bool staged = false;
  if constexpr (PR > 2) {
    const long long bs = a.T * (a.seq64 ? 8 : 4), bp = a.T * (a.pos64 ? 8 : 4);
    const long long offp = (bs + 15) & ~15LL;
    staged = offp + bp <= static_cast<long long>(Tr::kStages) * Tr::kStageBytes &&
             (reinterpret_cast<uintptr_t>(a.seq) & 15) == 0 &&
             (reinterpret_cast<uintptr_t>(a.pos) & 15) == 0;
    if (staged) {
      uint8_t* ss = smem;
      uint8_t* sp = smem + offp;
      const uint32_t sbar = smem_u32(&ctl->stage_bar);
      const long long bs16 = bs & ~15LL, bp16 = bp & ~15LL;
      if (tid == 0) {
        mbar_init(sbar, 1);
        fence_mbar_init();
        mbar_arrive_expect_tx(sbar, static_cast<uint32_t>(bs16 + bp16));
        if (bs16) bulk_load(smem_u32(ss), a.seq, static_cast<uint32_t>(bs16), sbar);
        if (bp16) bulk_load(smem_u32(sp), a.pos, static_cast<uint32_t>(bp16), sbar);
      }
      const uint8_t* gs = static_cast<const uint8_t*>(a.seq);
      const uint8_t* gp = static_cast<const uint8_t*>(a.pos);
      for (long long i = bs16 + tid; i < bs; i += NT) ss[i] = gs[i];  // tails (< 16 bytes)
      for (long long i = bp16 + tid; i < bp; i += NT) sp[i] = gp[i];
      __syncthreads();  // barrier initialised, tails stored
      if (__syncthreads_or(!mbar_wait(sbar, 0))) {  // CTA-uniform
        if (tid == 0) atomicOr(a.err, SS_DEVERR_TIMEOUT);
        mbar_wait(sbar, 0);  // let the copies land before the CTA releases its memory
        leave_early();
        return;
      }
      auto seq_at = [&](long long t) -> long long {
        return a.seq64 ? reinterpret_cast<const long long*>(ss)[t]
                       : static_cast<long long>(reinterpret_cast<const int*>(ss)[t]);
      };
      auto pos_at = [&](long long t) -> long long {
        return a.pos64 ? reinterpret_cast<const long long*>(sp)[t]
                       : static_cast<long long>(reinterpret_cast<const int*>(sp)[t]);
      };
      // token_units from the staged arrays (same predicate as token_in_long_run).
      auto units = [&](long long t, bool report, int* np_out) -> long long {
        const long long sq = seq_at(t);
        const TokInfo ti = token_info_from(a, sq, pos_at(t), report);
        bool in_run = false;
        if (d.min_run > 0) {
          int n = 1;
          for (long long j = t - 1; j >= 0 && n < d.min_run && seq_at(j) == sq; --j) ++n;
          for (long long j = t + 1; j < a.T && n < d.min_run && seq_at(j) == sq; ++j) ++n;
          in_run = n >= d.min_run;
        }
        const int np = in_run ? 0 : ti.npages;
        if (np_out) *np_out = np;
        if (!in_run && np == 0) return -1;
        return static_cast<long long>(np) * d.nkvblk;
      };
      const long long per = (a.T + NT - 1) / NT;  // consecutive tokens per thread
      const long long tb = static_cast<long long>(tid) * per, te = min(a.T, tb + per);
      long long s = 0;
#pragma unroll 1
      for (long long t = tb; t < te; ++t) {
        const long long u = units(t, blockIdx.x == 0, nullptr);
        if (u <= 0) note_empty(t, u);
        s += u > 0 ? u : 0;
      }
      long long start = block_excl_scan<NT>(s, ctl, U);
      const long long per_cta = max(1, d.wide_per);
      const long long ctas = min(static_cast<long long>(d.G),
                                 max(static_cast<long long>(d.lo_ctas), (U + per_cta - 1) / per_cta));
      chunk = max((U + ctas - 1) / ctas, static_cast<long long>(kMinChunk));
      u0 = static_cast<long long>(blockIdx.x) * chunk;
      if (u0 >= U) {  // uniform across the CTA; see the wait/trigger order below
        leave_early();
        return;
      }
#pragma unroll 1
      for (long long t = tb; t < te; ++t) {
        int np = 0;
        const long long u = units(t, false, &np);
        if (u > 0 && start <= u0 && u0 < start + u) {
          const long long off = u0 - start;
          ctl->r0 = t * d.nkvblk + off / np;
          ctl->off0 = static_cast<int>(off % np);
          ctl->found = 1;
        }
        start += u > 0 ? u : 0;
      }
    }
  }
  if (!staged) {
    // Each thread scans a run of consecutive tokens (one for batches up to the CTA's thread
    // count), the CTA's exclusive scan of the runs' unit counts gives every thread its
    // first unit, and the thread whose run holds unit u0 records this CTA's first row.
    const long long per = (a.T + NT - 1) / NT;
    const long long tb = static_cast<long long>(tid) * per, te = min(a.T, tb + per);
    // This CTA's first merge item is (row c / slices, slice c % slices): its row's unit
    // range, found by the same scan, spares the merge a descriptor read.
    const int m_row = static_cast<int>(blockIdx.x) / (HD / 32);
    const int m_t = m_row / d.nkvblk, m_b = m_row - m_t * d.nkvblk;
    long long s = 0, m_local = -1;
    int m_np = 0;
#pragma unroll 1
    for (long long t = tb; t < te; ++t) {
      int np = 0;
      const long long u = token_units<(PR > 2)>(d, t, blockIdx.x == 0, &np);
      if (u <= 0) note_empty(t, u);
      if (t == m_t) {
        m_local = s;
        m_np = u > 0 ? np : 0;
      }
      s += u > 0 ? u : 0;
    }
    long long start = block_excl_scan<NT>(s, ctl, U);
    if (m_local >= 0) {
      ctl->m_start = start + m_local + static_cast<long long>(m_b) * m_np;
      ctl->m_np = m_np;
    }
    long long ctas = d.G;  // CTAs that share the units
    if (PR > 2) {
      const long long per_cta = max(1, d.wide_per);
      ctas = min(static_cast<long long>(d.G),
                 max(static_cast<long long>(d.lo_ctas), (U + per_cta - 1) / per_cta));
    }
    chunk = max((U + ctas - 1) / ctas, static_cast<long long>(kMinChunk));
    u0 = static_cast<long long>(blockIdx.x) * chunk;
    if (u0 >= U) {  // uniform across the CTA; see the wait/trigger order below
      leave_early();
      return;
    }
    if (start <= u0 && u0 < start + s) {  // this thread's run holds unit u0
#pragma unroll 1
      for (long long t = tb; t < te; ++t) {
        int np = 0;
        const long long u = token_units<(PR > 2)>(d, t, false, &np);
        if (u > 0 && start <= u0 && u0 < start + u) {
          const long long off = u0 - start;
          ctl->r0 = t * d.nkvblk + off / np;
          ctl->off0 = static_cast<int>(off % np);
          ctl->found = 1;
          break;
        }
        start += u > 0 ? u : 0;
      }
    }
  }
  __syncthreads();
  if (!ctl->found) {  // cannot happen when u0 < U; uniform across the CTA
    leave_early();
    return;
  }
  const int n_units = static_cast<int>(min(chunk, U - u0));
  if (tid == 0) {  // read after the stream
    ctl->nactive = static_cast<int>((U + chunk - 1) / chunk);
    ctl->chunk = chunk;
  }
  // Order of programmatic-launch operations: every CTA waits for the preceding grid (the
  // KV append) before it lets the next grid (prefill tiles or the split-K merge) start, so
  // a dependent grid that starts reads pool pages the append has finished writing.
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
    // Block-table entries of the first 32 pages do not depend on the preceding kernel:
    // fetch them before waiting for it.
    int pf_page = -1;
    // The first row's token data, also taken before the wait and reused for its segment
    // (after griddepcontrol.wait these loads would miss L1 again).
    int np_first = 0;
    TokInfo ti_first;
    long long tf_first = 0;  // fused append: the first row's first new token and its page
    int fnp_first = 1 << 30;
    {
      const long long t = r / d.nkvblk;
      token_units<(PR > 2)>(d, t, false, &np_first);
      const TokInfo ti = token_info(a, t, false);
      ti_first = ti;
      if (d.app_k) {
        tf_first = t;
        while (tf_first > 0 && ld_index(a.seq, a.seq64, tf_first - 1) == ti.seq) --tf_first;
        const long long p_first = ld_index(a.pos, a.pos64, tf_first);
        fnp_first = p_first < 0 ? 0 : static_cast<int>(p_first / kPage);
      }
      const int idx = p + lane;
      if (idx < min(ti.npages, p + remaining)) {
        const long long pid = ld_index(a.bt, a.bt64, ti.seq * a.bt_sb + idx * a.bt_sn);
        pf_page = (pid < 0 || pid >= a.N) ? -2 : static_cast<int>(pid);
      }
      // Pool pages are written only by the preceding append, through L2, so a prefetch
      // issued before waiting for it never leaves a stale copy behind.
      if (lane < kPrefetchPages && pf_page >= 0) {
        const int b0 = static_cast<int>(r % d.nkvblk);
        tma_prefetch_5d(&tmK, 0, 0, 0, b0 * KVB, pf_page);
        tma_prefetch_5d(&tmV, 0, 0, 0, b0 * KVB, pf_page);
      }
    }
    bool use_pf = true;
    // From here on the pool pages (appended by the preceding kernel) and the workspace
    // are touched.
    griddep_wait();
    griddep_launch_dependents();
    while (remaining > 0 && ok) {
      const long long t = r / d.nkvblk;
      const int b = static_cast<int>(r % d.nkvblk);
      if (t >= a.T) {  // the walk and the prologue scan disagree: never expected
        atomicOr(a.err, SS_DEVERR_TIMEOUT);
        break;
      }
      int np = 0;
      TokInfo ti;
      if (use_pf) {  // the first row: its data came before the wait
        np = np_first;
        ti = ti_first;
      } else {
        token_units<(PR > 2)>(d, t, false, &np);
        ti = token_info(a, t, false);
      }
      if (p >= np) {
        ++r;
        p = 0;
        continue;
      }
      const int seg_end = min(np, p + remaining);
      const bool whole = (p == 0 && seg_end == np);
      // Fused append: this row's sequence starts its run of new tokens at t_first (tokens of
      // one sequence are contiguous); pages from the first new position on get their new
      // rows written before they are loaded.
      long long t_first = t;
      int first_new_page = 1 << 30;
      if (use_pf) {  // found before the wait
        t_first = tf_first;
        first_new_page = fnp_first;
      } else if (d.app_k) {
        while (t_first > 0 && ld_index(a.seq, a.seq64, t_first - 1) == ti.seq) --t_first;
        const long long p_first = ld_index(a.pos, a.pos64, t_first);
        first_new_page = p_first < 0 ? 0 : static_cast<int>(p_first / kPage);
      }
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
      if (p == 0 && lane == 0)  // this CTA holds the row's first page: describe the split
        d.desc[r] = make_int4(whole ? 1 : nparts, cfirst, late, 0);
      // The next row with pages inside this CTA's range, if any (lets consumers prefetch
      // its queries); looked up after the segment's first copies are issued.
      int next_row = -1;
      bool next_known = remaining <= seg_end - p;
      const long long bt_row = ti.seq * a.bt_sb;
      for (int pb = p; pb < seg_end && ok; pb += 32) {
        const int idx = pb + lane;
        int page_id = -1;
        if (idx < seg_end) {
          long long pid;
          if (use_pf) {
            pid = pf_page == -2 ? -1 : pf_page;
          } else {
            pid = ld_index(a.bt, a.bt64, bt_row + idx * a.bt_sn);
          }
          if (pid < 0 || pid >= a.N) {
            atomicOr(a.err, SS_DEVERR_PAGE);  // the TMA box reads zeros out of range
          } else {
            page_id = static_cast<int>(pid);
          }
        }
        use_pf = false;
        const int cnt = min(32, seg_end - pb);
        for (int k = 0; k < cnt; ++k) {
          const int pg = __shfl_sync(0xffffffffu, page_id, k);
          if (d.app_k && pb + k >= first_new_page && pg >= 0) {
            // New rows of tokens t_first .. t whose position lies in this page: each lane
            // moves 16 bytes of K and of V (heads b*KVB .. +KVB), then fences the generic
            // writes before the page's TMA load (async proxy).  Other CTAs loading the page
            // write the same bytes themselves.
            constexpr int kChunks = KVB * HD / 8;  // 16-byte chunks per token and tensor
            for (long long t2 = t_first; t2 <= t; ++t2) {
              const long long p2 = ld_index(a.pos, a.pos64, t2);
              if (p2 < 0 || p2 / kPage != pb + k) continue;
              const long long slot2 = ld_index(d.app_slots, d.app_slots64, t2);
              if (slot2 != static_cast<long long>(pg) * kPage + p2 % kPage || slot2 < 0 ||
                  slot2 >= a.N * kPage) {
                // Not the token's own position (runtime.py:38 builds slots so): the row
                // still goes to its slot when that lies in the pool, but this page does not
                // hold it.
                if (lane == 0) atomicOr(a.err, SS_DEVERR_SLOT);
                if (slot2 < 0 || slot2 >= a.N * kPage) continue;
              }
              if (lane < kChunks) {
                const int h = b * KVB + lane / (HD / 8), dd = (lane % (HD / 8)) * 8;
                const long long sp = slot2 / kPage, sr = slot2 % kPage;
                const uint4 kv = __ldg(reinterpret_cast<const uint4*>(d.app_k + t2 * d.ak_st +
                                                                      h * d.ak_sh + dd));
                const uint4 vv = __ldg(reinterpret_cast<const uint4*>(d.app_v + t2 * d.av_st +
                                                                      h * d.av_sh + dd));
                *reinterpret_cast<uint4*>(const_cast<__nv_bfloat16*>(a.kp) + sp * a.k_sn +
                                          sr * a.k_ss + h * a.k_sh + dd) = kv;
                *reinterpret_cast<uint4*>(const_cast<__nv_bfloat16*>(a.vp) + sp * a.v_sn +
                                          sr * a.v_ss + h * a.v_sh + dd) = vv;
              }
            }
            fence_proxy_async_global();
            __syncwarp();
          }
          if (lane == 0) {
            if (!mbar_wait(bar_empty + 8 * stage, phase ^ 1)) {
              ok = false;
            } else {
              // Copies first (expected bytes without the arrival), then the stage metadata,
              // then the arrival that lets the consumers read both.
              const uint32_t dst = sbase + stage * Tr::kStageBytes;
              mbar_expect_tx(bar_full + 8 * stage, Tr::kStageBytes);
              tma_load_5d(dst, &tmK, bar_full + 8 * stage, 0, 0, 0, b * KVB, pg, policy);
              tma_load_5d(dst + Tr::kSlab, &tmV, bar_full + 8 * stage, 0, 0, 0, b * KVB, pg,
                          policy);
              if (!next_known) {
                for (long long r2 = r + 1; r2 < a.T * d.nkvblk; ++r2) {
                  int np2 = 0;
                  token_units<(PR > 2)>(d, r2 / d.nkvblk, false, &np2);
                  if (np2 > 0) {
                    next_row = static_cast<int>(r2);
                    break;
                  }
                }
                next_known = true;
              }
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
              m.next_row = next_row;
              meta[stage] = m;
              mbar_arrive(bar_full + 8 * stage);
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
  griddep_wait();
  griddep_launch_dependents();
  const int g = warp / PR;  // KV head inside the block
  const int j = warp % PR;  // page parity this warp computes
  const int r = lane >> 2, qd = lane & 3;
  const int group = a.group;
  const float sc = a.scale_log2;

  uint32_t qa[HD / 16][2 * NG];
  float acc[NG][HD / 16][4];
  float m0 = -CUDART_INF_F, l0 = 0.f;  // head row r
  float m1 = -CUDART_INF_F, l1 = 0.f;  // head row r + 8 (NG == 2)
#pragma unroll
  for (int kk = 0; kk < HD / 16; ++kk)
#pragma unroll
    for (int i = 0; i < 2 * NG; ++i) qa[kk][i] = 0u;
#pragma unroll
  for (int n = 0; n < NG; ++n)
#pragma unroll
    for (int mt = 0; mt < HD / 16; ++mt) acc[n][mt][0] = acc[n][mt][1] = acc[n][mt][2] = acc[n][mt][3] = 0.f;

  // Queries of the next segment are copied (cp.async, 16 B) into a per-warp double buffer
  // while the current segment streams, when q rows are 16-byte addressable.
  constexpr bool q_vec = true;  // q rows are 16-byte addressable (checked by the host)
  uint8_t* qbuf = smem + Tr::kOffQ + warp * 2 * Tr::kQBufBytes;
  int qslot = 0;
  long long staged_row = -1;  // row whose q sits in qbuf[qslot ^ 1]
  // The first segment's token is known from the prologue: fetch its queries while the
  // first pages are still in flight.
  long long q_row = ctl->r0;
  {
    const long long t0 = q_row / d.nkvblk;
    const int b0 = static_cast<int>(q_row % d.nkvblk);
    load_q_frags<HD, NG>(a, t0, (b0 * KVB + g) * group, group, lane, qa);
  }

  int stage = 0;
  uint32_t phase = 0;
  int pos = 0;  // ring position counter: page `pos` is computed by warp parity pos % PR
  while (true) {
    if (!mbar_wait(bar_full + 8 * stage, phase)) {
      atomicOr(a.err, SS_DEVERR_TIMEOUT);
      break;
    }
    const StageMeta m = meta[stage];
    if (m.flags & kDone) break;
    const int h0 = (m.b * KVB + g) * group;
    if (m.flags & kFirst) {
      const long long row = static_cast<long long>(m.t) * d.nkvblk + m.b;
      if (row == staged_row) {  // prefetched during the previous segment
        asm volatile("cp.async.wait_all;" ::: "memory");
        __syncwarp();
        const uint8_t* qb = qbuf + (qslot ^ 1) * Tr::kQBufBytes;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const int d0 = kk * 16 + 2 * qd;
          qa[kk][0] = r < group ? *reinterpret_cast<const uint32_t*>(qb + (r * HD + d0) * 2) : 0u;
          qa[kk][1] = r < group ? *reinterpret_cast<const uint32_t*>(qb + (r * HD + d0 + 8) * 2) : 0u;
          if (NG == 2) {
            qa[kk][2 % (2 * NG)] =
                r + 8 < group ? *reinterpret_cast<const uint32_t*>(qb + ((r + 8) * HD + d0) * 2) : 0u;
            qa[kk][3 % (2 * NG)] =
                r + 8 < group ? *reinterpret_cast<const uint32_t*>(qb + ((r + 8) * HD + d0 + 8) * 2) : 0u;
          }
        }
      } else if (row != q_row) {
        load_q_frags<HD, NG>(a, m.t, h0, group, lane, qa);
      }
      q_row = -1;
      staged_row = -1;
      if (m.next_row >= 0 && q_vec) {  // start copying the next segment's queries
        const long long nt = m.next_row / d.nkvblk;
        const int nb = m.next_row % d.nkvblk;
        const int nh0 = (nb * KVB + g) * group;
        const int rows = min(group, Tr::kQRows);
        uint8_t* dst = qbuf + qslot * Tr::kQBufBytes;
        __syncwarp();
        for (int c = lane; c < rows * (HD / 8); c += 32) {
          const int rr = c / (HD / 8), cc = (c % (HD / 8)) * 8;
          const __nv_bfloat16* src = a.q + nt * a.q_st + static_cast<long long>(nh0 + rr) * a.q_sh + cc;
          asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst + (rr * HD + cc) * 2)),
                       "l"(src) : "memory");
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
        staged_row = m.next_row;
        qslot ^= 1;  // the buffer just filled is now qbuf[qslot ^ 1]
      }
      m0 = m1 = -CUDART_INF_F;
      l0 = l1 = 0.f;
#pragma unroll
      for (int n = 0; n < NG; ++n)
#pragma unroll
        for (int mt = 0; mt < HD / 16; ++mt)
          acc[n][mt][0] = acc[n][mt][1] = acc[n][mt][2] = acc[n][mt][3] = 0.f;
    }
    if ((pos % PR) != j) {
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_empty + 8 * stage);
    } else {
      const uint32_t ks = sbase + stage * Tr::kStageBytes;
      const uint32_t vs = ks + Tr::kSlab;
      // ---- S = Q K^T: 16 query-head rows x 16 keys (two n-tiles of 8 keys) -----------
      float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int kk = 0; kk < HD / 16; ++kk) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4(slab_addr<HD>(ks, g, kk, lane), b0, b1, b2, b3);
        const uint32_t a_[4] = {qa[kk][0], NG == 2 ? qa[kk][2 % (2 * NG)] : 0u, qa[kk][1],
                                NG == 2 ? qa[kk][3 % (2 * NG)] : 0u};
        mma_16816(s0, a_, b0, b1);
        mma_16816(s1, a_, b2, b3);
      }
      // ---- online softmax over this page's keys (base 2) -------------------------------
      const int kp = m.page * kPage + 2 * qd;  // key of s0[0]; s0[1] = kp+1, s1[*] = kp+8..
      float x[4] = {s0[0] * sc, s0[1] * sc, s1[0] * sc, s1[1] * sc};
      if (kp >= m.L) x[0] = -CUDART_INF_F;
      if (kp + 1 >= m.L) x[1] = -CUDART_INF_F;
      if (kp + 8 >= m.L) x[2] = -CUDART_INF_F;
      if (kp + 9 >= m.L) x[3] = -CUDART_INF_F;
      float mx = fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float mn = fmaxf(m0, mx);
      const float ms = mn == -CUDART_INF_F ? 0.f : mn;
      const float al = ex2(m0 - ms);
      float p[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) p[i] = ex2(x[i] - ms);
      l0 = l0 * al + (p[0] + p[1]) + (p[2] + p[3]);
      m0 = mn;
      float al8 = 1.f;
      float p8[4] = {0.f, 0.f, 0.f, 0.f};
      if (NG == 2) {
        float y[4] = {s0[2] * sc, s0[3] * sc, s1[2] * sc, s1[3] * sc};
        if (kp >= m.L) y[0] = -CUDART_INF_F;
        if (kp + 1 >= m.L) y[1] = -CUDART_INF_F;
        if (kp + 8 >= m.L) y[2] = -CUDART_INF_F;
        if (kp + 9 >= m.L) y[3] = -CUDART_INF_F;
        float my = fmaxf(fmaxf(y[0], y[1]), fmaxf(y[2], y[3]));
        my = fmaxf(my, __shfl_xor_sync(0xffffffffu, my, 1));
        my = fmaxf(my, __shfl_xor_sync(0xffffffffu, my, 2));
        const float mn8 = fmaxf(m1, my);
        const float ms8 = mn8 == -CUDART_INF_F ? 0.f : mn8;
        al8 = ex2(m1 - ms8);
#pragma unroll
        for (int i = 0; i < 4; ++i) p8[i] = ex2(y[i] - ms8);
        l1 = l1 * al8 + (p8[0] + p8[1]) + (p8[2] + p8[3]);
        m1 = mn8;
      }
      // O^T columns are query heads 2qd, 2qd+1 (+8): fetch their rescale factors.
      if (!__all_sync(0xffffffffu, al == 1.f && al8 == 1.f)) {
        const float c0 = __shfl_sync(0xffffffffu, al, (2 * qd) * 4);
        const float c1 = __shfl_sync(0xffffffffu, al, (2 * qd + 1) * 4);
#pragma unroll
        for (int mt = 0; mt < HD / 16; ++mt) {
          acc[0][mt][0] *= c0;
          acc[0][mt][1] *= c1;
          acc[0][mt][2] *= c0;
          acc[0][mt][3] *= c1;
        }
        if (NG == 2) {
          const float c8 = __shfl_sync(0xffffffffu, al8, (2 * qd) * 4);
          const float c9 = __shfl_sync(0xffffffffu, al8, (2 * qd + 1) * 4);
#pragma unroll
          for (int mt = 0; mt < HD / 16; ++mt) {
            acc[NG - 1][mt][0] *= c8;
            acc[NG - 1][mt][1] *= c9;
            acc[NG - 1][mt][2] *= c8;
            acc[NG - 1][mt][3] *= c9;
          }
        }
      }
      // ---- O^T += V^T P^T: M = head_dim (16 per tile), N = 8 heads, K = 16 keys ----------
      const uint32_t pb0 = pack_bf16(p[0], p[1]), pb1 = pack_bf16(p[2], p[3]);
      const uint32_t pc0 = pack_bf16(p8[0], p8[1]), pc1 = pack_bf16(p8[2], p8[3]);
#pragma unroll
      for (int mt = 0; mt < HD / 16; ++mt) {
        uint32_t v[4];
        ldsm_x4_trans(slab_addr<HD>(vs, g, mt, lane), v[0], v[1], v[2], v[3]);
        mma_16816(acc[0][mt], v, pb0, pb1);
        if (NG == 2) mma_16816(acc[NG - 1][mt], v, pc0, pc1);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_empty + 8 * stage);
    }
    ++pos;
    if (++stage == Tr::kStages) {
      stage = 0;
      phase ^= 1;
    }
    if (!(m.flags & kLast)) continue;

    // ---- end of this CTA's segment of a (token, KV block) row --------------------------
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    if (NG == 2) {
      l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
      l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    }
    float* mgh = merge + g * (PR - 1) * Tr::kMergePerHead;  // this head's PR - 1 slots
    if (j != 0) {  // publish this warp's page-parity state into slot j - 1
      float* mg = mgh + (j - 1) * Tr::kMergePerHead;
      float* mg_m = mg + 32 * Tr::kAccPerThread;
      float* mg_l = mg_m + 16;
#pragma unroll
      for (int n = 0; n < NG; ++n)
#pragma unroll
        for (int mt = 0; mt < HD / 16; ++mt)
#pragma unroll
          for (int i = 0; i < 4; ++i) mg[((n * (HD / 16) + mt) * 4 + i) * 32 + lane] = acc[n][mt][i];
      if (qd == 0) {
        mg_m[r] = m0;
        mg_l[r] = l0;
        if (NG == 2) {
          mg_m[r + 8] = m1;
          mg_l[r + 8] = l1;
        }
      }
    }
    named_bar_sync(1, Tr::kNCW * 32);
    const bool whole = (m.flags & kWhole) != 0;
    if (j == 0) {
      // Fold the other page-parity states of head row r (and r + 8) into this warp's.
      float M = m0, L = l0, M8 = m1, L8 = l1;
#pragma unroll
      for (int sl = 0; sl < PR - 1; ++sl) {
        const float* mg = mgh + sl * Tr::kMergePerHead;
        const float* mg_m = mg + 32 * Tr::kAccPerThread;
        const float* mg_l = mg_m + 16;
        const float mo = mg_m[r];
        const float Mn = fmaxf(M, mo);
        const float Ms = Mn == -CUDART_INF_F ? 0.f : Mn;
        const float e = ex2(M - Ms), eo = ex2(mo - Ms);
        L = L * e + mg_l[r] * eo;
        M = Mn;
        float e8 = 1.f, eo8 = 0.f;
        if (NG == 2) {
          const float mo8 = mg_m[r + 8];
          const float Mn8 = fmaxf(M8, mo8);
          const float Ms8 = Mn8 == -CUDART_INF_F ? 0.f : Mn8;
          e8 = ex2(M8 - Ms8);
          eo8 = ex2(mo8 - Ms8);
          L8 = L8 * e8 + mg_l[r + 8] * eo8;
          M8 = Mn8;
        }
        // Per-column (query head) factors of the O^T fragments: heads 2qd and 2qd + 1.
        float E[NG][2], EO[NG][2];
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int src = (2 * qd + c) * 4;
          E[0][c] = __shfl_sync(0xffffffffu, e, src);
          EO[0][c] = __shfl_sync(0xffffffffu, eo, src);
          if (NG == 2) {
            E[NG - 1][c] = __shfl_sync(0xffffffffu, e8, src);
            EO[NG - 1][c] = __shfl_sync(0xffffffffu, eo8, src);
          }
        }
#pragma unroll
        for (int n = 0; n < NG; ++n)
#pragma unroll
          for (int mt = 0; mt < HD / 16; ++mt)
#pragma unroll
            for (int i = 0; i < 4; ++i)
              acc[n][mt][i] = acc[n][mt][i] * E[n][i & 1] +
                              mg[((n * (HD / 16) + mt) * 4 + i) * 32 + lane] * EO[n][i & 1];
      }
      float LL[NG][2];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int src = (2 * qd + c) * 4;
        LL[0][c] = __shfl_sync(0xffffffffu, L, src);
        if (NG == 2) LL[NG - 1][c] = __shfl_sync(0xffffffffu, L8, src);
      }
      if (whole) {
        __nv_bfloat16* ot = a.out + static_cast<long long>(m.t) * a.o_st;
#pragma unroll
        for (int n = 0; n < NG; ++n)
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const int head = 8 * n + 2 * qd + c;
            if (head < group) {
              const float inv = LL[n][c] > 0.f ? 1.f / LL[n][c] : 0.f;
              __nv_bfloat16* o = ot + static_cast<long long>(h0 + head) * a.o_sh;
#pragma unroll
              for (int mt = 0; mt < HD / 16; ++mt) {
                const int dd = mt * 16 + r;
                o[dd] = __float2bfloat16(acc[n][mt][c] * inv);  // unit head_dim stride
                o[dd + 8] = __float2bfloat16(acc[n][mt][2 + c] * inv);
              }
            }
          }
      } else {
        float* ps = d.part + static_cast<long long>(m.slot) * Tr::kSlotFloats;
#pragma unroll
        for (int n = 0; n < NG; ++n)
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const int head = 8 * n + 2 * qd + c;
            float* pr = ps + (g * 16 + head) * HD;
#pragma unroll
            for (int mt = 0; mt < HD / 16; ++mt) {
              pr[mt * 16 + r] = acc[n][mt][c];
              pr[mt * 16 + r + 8] = acc[n][mt][2 + c];
            }
          }
        if (qd == 0) {
          ps[Tr::kRows * HD + g * 16 + r] = M;
          ps[Tr::kRows * HD + Tr::kRows + g * 16 + r] = L;
          if (NG == 2) {
            ps[Tr::kRows * HD + g * 16 + r + 8] = M8;
            ps[Tr::kRows * HD + Tr::kRows + g * 16 + r + 8] = L8;
          }
        }
      }
    }
    named_bar_sync(1, Tr::kNCW * 32);  // merge scratch is reused by the next segment
  }

  // ---- grid barrier, then the split-K merge by every active CTA --------------------------
  // Every CTA of the grid arrives once: the inactive ones (u0 >= U) as they leave the
  // prologue (after clearing the descriptors of tokens without units here), the active ones
  // 0 .. nactive - 1 when every consumer warp is done (the CTA's partial states and
  // descriptors are written: the producer wrote its descriptors before the stage arrivals
  // the consumers waited for).
  const int nactive = ctl->nactive;
  // Merge items go to active CTAs by index (item c of each round to CTA c): a CTA at or past
  // the item count has none, so it arrives and leaves at once, and its SM slot can take a
  // CTA of the next call while the others merge.
  // Items of 32 head_dim columns when no active CTA would get more than one (the merge is
  // then one round trip per CTA), else of 64 columns (half as many items, fewer rounds).
  const long long mrows = a.T * d.nkvblk;
  const bool items32 = mrows * (HD / 32) <= nactive;
  const long long npairs = mrows * (items32 ? HD / 32 : HD / 64);
  bool has_items = blockIdx.x < npairs;
  // At most one item per CTA: its split descriptor follows from the row's unit range; a
  // row inside one CTA (or without units) needs no merge, and its CTA does not wait.
  const bool known = items32 && has_items && ctl->m_np >= 0;
  int4 ds_known = make_int4(0, 0, 0, 0);
  if (known) {
    const long long ms = ctl->m_start, ch = ctl->chunk;
    const int mnp = ctl->m_np;
    if (mnp > 0) {
      const long long cf = ms / ch, cl = (ms + mnp - 1) / ch;
      ds_known = make_int4(static_cast<int>(cl - cf + 1), static_cast<int>(cf),
                           ms != cf * ch ? kFirstPartLate : 0, 0);
    }
    has_items = ds_known.x >= 2;
  }
  named_bar_sync(1, Tr::kNCW * 32);
  if (tid == 0) ctl->merge_mask = grid_barrier(d.gbar, static_cast<unsigned>(d.G), has_items);
  named_bar_sync(1, Tr::kNCW * 32);
  // Decode-only shape: the next grid on the stream (an append or attention call) may launch
  // now; its CTAs take SM slots only as this grid's CTAs leave.  (The wide shape released
  // the prefill tiles at its entry; the grid after them is released by the tiles.)
  if constexpr (PR <= 2) griddep_launch_dependents();
  const int code = ctl->merge_mask;
  // The stage ring is idle (every stage was consumed before the kDone stage): merge scratch.
  if (code == 2) {
    merge_all();
    return;
  }
  if (code == 0 || !has_items) return;
  const MergeIn mi = merge_in();
  if (items32)
    merge_split_rows<HD, KVB, Tr::kNCW * 32, 32>(mi, blockIdx.x, nactive, smem, known, ds_known);
  else
    merge_split_rows<HD, KVB, Tr::kNCW * 32, 64>(mi, blockIdx.x, nactive, smem, false, ds_known);
}


struct CachedOcc {
  int device = -1;
  int blocks = 0;
};

template <int HD, int KVB, int NG, int PR>
int occupancy(int device, const char** why) {
  using Tr = Traits<HD, KVB, NG, PR>;
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
  auto fn = decode_attention_kernel<HD, KVB, NG, PR>;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, Tr::kSmemBytes);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared);
  int blocks = 0;
  if (e == cudaSuccess)
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, fn, Tr::kThreads, Tr::kSmemBytes);
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

template <int HD, int KVB, int NG, int PR>
size_t partial_bytes_of(int device, const char** why) {
  return static_cast<size_t>(2) * sm_count(device) * occupancy<HD, KVB, NG, PR>(device, why) *
         Traits<HD, KVB, NG, PR>::kSlotFloats * sizeof(float);
}

// The partial-state region is sized for the largest kernel instance, so its size and the
// offset of the descriptor region behind it are the same for every call on a device.
size_t partial_region_bytes(int device, const char** why) {
  size_t m = 0;
  m = std::max(m, partial_bytes_of<128, 2, 1, 2>(device, why));
  m = std::max(m, partial_bytes_of<128, 2, 2, 2>(device, why));
  m = std::max(m, partial_bytes_of<128, 1, 1, 2>(device, why));
  m = std::max(m, partial_bytes_of<128, 1, 2, 2>(device, why));
  m = std::max(m, partial_bytes_of<64, 2, 1, 2>(device, why));
  m = std::max(m, partial_bytes_of<64, 2, 2, 2>(device, why));
  m = std::max(m, partial_bytes_of<64, 1, 1, 2>(device, why));
  m = std::max(m, partial_bytes_of<64, 1, 2, 2>(device, why));
  m = std::max(m, partial_bytes_of<128, 2, 1, kWidePR>(device, why));
  m = std::max(m, partial_bytes_of<128, 1, 1, kWidePR>(device, why));
  return align_up(m, 256);
}

template <int HD, int KVB, int NG, int PR>
bool geometry_for(int device, long long tokens, int kv_heads, DecodeGeometry* g, const char** why) {
  using Tr = Traits<HD, KVB, NG, PR>;
  const int per_sm = occupancy<HD, KVB, NG, PR>(device, why);
  if (per_sm <= 0) return false;
  const int sms = sm_count(device);
  if (sms <= 0) {
    *why = "cannot query SM count";
    return false;
  }
  g->kvb = KVB;
  g->ng = NG;
  g->pr = PR;
  g->nkvblk = kv_heads / KVB;
  // The wide configuration has one CTA per SM; the kernel keeps as many of them as its
  // decode rows need (between a quarter and three quarters) and leaves the other SMs to the
  // prefill tiles launched after it.
  g->G = sms * per_sm;
  g->threads = Tr::kThreads;
  g->smem = Tr::kSmemBytes;
  g->part_bytes = partial_region_bytes(device, why);
  g->desc_bytes = align_up(static_cast<size_t>(tokens) * g->nkvblk * sizeof(int4), 256);
  return true;
}

template <int HD, int KVB>
bool geometry_ng(int device, long long tokens, int kv_heads, int group, bool wide,
                 DecodeGeometry* g, const char** why) {
  if (wide && HD == 128 && group <= 8)
    return geometry_for<128, KVB, 1, kWidePR>(device, tokens, kv_heads, g, why);
  return group <= 8 ? geometry_for<HD, KVB, 1, 2>(device, tokens, kv_heads, g, why)
                    : geometry_for<HD, KVB, 2, 2>(device, tokens, kv_heads, g, why);
}

}  // namespace

int wide_grid(DecodeGeometry* g, int device, long long rows, long long cols, long long tokens,
              int* per_out) {
  const int sms = sm_count(device);
  const int lo = std::max(1, sms / 4), hi = std::max(lo, 3 * sms / 4);
  const long long slab = static_cast<long long>(kPage) * g->kvb * 128 * 2;
  // Prefill tokens, about: every token beyond one per block-table row.
  const double pre = static_cast<double>(std::max(0LL, tokens - rows));
  const double scale = std::pow(std::max(1.0, pre / kWideBaseTokens), kWideTokenExp);
  const long long per = std::max(
      1LL, std::min<long long>(1LL << 30,
                               static_cast<long long>(scale * (kWideBytesPerCta / (2 * slab)))));
  *per_out = static_cast<int>(per);
  const long long bound = rows * cols * g->nkvblk;  // decode pages at most
  g->G = static_cast<int>(std::min<long long>(hi, std::max<long long>(lo, (bound + per - 1) / per)));
  return lo;
}

bool decode_geometry(int device, long long tokens, int heads, int kv_heads, int head_dim,
                     bool wide, DecodeGeometry* g, const char** why) {
  const int group = heads / kv_heads;
  if (group > 16) {
    *why = "more than 16 query heads per KV head";
    return false;
  }
  const bool pair = (kv_heads % 2) == 0;
  if (head_dim == 128) {
    return pair ? geometry_ng<128, 2>(device, tokens, kv_heads, group, wide, g, why)
                : geometry_ng<128, 1>(device, tokens, kv_heads, group, wide, g, why);
  }
  if (head_dim == 64) {
    return pair ? geometry_ng<64, 2>(device, tokens, kv_heads, group, wide, g, why)
                : geometry_ng<64, 1>(device, tokens, kv_heads, group, wide, g, why);
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
#define SS_LAUNCH(HD_, KVB_, NG_, PR_)                                                         \
  if (hd == HD_ && g.kvb == KVB_ && g.ng == NG_ && g.pr == PR_)                               \
    return cudaLaunchKernelEx(&cfg, decode_attention_kernel<HD_, KVB_, NG_, PR_>, tmK, tmV, d);
  SS_LAUNCH(128, 2, 1, 2)
  SS_LAUNCH(128, 2, 2, 2)
  SS_LAUNCH(128, 1, 1, 2)
  SS_LAUNCH(128, 1, 2, 2)
  SS_LAUNCH(64, 2, 1, 2)
  SS_LAUNCH(64, 2, 2, 2)
  SS_LAUNCH(64, 1, 1, 2)
  SS_LAUNCH(64, 1, 2, 2)
  SS_LAUNCH(128, 2, 1, kWidePR)
  SS_LAUNCH(128, 1, 1, kWidePR)
#undef SS_LAUNCH
  return cudaErrorInvalidValue;
}

}  // namespace ss
