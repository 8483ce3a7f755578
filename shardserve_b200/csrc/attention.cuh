// Internal declarations shared by the attention / append kernels and the C-ABI layer.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/shardserve_b200.h"

namespace ss {

constexpr int kPage = SS_BLOCK_SIZE;  // tokens per KV page (reference kernel.py:8)

// Arguments common to every attention kernel.  Strides are in elements.
struct AttnArgs {
  const __nv_bfloat16* q;
  long long q_st, q_sh, q_sd;
  const void* bt;
  long long bt_sb, bt_sn;
  int bt64;
  const void* seq;
  int seq64;
  const void* pos;
  int pos64;
  __nv_bfloat16* out;
  long long o_st, o_sh, o_sd;
  const __nv_bfloat16* kp;
  long long k_sn, k_ss, k_sh, k_sd;
  const __nv_bfloat16* vp;
  long long v_sn, v_ss, v_sh, v_sd;
  long long T;  // query tokens
  long long B;  // block-table rows
  long long W;  // block-table columns (pages per row)
  long long N;  // pool pages
  int H, KVH, D, group;
  float sm_scale;
  float scale_log2;  // sm_scale * log2(e): softmax runs in base 2
  unsigned* err;     // device error word (workspace byte 0)
};

// Extra state of the split-K decode kernel.
struct DecodeArgs {
  AttnArgs a;
  int kvb;       // KV heads per CTA (1 or 2)
  int nkvblk;    // KVH / kvb
  int G;         // CTAs in the grid
  int min_run;   // see token_in_long_run(); 0 = this launch owns every token
  int lo_ctas;   // wide shape: fewest CTAs that share the decode units (a quarter of the SMs)
  int wide_per;  // wide shape: decode units (pages) per active CTA
  int4* desc;    // [T * nkvblk] split descriptor per row: {parts (0 none, 1 whole), first
                 // CTA, first part in the CTA's second slot, 0}; rewritten every call
  float* part;   // [2 * G] partial-state slots
  unsigned* gbar;  // grid barrier: 64-bit arrival counter (workspace bytes 72..79)
  // Fused append (decode-only launches; app_k null: none).  The step's new K/V rows k / v
  // [T, KVH, D] (unit stride along head_dim, rows 16-byte addressable) go to slots[t]; the
  // CTA that loads a page writes the new rows of its token's sequence that fall in that
  // page, then loads it, so no separate append kernel runs before the call.
  const __nv_bfloat16* app_k;
  const __nv_bfloat16* app_v;
  long long ak_st, ak_sh, av_st, av_sh;
  const void* app_slots;
  int app_slots64;
};

__device__ __forceinline__ long long ld_index(const void* p, int is64, long long i) {
  return is64 ? static_cast<long long>(__ldg(static_cast<const long long*>(p) + i))
              : static_cast<long long>(__ldg(static_cast<const int*>(p) + i));
}

struct TokInfo {
  long long seq;  // block-table row
  int L;          // keys attended: positions 0 .. L-1 (reference: seq_len = pos + 1, kernel.py:119)
  int npages;     // ceil(L / 16)
};

// Decodes one query token's (sequence row, absolute position) pair.  Out-of-range values
// are clamped to something safe and reported through the error word when `report` is set:
//  * seq outside [0, B)          -> no keys (output zeros), SS_DEVERR_SEQ
//  * position < 0                -> no keys (output zeros), SS_DEVERR_POS
//  * position + 1 > 16 * W       -> keys clamped to the 16 * W the table can name, SS_DEVERR_POS
__device__ __forceinline__ TokInfo token_info_from(const AttnArgs& a, long long seq, long long pos,
                                                   bool report) {
  TokInfo r;
  unsigned e = 0;
  long long L = pos + 1;
  if (seq < 0 || seq >= a.B) {
    e |= SS_DEVERR_SEQ;
    L = 0;
  }
  if (pos < 0) {
    e |= SS_DEVERR_POS;
    L = 0;
  } else if (L > a.W * kPage) {
    e |= SS_DEVERR_POS;
    L = a.W * kPage;
  }
  if (e && report) atomicOr(a.err, e);
  r.seq = seq;
  r.L = static_cast<int>(L);
  r.npages = static_cast<int>((L + kPage - 1) / kPage);
  return r;
}
__device__ __forceinline__ TokInfo token_info(const AttnArgs& a, long long t, bool report) {
  return token_info_from(a, ld_index(a.seq, a.seq64, t), ld_index(a.pos, a.pos64, t), report);
}

// Chunked-prefill tokens: a token belongs to a "long run" when at least `min_run`
// consecutive query tokens (itself included) carry its sequence id.  Such tokens are
// processed by the tensor-core prefill kernel; every other token by the split-K decode
// kernel.  Both kernels evaluate this same predicate, so each token has exactly one owner.
__device__ __forceinline__ bool token_in_long_run(const AttnArgs& a, int min_run, long long t,
                                                  long long seq) {
  if (min_run <= 0) return false;
  int n = 1;
  for (long long j = t - 1; j >= 0 && n < min_run; --j) {
    if (ld_index(a.seq, a.seq64, j) != seq) break;
    ++n;
  }
  for (long long j = t + 1; j < a.T && n < min_run; ++j) {
    if (ld_index(a.seq, a.seq64, j) != seq) break;
    ++n;
  }
  return n >= min_run;
}

// ---- host-side launchers (defined next to their kernels) ------------------------------
struct DecodeGeometry {
  int kvb, ng, pr, nkvblk, G, threads;
  size_t smem;
  size_t desc_bytes, part_bytes;  // workspace regions
};

// Geometry of the split-K decode kernel on `device`; false if head_dim/kv layout has no
// decode kernel instance.  `wide`: the launch is followed by prefill tiles, so take the
// one-CTA-per-SM configuration on half of the SMs when the layout has it.
bool decode_geometry(int device, long long tokens, int heads, int kv_heads, int head_dim,
                     bool wide, DecodeGeometry* g, const char** why);
// Wide shape: the grid for a launch of `tokens` query tokens whose block table has `rows` x
// `cols` entries (an upper bound of its decode pages), between a quarter and three quarters
// of the SMs; sets g->G and *per (DecodeArgs::wide_per) and returns the lower bound the
// kernel keeps (DecodeArgs::lo_ctas).
int wide_grid(DecodeGeometry* g, int device, long long rows, long long cols, long long tokens,
              int* per);

// Launches the TMA split-K decode kernel; returns a cudaError_t.
cudaError_t launch_decode(const DecodeGeometry& g, const CUtensorMap& tmK, const CUtensorMap& tmV,
                          const DecodeArgs& d, cudaStream_t stream);

cudaError_t launch_generic_attention(const AttnArgs& a, cudaStream_t stream);

// tcgen05 chunked-prefill tiles (prefill_attention.cu): layouts the tile kernel handles,
// the run length that makes a token a prefill token, and the launch (programmatic
// dependent launch after the decode kernel).
bool prefill_supported(const AttnArgs& a);
int prefill_min_run();
cudaError_t launch_prefill(const CUtensorMap& tmQ, const CUtensorMap& tmK, const CUtensorMap& tmV,
                           const AttnArgs& a, cudaStream_t stream);

struct AppendArgs {
  const __nv_bfloat16* k;
  long long k_st, k_sh, k_sd;
  const __nv_bfloat16* v;
  long long v_st, v_sh, v_sd;
  __nv_bfloat16* kp;
  long long kp_sn, kp_ss, kp_sh, kp_sd;
  __nv_bfloat16* vp;
  long long vp_sn, vp_ss, vp_sh, vp_sd;
  const void* slots;
  int slots64;
  long long T, N;
  int KVH, D;
  unsigned* err;  // may be null
};
cudaError_t launch_kv_append(const AppendArgs& a, bool vectorised, cudaStream_t stream);

// Rotary position embedding of q and k fused with the slot-mapped K/V append
// (rope_append.cu).  The append part reuses AppendArgs (k = the unrotated keys).
struct RopeArgs {
  AppendArgs app;
  const __nv_bfloat16* q;
  long long q_st, q_sh, q_sd;
  __nv_bfloat16* qo;  // rotated queries (may equal q)
  long long qo_st, qo_sh, qo_sd;
  const float* cos;
  const float* sin;
  long long cos_sr, cos_sd, sin_sr, sin_sd;
  long long rows;  // table rows: positions must lie in [0, rows)
  const void* pos;
  int pos64;
  int H;
};
cudaError_t launch_rope_append(const RopeArgs& r, bool vectorised, cudaStream_t stream);

// Per-step attention metadata built on the device (metadata.cu).
struct MetadataArgs {
  const long long* packed;  // [rows x 4 | n_sel | tokens] int64
  long long rows, n_sel, tokens;
  const int* store;         // int32 block lists of live requests, row stride store_rs
  const int* store_lens;    // blocks held by each store row
  long long store_rows, store_rs;
  long long pad_base;       // first graph-padding block (the allocator's block count)
  int* tables;
  long long table_cols, table_rs;
  long long* ids;
  long long* positions;
  int* seqs;
  long long* slots;
  long long* selected;
  unsigned* err;            // may be null
};
cudaError_t launch_build_metadata(const MetadataArgs& m, cudaStream_t stream);

// TP2 o_proj GEMM fused with the two-rank all-reduce (tp2_oproj.cu).
struct OprojArgs {
  long long T, T_max;      // tokens of this call, inbox capacity in tokens
  int N, K;                // output features, per-rank input features
  __nv_bfloat16* out;      // [T, N], row stride out_rs
  long long out_rs;
  const void* local_inbox; // [2][T_max][N / 2] 8-byte words {bf16 pair, epoch}
  void* peer_inbox;        // the other rank's inbox (peer memory)
  int a_rows;              // rows of the attention box actually loaded (<= 128)
  int tile_n;              // output features per CTA (oproj_tile_n)
  int atoms;               // 64-column K atoms per ring stage
  int stages;              // depth of the A/W ring (oproj_ring)
  unsigned* epoch_ctr;     // [0] last completed call number, [1] CTAs finished (device)
  unsigned* err;
};
int oproj_tile_tokens();
int oproj_min_k_step();
int oproj_tile_n(long long tokens);
void oproj_ring(int a_rows, int tn, int k, int* atoms, int* stages);
cudaError_t launch_tp2_oproj(const CUtensorMap& tmA, const CUtensorMap& tmW, const OprojArgs& o,
                             cudaStream_t stream);

// Sets the text ss_last_error_message() returns on this thread (printf-style).
void set_error_message(const char* fmt, ...);

// Workspace layout (fixed per device): [0, 256) header (error word at byte 0, chunked-prefill
// work counter at bytes 64..71, decode grid barrier counter at bytes 72..79:
// zero before the first call, left consistent by every call), then the partial-state region
// (sized for the
// largest decode kernel instance), then one int4 split descriptor per (token, KV block) row.
constexpr size_t kWsHeader = 256;
inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

}  // namespace ss
