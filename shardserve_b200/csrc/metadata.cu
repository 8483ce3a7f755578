// Device-side build of the per-step attention metadata.
//
// Replaces the host loops of the reference's `metadata(plan, cache, device, context, bucket)`
// (shardserve/runtime.py:28-49), which build the block tables, token ids, positions,
// sequence ids, append slots and sampled-token indices of a step in Python and copy each
// to the device.  Here the block list of every live request is kept on the device (written
// once at admission), the host sends one packed int64 buffer per step
//     [rows x 4]   store row (-1: graph-padding row), query length, first position, offset
//     [n_sel]      sampled token indices (runtime.py:39-40)
//     [tokens]     token ids
// and one CTA per table row writes, bit for bit what the reference builds:
//     tables[i, :]   = the request's block list, zeros after it     (runtime.py:35-36)
//     positions[t]   = first position + j, seqs[t] = i               (scheduler.py:129)
//     slots[t]       = table[p / 16] * 16 + p % 16                   (runtime.py:38)
//     padding row i: tables[i, 0] = pad_base + i, one token: id 0, position 0, slot
//                    (pad_base + i) * 16                             (runtime.py:41-44)
// A store row outside the store, a negative position or a position past the request's
// blocks (where the reference's list indexing would raise) sets SS_DEVERR_SEQ / _POS and
// writes slot -1, which the append then skips.
#include <cuda_runtime.h>

#include "attention.cuh"

namespace ss {

namespace {

__global__ void __launch_bounds__(256) build_metadata_kernel(const MetadataArgs m) {
  const long long i = blockIdx.x;  // table row
  const long long* desc = m.packed + 4 * i;
  const long long sr = desc[0], ql = desc[1], p0 = desc[2], off = desc[3];
  const bool pad = sr < 0;
  const bool row_ok = pad || sr < m.store_rows;
  if (!row_ok && m.err && threadIdx.x == 0) atomicOr(m.err, SS_DEVERR_SEQ);
  const int* srow = (!pad && row_ok) ? m.store + sr * m.store_rs : nullptr;
  const long long len = (!pad && row_ok) ? m.store_lens[sr] : (pad ? 1 : 0);
  auto block_at = [&](long long c) -> long long {  // entry c of this row's block list
    if (pad) return c == 0 ? m.pad_base + i : 0;
    return (srow && c < len) ? srow[c] : 0;
  };
  for (long long c = threadIdx.x; c < m.table_cols; c += blockDim.x)
    m.tables[i * m.table_rs + c] = static_cast<int>(block_at(c));
  const long long* ids = m.packed + 4 * m.rows + m.n_sel;
  for (long long j = threadIdx.x; j < ql; j += blockDim.x) {
    const long long t = off + j;
    if (t < 0 || t >= m.tokens) continue;
    const long long p = p0 + j;
    m.ids[t] = ids[t];
    m.positions[t] = p;
    m.seqs[t] = static_cast<int>(i);
    long long slot = -1;
    if (p >= 0 && p / kPage < len && row_ok) {
      slot = block_at(p / kPage) * kPage + p % kPage;
    } else if (m.err) {
      atomicOr(m.err, SS_DEVERR_POS);
    }
    m.slots[t] = slot;
  }
  if (i == 0)
    for (long long s = threadIdx.x; s < m.n_sel; s += blockDim.x)
      m.selected[s] = m.packed[4 * m.rows + s];
}

}  // namespace

cudaError_t launch_build_metadata(const MetadataArgs& m, cudaStream_t stream) {
  build_metadata_kernel<<<static_cast<unsigned>(m.rows), 256, 0, stream>>>(m);
  return cudaGetLastError();
}

}  // namespace ss
