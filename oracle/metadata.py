"""CPU oracle of the per-step attention metadata build — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm may import
this module, and only as the checker.  The product path (shardserve_b200) never calls it.

Restates the reference's `metadata(plan, cache, device, context, bucket)`
(shardserve/runtime.py:28-49) on host lists:

* tables   int32 [n, ceil(context / 16)]: row i holds the block list of plan row i
           (cache.blocks.tables[request_id], runtime.py:35-36), zeros after it;
* ids, positions (int64), seqs (int32), slots (int64): one entry per query token, rows in
  plan order; slot = table[p // 16] * 16 + p % 16 (runtime.py:38);
* selected int64: offset + query_length - 1 of every row with sample set (runtime.py:39-40);
* padding rows i in [len(rows), bucket): tables[i, 0] = count + i, one token with id 0,
  position 0, seq i and slot (count + i) * 16 (runtime.py:41-44).
Pinned against the reference's own output by tests/golden/make_golden_metadata.py.
"""
from __future__ import annotations

import numpy as np


def metadata(rows: list, tables_by_key: dict, count: int, context: int,
             bucket: int | None = None) -> dict:
    n = bucket or len(rows)
    tables = np.zeros((n, (context + 15) // 16), dtype=np.int32)
    tokens, positions, seqs, slots, selected = [], [], [], [], []
    for i, row in enumerate(rows):
        table = tables_by_key[row["request_id"]]
        tables[i, :len(table)] = np.asarray(table, dtype=np.int32)
        tokens.extend(row["tokens"])
        positions.extend(row["positions"])
        seqs.extend([i] * row["query_length"])
        slots.extend(table[p // 16] * 16 + p % 16 for p in row["positions"])
        if row["sample"]:
            selected.append(row["offset"] + row["query_length"] - 1)
    for i in range(len(rows), n):
        block = count + i
        tables[i, 0] = block
        tokens.append(0)
        positions.append(0)
        seqs.append(i)
        slots.append(block * 16)
    return dict(ids=np.asarray(tokens, dtype=np.int64),
                positions=np.asarray(positions, dtype=np.int64), tables=tables,
                seqs=np.asarray(seqs, dtype=np.int32), slots=np.asarray(slots, dtype=np.int64),
                selected=np.asarray(selected, dtype=np.int64))
