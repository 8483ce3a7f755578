"""Generates tests/golden/metadata_<case>.npz by running the REFERENCE metadata build itself.

For every plan below this script imports ShardServe unchanged from the reference checkout
(the directory named by the SHARDSERVE_REFERENCE environment variable), reserves the plan's requests
in the reference's own `Blocks` allocator (shardserve/cache.py:6-35, so block ids follow its
free-list order) and records the output of `metadata(plan, cache, 'cpu', context, bucket)`
(shardserve/runtime.py:28-49).  Stored: the plan (as JSON text), the block tables, the
allocator size, context and bucket, and every output tensor.

Run once in a container that has the reference (it is not needed afterwards):
    python tests/golden/make_golden_metadata.py
"""
from __future__ import annotations

import json
import os
import random
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.environ.get("SHARDSERVE_REFERENCE")
if not REF:
    sys.exit("set SHARDSERVE_REFERENCE to the reference checkout (its shardserve package)")
sys.path.insert(0, REF)
from shardserve.cache import Blocks  # noqa: E402
from shardserve.runtime import metadata  # noqa: E402


class _Cache:  # the attributes metadata() reads from a Cache
    def __init__(self, blocks):
        self.blocks = blocks


def make_plan(kind: str, seed: int):
    """(capacity per request, rows) for a plan of this kind; rows follow scheduler.py:129."""
    rnd = random.Random(seed)
    rows, caps, offset = [], {}, 0
    if kind == "decode":
        specs = [(f"r{i}", rnd.randint(1, 3000), 1) for i in range(12)]
    elif kind == "mixed":
        specs = [(f"d{i}", rnd.randint(16, 2000), 1) for i in range(5)]
        specs += [(f"p{i}", rnd.randint(0, 700), rnd.randint(2, 300)) for i in range(3)]
    elif kind == "padded":
        specs = [(f"r{i}", rnd.randint(1, 400), 1) for i in range(3)]
    else:  # "boundaries": chunks that start or end on page edges
        specs = [("a", 0, 16), ("b", 16, 17), ("c", 31, 1), ("d", 47, 33), ("e", 4095, 1)]
    for key, cursor, n in specs:
        caps[key] = min(cursor + n + rnd.randint(0, 40), 4096)  # admission caps at context
        tokens = [rnd.randint(1, 150000) for _ in range(n)]
        rows.append(dict(request_id=key, tokens=tokens, context=cursor,
                         positions=list(range(cursor, cursor + n)), offset=offset,
                         query_length=n, sample=rnd.random() < 0.7))
        offset += n
    return caps, rows


CASES = {  # name: (kind, seed, context, bucket, allocator blocks)
    "metadata_decode": ("decode", 1, 4096, None, 4000),
    "metadata_mixed": ("mixed", 2, 4096, None, 2000),
    "metadata_padded": ("padded", 3, 4096, 8, 200),
    "metadata_boundaries": ("boundaries", 4, 4096, None, 600),
}


def main() -> None:
    for name, (kind, seed, context, bucket, count) in CASES.items():
        caps, rows = make_plan(kind, seed)
        blocks = Blocks(count)
        blocks.reserve(caps)
        out = metadata({"rows": rows}, _Cache(blocks), "cpu", context, bucket)
        rec = {k: v.numpy() for k, v in out.items()}
        rec["plan_json"] = np.array(json.dumps(rows))
        rec["tables_json"] = np.array(json.dumps(blocks.tables))
        rec["params"] = np.array([count, context, bucket or 0], dtype=np.int64)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **rec)
        print(name, {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
