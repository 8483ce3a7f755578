"""GPU parity of the device-side metadata build (DeviceMetadata / ss_build_metadata):
bit-exact with the reference's runtime.metadata() output and with the CPU oracle."""
import json
import os
import random

import numpy as np
import pytest
import torch

from oracle.metadata import metadata as oracle_metadata
from helpers import page_allocator
from shardserve_b200 import DeviceMetadata
from shardserve_b200 import kernel as K
from shardserve_b200.metadata import metadata as device_metadata

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
META_CASES = ["metadata_decode", "metadata_mixed", "metadata_padded", "metadata_boundaries"]
KEYS = ("ids", "positions", "tables", "seqs", "slots", "selected")


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return torch.device("cuda:0")


class _Blocks:  # the allocator attributes DeviceMetadata reads
    def __init__(self, tables, count):
        self.tables, self.count = tables, count


def check(out, want):
    for k in KEYS:
        got = out[k].cpu().numpy()
        assert got.dtype == want[k].dtype, k
        np.testing.assert_array_equal(got, want[k], err_msg=k)


@pytest.mark.parametrize("name", META_CASES)
def test_device_metadata_matches_reference_vectors(dev, name):
    z = np.load(os.path.join(HERE, "golden", f"{name}.npz"))
    rows = json.loads(str(z["plan_json"]))
    tables = json.loads(str(z["tables_json"]))
    count, context, bucket = (int(x) for x in z["params"])
    dm = DeviceMetadata(_Blocks(tables, count), dev, context)
    out = dm.build({"rows": rows}, bucket or None)
    check(out, z)
    again = dm.build({"rows": rows}, bucket or None, out={k: torch.empty_like(v) for k, v in out.items()})
    check(again, z)


def _random_plan(rnd, blocks, n_rows, start):
    rows, offset, caps = [], 0, {}
    for i in range(n_rows):
        key = f"q{start + i}"
        cursor = rnd.randint(0, 3000)
        n = 1 if rnd.random() < 0.6 else rnd.randint(2, 200)
        caps[key] = min(cursor + n + rnd.randint(0, 50), 4096)
        rows.append(dict(request_id=key, tokens=[rnd.randint(1, 9999) for _ in range(n)],
                         context=cursor, positions=list(range(cursor, cursor + n)),
                         offset=offset, query_length=n, sample=rnd.random() < 0.5))
        offset += n
    blocks.reserve(caps)
    return rows


def test_device_metadata_tracks_admissions_and_releases(dev):
    """Steps with new requests, released and re-reserved keys, padding buckets and the
    drop-in function; every step equals the oracle on the allocator's current tables."""
    rnd = random.Random(7)
    blocks = page_allocator()(6000)
    cache = type("C", (), {})()
    cache.blocks = blocks
    dm = DeviceMetadata(blocks, dev, 4096, capacity=24)
    live = []
    for step in range(12):
        rows = _random_plan(rnd, blocks, rnd.randint(1, 6), step * 10)
        live += [r["request_id"] for r in rows]
        bucket = 8 if len(rows) <= 8 and step % 3 == 0 else None
        want = oracle_metadata(rows, blocks.tables, blocks.count, 4096, bucket)
        check(dm.build({"rows": rows}, bucket), want)
        check(device_metadata({"rows": rows}, cache, dev, 4096, bucket), want)
        for key in rnd.sample(live, k=min(len(live), 3)):
            blocks.release(key)
            live.remove(key)
        if live and step % 4 == 1:  # re-reserve a released key under a new block list
            key = live.pop()
            blocks.release(key)
            blocks.reserve({key: 900})
            row = dict(request_id=key, tokens=[5], context=899, positions=[899], offset=0,
                       query_length=1, sample=True)
            want = oracle_metadata([row], blocks.tables, blocks.count, 4096)
            check(dm.build({"rows": [row]}), want)
            live.append(key)


def test_position_outside_the_request_blocks_gives_slot_minus_one(dev):
    blocks = _Blocks({"a": [7, 9]}, 100)
    dm = DeviceMetadata(blocks, dev, 4096)
    K._workspace(dev, 4, 16, 2, 128)
    K.device_errors(dev, clear=True)
    row = dict(request_id="a", tokens=[1, 2], context=31, positions=[31, 32], offset=0,
               query_length=2, sample=False)
    out = dm.build({"rows": [row]})
    assert out["slots"].tolist() == [9 * 16 + 15, -1]
    assert K.device_errors(dev) & 0x4
