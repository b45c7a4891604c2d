"""CPU: the host-side split choice of the decode attention (ops.gqa_splits): the splits always cover the table's
columns, split lengths are multiples of the kernel's tile (128 keys for head dim 128, 32 otherwise), one split is
the default (the reference's setting for this model), and the automatic choice splits only small batches of long
caches."""

from __future__ import annotations

import pytest


@pytest.mark.parametrize("hd", [32, 64, 128])
@pytest.mark.parametrize("num_splits", [1, 0, 2, 3, 7])
@pytest.mark.parametrize("batch,kv_heads,max_len", [(1, 4, 1), (1, 4, 4000), (8, 4, 1628), (256, 4, 1628),
                                                     (3, 8, 129), (64, 2, 100000)])
def test_splits_cover_the_table(zb, hd, num_splits, batch, kv_heads, max_len):
    splits, split_len = zb.ops.gqa_splits(batch, kv_heads, max_len, num_splits, hd)
    tile = zb.ops.gqa_tile(hd)
    assert tile == (128 if hd == 128 else 32)
    assert splits >= 1 and split_len % tile == 0 and split_len > 0
    assert splits * split_len >= max_len
    assert (splits - 1) * split_len < max(max_len, 1)  # no split is empty by construction
    if num_splits == 1:
        assert splits == 1


def test_automatic_split_choice(zb):
    # a full batch keeps one split; a single request with a long cache is spread over the SMs
    assert zb.ops.gqa_splits(256, 4, 1628, 0, 128)[0] == 1
    s, length = zb.ops.gqa_splits(1, 4, 16384, 0, 128)
    assert s > 1 and length >= 256
    # never below 256 keys per split
    assert zb.ops.gqa_splits(1, 1, 300, 0, 128)[0] == 1
