"""Token indexing and data-parallel partitioning (CPU): the product's batch_at
and stream against the oracle's restatement of the reference, and the rank
windows against one global batch_at (bit-exact)."""
import numpy as np
import pytest
import torch

from oracle import stream as ost
from reversability_b200 import data as rdata


def test_stream_identical_to_oracle():
    a = rdata.synthetic_stream(20_000, seed=1337)
    b = ost.synthetic_stream(20_000, seed=1337)
    assert np.array_equal(a, b) and a.dtype == np.uint16


@pytest.mark.parametrize("case", [(0, 4, 16, 5999), (100, 3, 17, 150), (5900, 4, 32, 5999), (1, 1, 5, 2)])
def test_batch_at_identical_to_oracle(case):
    s = rdata.synthetic_stream(6000, seed=3, vocab_size=101, eos=100, mean_doc=60.0)
    x, y, c = rdata.batch_at(s, *case)
    ox, oy, oc = ost.batch_at(s, *case)
    assert c == oc and torch.equal(x, ox) and torch.equal(y, oy)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_rank_windows_concatenate_to_global_batch(world):
    B, T, acc = 3, 16, 2
    s = rdata.synthetic_stream(world * acc * B * T * 3 + 1, seed=11, vocab_size=101, eos=100, mean_doc=40.0)
    committed = world * acc * B * T
    gx, gy, gc = rdata.batch_at(s, committed, world * acc * B, T, committed + world * acc * B * T)
    pieces_x, pieces_y, denoms = [], [], set()
    for m in range(acc):
        for r in range(world):
            batches, targets = rdata.update_batches(s, committed, r, world, B, T, acc, len(s) - 1)
            denoms.add(targets)
            pieces_x.append(batches[m][0])
            pieces_y.append(batches[m][1])
    assert denoms == {gc}
    assert torch.equal(torch.cat(pieces_x), gx) and torch.equal(torch.cat(pieces_y), gy)


def test_partial_final_update_pads_and_counts():
    s = np.arange(100, dtype=np.uint16)
    batches, targets = rdata.update_batches(s, 0, 0, 1, 2, 8, 4, 40)
    assert targets == 40
    assert [c for _, _, c in batches] == [16, 16, 8]
    assert int((batches[-1][1] != -100).sum()) == 8
