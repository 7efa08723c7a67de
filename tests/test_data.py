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


def test_stream_file_roundtrip_and_memmap(tmp_path):
    """The on-disk format: a flat uint16 file read back through np.memmap
    (train_baseline.py:161-162) gives the same ids and the same batches."""
    s = rdata.synthetic_stream(5000, seed=4)
    path = rdata.write_stream(tmp_path / "train.bin", s)
    assert path.stat().st_size == 2 * s.size
    mm = rdata.open_stream(path)
    assert mm.dtype == np.uint16 and np.array_equal(np.asarray(mm), s)
    for case in [(0, 4, 16, 4999), (4900, 4, 32, 4999)]:
        x, y, c = rdata.batch_at(mm, *case)
        ox, oy, oc = ost.batch_at(s, *case)
        assert c == oc and torch.equal(x, ox) and torch.equal(y, oy)
    with pytest.raises(ValueError):
        rdata.write_stream(tmp_path / "bad.bin", np.array([0, 70000]))
    (tmp_path / "odd.bin").write_bytes(b"\x00\x01\x02")
    with pytest.raises(ValueError):
        rdata.open_stream(tmp_path / "odd.bin")


@pytest.mark.parametrize("world,rank,limit", [(1, 0, None), (2, 1, None), (2, 0, 700)])
def test_prefetcher_yields_update_batches(world, rank, limit):
    """Every staged update equals update_batches over the same window (padded
    to the full [accumulation, B, T] shape), the ring of pinned slots is
    reused only after release, and the stream's tail ends the iteration."""
    B, T, acc = 3, 16, 2
    s = rdata.synthetic_stream(world * acc * B * T * 5 + 1, seed=8, vocab_size=101, eos=100, mean_doc=30.0)
    limit = len(s) - 1 if limit is None else limit
    pf = rdata.UpdatePrefetcher(s, rank, world, B, T, acc, limit, depth=2)
    seen = 0
    committed = 0
    for staged in pf:
        assert staged.committed == committed
        batches, targets = rdata.update_batches(s, committed, rank, world, B, T, acc, limit)
        assert staged.update_targets == targets
        ids = torch.zeros(acc, B, T, dtype=torch.int64)
        lab = torch.full((acc, B, T), -100, dtype=torch.int64)
        for m, (x, y, _) in enumerate(batches):
            ids[m, :x.shape[0]] = x
            lab[m, :y.shape[0]] = y
        assert torch.equal(staged.ids, ids) and torch.equal(staged.labels, lab)
        pf.release(staged)
        committed += world * acc * B * T
        seen += 1
    assert seen == -(-limit // (world * acc * B * T))
    pf.close()


def test_prefetcher_close_midway():
    s = rdata.synthetic_stream(20_000, seed=2, vocab_size=101, eos=100, mean_doc=30.0)
    pf = rdata.UpdatePrefetcher(s, 0, 1, 2, 16, 2, len(s) - 1, depth=1)
    first = next(pf)
    assert first.committed == 0
    pf.close()  # the thread is blocked on a full queue / free ring: close must not hang
