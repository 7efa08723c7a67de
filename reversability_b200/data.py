"""Token stream and batch indexing for training (product side).

batch_at keeps the exact semantics of the reference trainer's batch_at
(scripts/train_baseline.py:50-63): x = data[c:c+n], y = data[c+1:c+n+1] with
n = min(B*T, limit - cursor), a partial tail padded with x=0 / y=-100, and
StopIteration when nothing is left. The stream format is the reference's
uint16 token file (scripts/prepare_fineweb_edu.py:78); the FineWeb-Edu file is
not available here, so `synthetic_stream` generates a seeded stand-in with the
same vocabulary, EOS convention and dtype: geometric document lengths (mean
900), Zipf(1.1) token ids rejection-sampled into [0, 50256), EOS=50256 after
every document.

Data-parallel partitioning: one update consumes the contiguous window
[committed, committed + world*accumulation*B*T); rank r's microstep m reads
batch_at at committed + (m*world + r)*B*T, so the ranks together read exactly
what one process would read for the same window.

On disk the stream is a flat little-endian uint16 file (`{split}.bin`, the
layout prepare_fineweb_edu.py:78 writes through np.memmap); `open_stream`
maps it read-only like train_baseline.py:161-162. `UpdatePrefetcher` builds
each update's batches on a background thread into page-locked host buffers,
so the host side of an update (batch_at, the int64 widening, pinning) runs
while the previous update is on the GPU and the copy to the device is one
asynchronous transfer per tensor.
"""
from __future__ import annotations

import math
import os
import queue
import threading
from pathlib import Path

import numpy as np
import torch

IGNORE_INDEX = -100


def synthetic_stream(n_tokens: int, seed: int = 1337, vocab_size: int = 50257, eos: int = 50256,
                     mean_doc: float = 900.0, zipf_s: float = 1.1) -> np.ndarray:
    """Seeded Zipf/EOS uint16 stream of exactly n_tokens ids."""
    rng = np.random.default_rng(seed)
    out = np.empty(n_tokens, dtype=np.uint16)
    pos = 0
    while pos < n_tokens:
        length = int(rng.geometric(1.0 / mean_doc))
        parts, have = [], 0
        while have < length:
            draw = rng.zipf(zipf_s, size=length - have) - 1
            kept = draw[draw < eos]
            parts.append(kept)
            have += kept.size
        doc = np.concatenate(parts)[:length] if parts else np.empty(0, dtype=np.int64)
        take = min(length, n_tokens - pos)
        out[pos:pos + take] = doc[:take]
        pos += take
        if pos < n_tokens:
            out[pos] = eos
            pos += 1
    return out


def batch_at(data, cursor: int, batch_size: int, sequence_length: int, target_limit: int):
    """(x, y, count) with the reference trainer's indexing (train_baseline.py:50-63)."""
    count = min(batch_size * sequence_length, target_limit - cursor)
    if count <= 0:
        raise StopIteration
    sequences = math.ceil(count / sequence_length)
    needed = sequences * sequence_length
    raw = np.asarray(data[cursor:cursor + count + 1], dtype=np.int64)
    x = np.zeros(needed, dtype=np.int64)
    y = np.full(needed, IGNORE_INDEX, dtype=np.int64)
    x[:count] = raw[:-1]
    y[:count] = raw[1:]
    return (torch.from_numpy(x.reshape(sequences, sequence_length)),
            torch.from_numpy(y.reshape(sequences, sequence_length)), count)


def rank_cursor(committed: int, microstep: int, rank: int, world: int, batch_size: int,
                sequence_length: int) -> int:
    """Start of (rank, microstep)'s batch inside the update window at `committed`."""
    return committed + (microstep * world + rank) * batch_size * sequence_length


def update_batches(data, committed: int, rank: int, world: int, batch_size: int, sequence_length: int,
                   accumulation: int, target_limit: int):
    """This rank's microstep batches for one update, plus the update's global
    target count (the loss denominator every rank uses, known without
    communication)."""
    capacity = world * accumulation * batch_size * sequence_length
    limit = min(target_limit, committed + capacity)
    batches = []
    for m in range(accumulation):
        cur = rank_cursor(committed, m, rank, world, batch_size, sequence_length)
        if cur >= limit:
            break
        batches.append(batch_at(data, cur, batch_size, sequence_length, limit))
    return batches, limit - committed


# --------------------------------------------------------------------- on disk
def write_stream(path, tokens) -> Path:
    """Writes `tokens` as a flat uint16 file (the prepare_fineweb_edu.py:78
    layout) and returns its path; ids must fit in uint16."""
    arr = np.asarray(tokens)
    if arr.size and (arr.min() < 0 or arr.max() > np.iinfo(np.uint16).max):
        raise ValueError("token ids do not fit uint16")
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_name(path.name + f".tmp{os.getpid()}")
    mm = np.memmap(tmp, dtype=np.uint16, mode="w+", shape=(arr.size,))
    mm[:] = arr.astype(np.uint16, copy=False)
    mm.flush()
    del mm
    os.replace(tmp, path)
    return path


def open_stream(path) -> np.memmap:
    """Read-only uint16 memory map of a token file (train_baseline.py:161-162)."""
    path = Path(path)
    if path.stat().st_size % 2:
        raise ValueError(f"{path} is not a uint16 token file (odd byte count)")
    return np.memmap(path, dtype=np.uint16, mode="r")


# --------------------------------------------------------------- prefetching
class StagedUpdate:
    """One update's batches in page-locked host memory: ids and labels
    [accumulation, B, T] int64 (microsteps past the end of the stream hold
    x = 0, y = -100), the update's global target count and its start."""

    def __init__(self, committed: int, ids: torch.Tensor, labels: torch.Tensor, update_targets: int,
                 slot: int):
        self.committed = committed
        self.ids = ids
        self.labels = labels
        self.update_targets = update_targets
        self.slot = slot
        self.copied = None  # CUDA event after the device copy (set by the consumer)


class UpdatePrefetcher:
    """Iterates this rank's updates over `data` from `start` to `target_limit`,
    each as a StagedUpdate whose pinned buffers a background thread filled
    ahead of time (`depth` updates ahead).

    The buffers form a ring of depth + 1 slots. The consumer copies a slot to
    the device and calls `release(staged, event)` with a CUDA event recorded
    after the copy; the thread refills that slot only once the event has
    completed, so an asynchronous copy never reads a buffer being rewritten.
    Every rank of a data-parallel run builds its own slice of the same update
    windows (update_batches), so no communication is needed.
    """

    def __init__(self, data, rank: int, world: int, batch_size: int, sequence_length: int, accumulation: int,
                 target_limit: int, start: int = 0, depth: int = 2, pin: bool = True):
        if depth < 1:
            raise ValueError("depth must be at least 1")
        self.data = data
        self.rank, self.world = rank, world
        self.B, self.T, self.acc = batch_size, sequence_length, accumulation
        self.limit = target_limit
        self.committed = start
        self.update_size = world * accumulation * batch_size * sequence_length
        shape = (accumulation, batch_size, sequence_length)
        pin = pin and torch.cuda.is_available()
        self._slots = []
        for _ in range(depth + 1):
            ids = torch.zeros(shape, dtype=torch.int64)
            lab = torch.full(shape, IGNORE_INDEX, dtype=torch.int64)
            self._slots.append((ids.pin_memory() if pin else ids, lab.pin_memory() if pin else lab))
        self._free = queue.Queue()
        for i in range(depth + 1):
            self._free.put((i, None))
        self._ready = queue.Queue(maxsize=depth)
        self._stop = threading.Event()
        self._error = None
        self._thread = threading.Thread(target=self._run, name="update-prefetch", daemon=True)
        self._thread.start()

    def _fill(self, slot: int, committed: int):
        ids, lab = self._slots[slot]
        batches, targets = update_batches(self.data, committed, self.rank, self.world, self.B, self.T, self.acc,
                                          self.limit)
        ids.zero_()
        lab.fill_(IGNORE_INDEX)
        for m, (x, y, _) in enumerate(batches):
            ids[m, :x.shape[0]].copy_(x)
            lab[m, :y.shape[0]].copy_(y)
        return StagedUpdate(committed, ids, lab, targets, slot)

    def _run(self):
        committed = self.committed
        try:
            while not self._stop.is_set() and committed < self.limit:
                slot, event = self._free.get()
                if slot is None:
                    break
                if event is not None:
                    event.synchronize()
                self._ready.put(self._fill(slot, committed))
                committed += self.update_size
        except BaseException as exc:  # surfaced to the consumer by __next__
            self._error = exc
        finally:
            self._ready.put(None)

    def __iter__(self):
        return self

    def __next__(self) -> StagedUpdate:
        item = self._ready.get()
        if item is None:
            self._ready.put(None)  # later calls stop too
            if self._error is not None:
                raise RuntimeError("update prefetch failed") from self._error
            raise StopIteration
        self.committed = item.committed + self.update_size
        return item

    def release(self, staged: StagedUpdate, event=None):
        """Returns a slot to the ring; `event` (a torch.cuda.Event recorded
        after the device copy) must complete before the slot is refilled."""
        self._free.put((staged.slot, event))

    def close(self):
        self._stop.set()
        self._free.put((None, None))
        while self._thread.is_alive():
            try:
                self._ready.get(timeout=0.1)
            except queue.Empty:
                pass
        self._thread.join()
