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
"""
from __future__ import annotations

import math

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
