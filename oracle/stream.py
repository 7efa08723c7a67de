"""Token stream and batch indexing (oracle side).

batch_at restates scripts/train_baseline.py:50-63 of the reference with plain
Python loops (small inputs only); the synthetic stream restates the benchmark's
stand-in for the FineWeb-Edu uint16 token file: seeded numpy default_rng,
geometric document lengths, Zipf(s) token ids rejection-sampled into
[0, eos), an EOS token after every document, stored as uint16
(scripts/prepare_fineweb_edu.py:78 writes the same dtype).
"""
from __future__ import annotations

import numpy as np
import torch

IGNORE = -100


def batch_at(data, cursor: int, batch_size: int, sequence_length: int, target_limit: int):
    """(x, y, count) exactly as train_baseline.py:50-63: x = data[c:c+n],
    y = data[c+1:c+n+1] with n = min(B*T, limit - cursor); the partial tail
    pads x with 0 and y with -100; raises StopIteration when n <= 0."""
    count = min(batch_size * sequence_length, target_limit - cursor)
    if count <= 0:
        raise StopIteration
    rows = -(-count // sequence_length)
    needed = rows * sequence_length
    x = [0] * needed
    y = [IGNORE] * needed
    for i in range(count):
        x[i] = int(data[cursor + i])
        y[i] = int(data[cursor + i + 1])
    xt = torch.tensor(x, dtype=torch.int64).reshape(rows, sequence_length)
    yt = torch.tensor(y, dtype=torch.int64).reshape(rows, sequence_length)
    return xt, yt, count


def rank_window(committed: int, microstep: int, rank: int, world: int, batch_size: int, sequence_length: int) -> int:
    """Cursor of (rank, microstep) inside one data-parallel update: the update
    consumes the contiguous window starting at `committed`, ordered microstep
    major, rank minor, so concatenating the ranks' batches reproduces one
    global batch_at over the same window."""
    return committed + (microstep * world + rank) * batch_size * sequence_length


def synthetic_stream(n_tokens: int, seed: int = 1337, vocab_size: int = 50257, eos: int = 50256,
                     mean_doc: float = 900.0, zipf_s: float = 1.1) -> np.ndarray:
    """Seeded Zipf/EOS token stream of exactly n_tokens uint16 ids."""
    rng = np.random.default_rng(seed)
    out = np.empty(n_tokens, dtype=np.uint16)
    pos = 0
    while pos < n_tokens:
        length = int(rng.geometric(1.0 / mean_doc))
        doc = []
        while len(doc) < length:
            draw = rng.zipf(zipf_s, size=length - len(doc)) - 1
            doc.extend(int(v) for v in draw[draw < eos])
        take = min(length, n_tokens - pos)
        out[pos:pos + take] = np.asarray(doc[:take], dtype=np.uint16)
        pos += take
        if pos < n_tokens:
            out[pos] = eos
            pos += 1
    return out
