"""Seeded synthetic inputs for the five sampling workloads.

No public dataset is involved: every input is drawn from numpy's PCG64
generator with a fixed seed, row by row, so the first b rows of a workload
are the same whatever the total batch size (tests use prefixes of the full
workloads).

  single_row   256 rows ~ N(0, 2^2), seed 0; T=1.0, topp=0.9, ONE sampler
               seeded 42 advancing over the 256 rows.
  argmax       B=256 ~ N(0, 1), seed 1, T=0; in 10% of rows the row max is
               copied to 2-4 other random positions (lowest-index tie-break).
  mult         B=1024 ~ N(0, 3^2), seed 2, T=0.8, topp=1.0 (sample_mult),
               per-row state 42 + row.
  topp         B=4096, seed 3: Gumbel(0, 1) noise plus a Zipf(s=1.1) ranked
               bonus A_r * k^-1.1 (k = 1..V over a per-row random
               permutation, A_r ~ U[0, 12] nats), T=0.7, topp 0.9 (even rows)
               / 0.95 (odd rows), per-row state 42 + row.  Row r has its own
               generator, SeedSequence(3, spawn_key=(r,)), so any range of
               global rows (a rank's shard of a multi-GPU batch) is drawn
               without drawing the rows before it.  Nucleus sizes of the first
               4096 rows span 1 to 2683 tokens, mean 156 (tests/golden/topp.json).
  fused        hidden [8192, 4096] bf16 ~ N(0, 1), seed 4; wcls [32000, 4096]
               bf16 ~ N(0, 0.02^2); T=0.8, topp=0.9.
"""
import numpy as np

VOCAB = 32000
DIM = 4096


def single_row(rows=256, vocab=VOCAB):
    rng = np.random.default_rng(0)
    x = rng.normal(0.0, 2.0, size=(rows, vocab)).astype(np.float32)
    return dict(logits=x, temperature=1.0, topp=0.9, seed=42)


def argmax(rows=256, vocab=VOCAB):
    rng = np.random.default_rng(1)
    x = rng.normal(0.0, 1.0, size=(rows, vocab)).astype(np.float32)
    tie = np.random.default_rng(1001)
    for r in range(rows):
        if tie.random() < 0.10:
            k = int(tie.integers(2, 5))
            pos = tie.choice(vocab, size=k, replace=False)
            x[r, pos] = x[r].max()
    return dict(logits=x, temperature=0.0, topp=0.9, seed=42)


def mult(rows=1024, vocab=VOCAB):
    rng = np.random.default_rng(2)
    x = rng.normal(0.0, 3.0, size=(rows, vocab)).astype(np.float32)
    return dict(logits=x, temperature=0.8, topp=1.0, seed=42)


def topp(rows=4096, vocab=VOCAB, first=0):
    """Global rows [first, first + rows) of the top-p workload."""
    x = np.empty((rows, vocab), dtype=np.float32)
    ranks = np.arange(1, vocab + 1, dtype=np.float64) ** -1.1
    for i in range(rows):
        rng = np.random.default_rng(np.random.SeedSequence(3, spawn_key=(first + i,)))
        g = rng.gumbel(0.0, 1.0, size=vocab)
        a = rng.uniform(0.0, 12.0)
        perm = rng.permutation(vocab)
        bonus = np.empty(vocab, dtype=np.float64)
        bonus[perm] = a * ranks
        x[i] = (g + bonus).astype(np.float32)
    topp_rows = np.where((first + np.arange(rows)) % 2 == 0, 0.9, 0.95).astype(np.float32)
    return dict(logits=x, temperature=0.7, topp=0.9, topp_rows=topp_rows, seed=42)


def debug_rows(rows=64, vocab=VOCAB):
    """Rows for the sample_debug / do_sample rules: N(0, 2^2) from seed 5,
    with NaN planted in every seventh row (one position; all positions in
    row 21)."""
    rng = np.random.default_rng(5)
    x = rng.normal(0.0, 2.0, size=(rows, vocab)).astype(np.float32)
    for r in range(0, rows, 7):
        x[r, int(rng.integers(vocab))] = np.nan
    if rows > 21:
        x[21, :] = np.nan
    return dict(logits=x, temperatures=[0.8, 5e-7, 1e-6, 0.0, -0.5], topps=[0.9, 1.0], seed=42)


def fused(rows=8192, dim=DIM, vocab=VOCAB):
    """bf16 operands as uint16 bit patterns (round-to-nearest-even of fp32)."""
    rng = np.random.default_rng(4)
    h = rng.normal(0.0, 1.0, size=(rows, dim)).astype(np.float32)
    w = rng.normal(0.0, 0.02, size=(vocab, dim)).astype(np.float32)
    return dict(hidden=to_bf16_bits(h), wcls=to_bf16_bits(w), temperature=0.8, topp=0.9, seed=42)


def to_bf16_bits(a):
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    r = ((u >> 16) & 1) + 0x7FFF
    return ((u + r) >> 16).astype(np.uint16)


def row_seeds(rows, seed=42, offset=0):
    return (np.uint64(seed) + np.arange(offset, offset + rows, dtype=np.uint64)).astype(np.uint64)


WORKLOADS = dict(single_row=single_row, argmax=argmax, mult=mult, topp=topp)
