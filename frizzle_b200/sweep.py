"""a steering sweep of steered sequences and their unsteered twins.

Each pair shares one prompt and one sampling seed; the steered sequence pins k neurons of one layer's
GeGLU activation (the in-kernel edit of Frizzle's steering hook, edit/edit.h:50-60) from the first
generated token on, k uniform in {1..8}, neurons uniform in [0, ffn), values uniform in [-10, 10]
(SET edits).  Pairs are independent, so they are sharded across ranks (one process per GPU) in
contiguous blocks with no collective on the data path; the drawn tokens are gathered to rank 0 at the
end.  The gather works on any torch.distributed backend (gloo on CPU, NCCL on GPUs).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import edits as E


@dataclass
class Pair:
    index: int
    neurons: np.ndarray     # uint32 [k]
    values: np.ndarray      # float32 [k]
    seed: tuple             # (seed0, seed1) shared by the twins

    def edits(self, layer: int) -> list:
        return [E.Edit(layer, int(n), E.SET, float(v), 0) for n, v in zip(self.neurons, self.values)]


def make_pairs(n_pairs: int = 64, ffn: int = 6912, seed: int = 0) -> list:
    """The sweep's pairs, from one seeded generator (the same on every rank)."""
    rng = np.random.default_rng([seed, 4])
    pairs = []
    for i in range(n_pairs):
        k = int(rng.integers(1, 9))
        neurons = np.sort(rng.choice(ffn, size=k, replace=False)).astype(np.uint32)
        values = rng.uniform(-10.0, 10.0, size=k).astype(np.float32)
        s = rng.integers(0, 2**32, size=2, dtype=np.uint64)
        pairs.append(Pair(i, neurons, values, (int(s[0]), int(s[1]))))
    return pairs


def shard(n: int, world: int, rank: int) -> range:
    """Rank `rank`'s contiguous block of n items (the first n % world ranks take one more)."""
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def sequences(pairs: list) -> list:
    """Flattened sequence list: pair i gives (i, steered=True) then (i, steered=False)."""
    out = []
    for p in pairs:
        out.append((p, True))
        out.append((p, False))
    return out


def run(model, prompt, pairs: list, steps: int, layer: int, batch_seqs: int = 8, context: int = 1024,
        top_k: int = 64, temperature: float = 1.0, batches: dict = None) -> dict:
    """Generates `steps` tokens for every sequence of `pairs` on this rank's GPU.

    `batches` ({group size: engine.Batch}) keeps the batches, with their
    captured step graphs, for the caller to reuse and free; by default they
    are made here and freed at the end.
    Returns {pair index: int32 [2][steps]} (row 0 steered, row 1 unsteered)."""
    from . import engine
    seqs = sequences(pairs)
    out = {p.index: np.zeros((2, steps), dtype=np.int32) for p in pairs}
    n = len(prompt)
    sampling = engine.Sampling(temperature=temperature, top_k=top_k, top_p=1.0, min_p=0.0)
    # One batch serves every group of the same size (a new group's prefill rewrites its caches from
    # position 0, and the step graphs captured for the first group are reused).
    own = batches is None
    if own:
        batches = {}
    try:
        for b0 in range(0, len(seqs), batch_seqs):
            group = seqs[b0:b0 + batch_seqs]
            S = len(group)
            if S not in batches:
                batches[S] = engine.Batch(model, S, context)
            batch = batches[S]
            seeds = np.array([p.seed for p, _ in group], dtype=np.uint32)
            for s, (p, steered) in enumerate(group):
                words = E.table(p.edits(layer), model.info.layers, n - 1) if steered else None
                batch.set_edits(s, words)
            # The shared prompt in one step (more than 16 rows: the tensor-core path).
            ids = np.tile(np.asarray(prompt, dtype=np.uint32), (S, 1))
            batch.step(0, ids, tokens=n, logits=True, sampling=sampling, seeds=seeds)
            for i in range(steps):
                toks = batch.tokens()
                for s, (p, steered) in enumerate(group):
                    out[p.index][0 if steered else 1, i] = toks[s]
                if i + 1 < steps:
                    batch.step(n + i, fed=True, tokens=1, logits=True, sampling=sampling, seeds=seeds)
    finally:
        if own:
            for b in batches.values():
                b.free()
    return out


def gather(results: dict, n_pairs: int, steps: int, dist, device=None):
    """Every rank's {pair: tokens}; returns the full [n_pairs][2][steps] array on rank 0 (None elsewhere).

    A padded all-gather of one int64 tensor per rank: [count, then count x (index, 2 x steps tokens)]."""
    import torch
    world, rank = dist.get_world_size(), dist.get_rank()
    width = 1 + 2 * steps
    local = np.zeros((len(results), width), dtype=np.int64)
    for row, (idx, toks) in enumerate(sorted(results.items())):
        local[row, 0] = idx
        local[row, 1:] = toks.reshape(-1)
    cap = max(len(shard(n_pairs, world, r)) for r in range(world))
    buf = np.zeros((1 + cap * width,), dtype=np.int64)
    buf[0] = len(results)
    buf[1:1 + local.size] = local.reshape(-1)
    t = torch.from_numpy(buf)
    if device is not None:
        t = t.to(device)
    parts = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(parts, t)
    if rank != 0:
        return None
    full = np.full((n_pairs, 2, steps), -1, dtype=np.int32)
    for p in parts:
        a = p.cpu().numpy()
        count = int(a[0])
        rows = a[1:1 + count * width].reshape(count, width)
        for r in rows:
            full[int(r[0])] = r[1:].reshape(2, steps)
    return full
