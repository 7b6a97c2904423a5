"""Independent sequences split across ranks (one process per GPU).

The batched stochastic workload decodes many independent sequences. They
shard with no exchange on the data path: every rank holds a full weight
replica, takes a contiguous share of the sequence ids and decodes them with
its own engine. Each sequence draws from a Philox stream keyed by its global
id, so its tokens do not depend on the number of ranks or on which other
sequences share its rank. The only cross-rank traffic is the optional gather
of finished tokens for reporting.
"""
from __future__ import annotations

import numpy as np


def shard_of(nseq: int, rank: int, world: int) -> range:
    """Contiguous share of sequence ids [0, nseq) for `rank` of `world`;
    shares differ in size by at most one and cover every id once."""
    if world < 1 or not 0 <= rank < world or nseq < 0:
        raise ValueError(f"bad shard request: nseq={nseq} rank={rank} world={world}")
    return range(rank * nseq // world, (rank + 1) * nseq // world)


def prompts_for(ids, prompt_len: int, vocab: int, seed: int) -> np.ndarray:
    """Seeded uniform prompt ids per sequence: row i depends only on (seed, ids[i])."""
    return np.stack([np.random.default_rng([seed, int(s)]).integers(0, vocab, prompt_len) for s in ids]).astype(
        np.int32) if len(ids) else np.zeros((0, prompt_len), np.int32)


def run_shard(engine, ids, prompt_len: int, n_new: int, k: int, vocab: int, prompt_seed: int):
    """Decodes this rank's sequences; returns (ids, tokens [n, n_new], steps
    [n], device seconds)."""
    ids = np.asarray(list(ids), np.uint32)
    if ids.size == 0:
        return ids, np.zeros((0, n_new), np.int32), np.zeros(0, np.int32), 0.0
    prompts = prompts_for(ids, prompt_len, vocab, prompt_seed)
    toks, steps, secs = engine.spec_generate_batch(prompts, n_new, k, seq_ids=ids)
    return ids, toks, steps, secs


def gather_tokens(dist, ids, toks, nseq: int) -> np.ndarray | None:
    """Rank 0 receives every rank's tokens in sequence-id order (reporting
    only; None on the other ranks)."""
    parts = [None] * dist.get_world_size()
    dist.all_gather_object(parts, (np.asarray(ids).tolist(), np.asarray(toks).tolist()))
    if dist.get_rank() != 0:
        return None
    width = max((len(t[0]) for _, tk in parts for t in [tk] if len(tk)), default=0)
    out = np.zeros((nseq, width), np.int32)
    seen = np.zeros(nseq, bool)
    for pid, ptok in parts:
        for s, row in zip(pid, ptok):
            if seen[s]:
                raise RuntimeError(f"sequence {s} decoded twice")
            out[s] = row
            seen[s] = True
    if not seen.all():
        raise RuntimeError(f"sequences missing: {np.nonzero(~seen)[0].tolist()}")
    return out
