"""Sequence sharding across ranks (host logic; gloo world_size 2 on CPU with
a stand-in decoder, since this container has no GPU)."""
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

import shard


def test_shards_partition_ids():
    for nseq in (0, 1, 7, 64, 65):
        for world in (1, 2, 3, 4, 8):
            ids = [s for r in range(world) for s in shard.shard_of(nseq, r, world)]
            assert ids == list(range(nseq))
            sizes = [len(shard.shard_of(nseq, r, world)) for r in range(world)]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard.shard_of(4, 2, 2)


def test_prompts_depend_only_on_sequence_id():
    a = shard.prompts_for([3, 9], 16, 1000, 5)
    b = shard.prompts_for([9], 16, 1000, 5)
    assert np.array_equal(a[1], b[0]) and a.shape == (2, 16) and a.max() < 1000


class FakeEngine:
    """Deterministic stand-in for the device engine: tokens are a function of
    (prompt, sequence id) only, as the Philox-keyed sampler guarantees."""

    def spec_generate_batch(self, prompts, n_new, k, seq_ids=None):
        out = np.stack([(np.arange(n_new) * 7 + int(p.sum()) + 31 * int(s)) % 1000
                        for p, s in zip(prompts, seq_ids)]).astype(np.int32)
        return out, np.full(len(prompts), n_new // (k + 1) + 1, np.int32), 0.0


def _worker(rank, world, port, nseq, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ids, toks, steps, _ = shard.run_shard(FakeEngine(), shard.shard_of(nseq, rank, world), 12, 10, 4, 1000, 2024)
        full = shard.gather_tokens(dist, ids, toks, nseq)
        if rank == 0:
            q.put(full)
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [1, 2])
def test_gathered_streams_independent_of_world_size(world):
    nseq = 5
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, nseq, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = q.get(timeout=120)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    ids = np.arange(nseq, dtype=np.uint32)
    want, _, _ = FakeEngine().spec_generate_batch(shard.prompts_for(ids, 12, 1000, 2024), 10, 4, ids)
    assert np.array_equal(got, want)
