"""The multi-GPU decompositions, run as two gloo ranks on the CPU with the
oracle standing in for each GPU's kernel:

* config 3: sequences sharded by greedy length balancing, each rank owning
  its own pages, no collective; the union of the ranks' outputs must equal
  the single-process result exactly.
* config 4: KV heads split across ranks (each rank holds only its heads'
  columns of the pages, same block table), per-head outputs all-gathered;
  the gathered output must equal the all-heads result exactly.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from inference_c_b200 import workloads as W


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case(seed=9):
    lengths = np.array([5, 140, 33, 700, 64, 17, 301, 1])
    q_heads, kv_heads, d, bs = 8, 4, 64, 16
    pool_pages = int(((lengths + bs - 1) // bs).sum()) + 4
    tables, _ = W.shuffled_tables(lengths, bs, pool_pages, seed)
    kv = kv_heads * d
    kpool = W.normal_bits(seed, (pool_pages * bs, kv), "f16", stream=1)
    vpool = W.normal_bits(seed, (pool_pages * bs, kv), "f16", stream=2)
    q = W.normal_bits(seed, (len(lengths), q_heads, d), "f16", stream=3)
    return lengths, q_heads, kv_heads, d, bs, tables, kpool, vpool, q


def _worker(rank: int, world: int, port: int, results):
    from oracle import oracle as O
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        lengths, qh, kvh, d, bs, tables, kpool, vpool, q = _case()
        scale = float(1 / np.sqrt(d))
        # config 3: sequence shards, no collective on the data path
        mine = W.shard_by_length(lengths, world)[rank]
        out = O.paged_decode(q[mine], "f16", kpool, vpool, kvh, d, bs, tables[mine],
                             lengths[mine], scale)
        shards = [None] * world
        dist.all_gather_object(shards, (mine.tolist(), out))
        # config 4: this rank's KV heads only (its columns of every page)
        kvl = kvh // world
        cols = slice(rank * kvl * d, (rank + 1) * kvl * d)
        group = qh // kvh
        qcols = slice(rank * kvl * group, (rank + 1) * kvl * group)
        part = O.paged_decode(np.ascontiguousarray(q[:, qcols]), "f16",
                              np.ascontiguousarray(kpool[:, cols]),
                              np.ascontiguousarray(vpool[:, cols]), kvl, d, bs, tables, lengths,
                              scale)
        gathered = [torch.empty(part.shape) for _ in range(world)]
        dist.all_gather(gathered, torch.from_numpy(part))
        if rank == 0:
            results["shards"] = shards
            results["heads"] = torch.cat(gathered, dim=1).numpy()
    finally:
        dist.destroy_process_group()


@pytest.fixture(scope="module")
def two_rank_results(oracle_mod):
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        results = mgr.dict()
        mp.start_processes(_worker, args=(2, _free_port(), results), nprocs=2, join=True,
                           start_method="spawn")
        return dict(results)


def test_sequence_shards_cover_the_batch_once(two_rank_results, oracle_mod):
    lengths, qh, kvh, d, bs, tables, kpool, vpool, q = _case()
    seen = sorted(i for idx, _ in two_rank_results["shards"] for i in idx)
    assert seen == list(range(len(lengths)))
    full = oracle_mod.paged_decode(q, "f16", kpool, vpool, kvh, d, bs, tables, lengths,
                                   float(1 / np.sqrt(d)))
    for idx, out in two_rank_results["shards"]:
        assert np.array_equal(out, full[idx])


def test_head_split_allgather_equals_all_heads(two_rank_results, oracle_mod):
    lengths, qh, kvh, d, bs, tables, kpool, vpool, q = _case()
    full = oracle_mod.paged_decode(q, "f16", kpool, vpool, kvh, d, bs, tables, lengths,
                                   float(1 / np.sqrt(d)))
    assert np.array_equal(two_rank_results["heads"], full)


def test_length_balancing():
    lengths = W.context_lengths(3, 0)
    for world in (1, 2, 4, 8):
        parts = W.shard_by_length(lengths, world)
        assert sorted(np.concatenate(parts).tolist()) == list(range(len(lengths)))
        loads = [int(lengths[p].sum()) for p in parts]
        assert max(loads) - min(loads) <= int(lengths.max())
