"""The N>1 host path on CPU: two gloo ranks shard the sequences, run the
decode loop on their shard (the oracle stands in for the per-GPU engine),
take the max of their timings and gather the ids; the result equals one
process doing every sequence."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from conftest import ROOT, make_model


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, path, prompts, U, out_dir):
    import sys
    sys.path.insert(0, ROOT)
    import datetime

    import torch.distributed as dist

    import oracle as O
    from snai_b200.shard import gather_ids, gather_ids_host, max_over_ranks, shard_range

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    a, b = shard_range(len(prompts), rank, world)
    o = O.Oracle(path, num_heads=2)
    ids, _, secs = o.generate(prompts[a:b], U.shape[1], U[a:b], 1, 0.7, 1.1, 40, 0.9, nthreads=2)
    # rows of ids in sequence order: shard (a, b) of sequences = elements (a*steps, b*steps)
    flat = gather_ids(ids.ravel(), len(prompts) * U.shape[1])
    at0 = gather_ids_host(ids.ravel(), len(prompts) * U.shape[1])
    assert (at0 is None) == (rank != 0)
    m = max_over_ranks(secs if rank == 0 else secs + 1000.0)
    if rank == 0:
        assert np.array_equal(at0.numpy(), flat.numpy())
        np.save(os.path.join(out_dir, "ids.npy"), flat.numpy())
        np.save(os.path.join(out_dir, "max.npy"), np.array([m]))
    dist.barrier()
    dist.destroy_process_group()


def test_shard_range():
    from snai_b200.shard import shard_range
    for total in (0, 1, 7, 4096):
        for world in (1, 2, 3, 8):
            parts = [shard_range(total, r, world) for r in range(world)]
            assert parts[0][0] == 0 and parts[-1][1] == total
            assert all(parts[i][1] == parts[i + 1][0] for i in range(world - 1))
            assert max(b - a for a, b in parts) - min(b - a for a, b in parts) <= 1


def test_two_gloo_ranks_match_one_process(model_dir, tmp_path, built):
    path = make_model(model_dir, "mr.snai", 200, 64, 40, 1, seed=4, std=0.1)
    rng = np.random.default_rng(0)
    prompts = rng.integers(0, 200, (6, 8)).astype(np.int32)  # shards of 3 and 3 sequences
    U = rng.random((6, 5)).astype(np.float32)
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, path, prompts, U, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    import oracle as O
    ref, _, _ = O.Oracle(path, num_heads=2).generate(prompts, 5, U, 1, 0.7, 1.1, 40, 0.9, nthreads=2)
    got = np.load(tmp_path / "ids.npy")
    assert np.array_equal(got, ref.ravel())
    assert np.load(tmp_path / "max.npy")[0] >= 1000.0  # the max came from rank 1
