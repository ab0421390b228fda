"""Multi-rank environment sharding on CPU: two gloo ranks each advance their
slice of the environments (CPU oracle as the physics) and the concatenated
result equals one process advancing all environments, bit for bit; the timing
reduction returns the slowest rank.  No GPU is involved."""

import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from duck_gym_b200.sharding import max_over_ranks, rank_seed, shard, weak_shard


def test_shard_slices_cover_all_envs():
    for total, world in [(10, 3), (4096, 8), (7, 7)]:
        slices = [shard(total, r, world) for r in range(world)]
        assert slices[0].first == 0 and slices[-1].stop == total
        assert all(a.stop == b.first for a, b in zip(slices, slices[1:]))
        assert max(s.count for s in slices) - min(s.count for s in slices) <= 1
    assert weak_shard(4096, 3, 8).first == 3 * 4096
    assert len({rank_seed(0, r) for r in range(8)}) == 8
    with pytest.raises(ValueError):
        shard(2, 2, 2)


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, model, home, targets, out_dir):
    import time

    import torch.distributed as dist

    from oracle.oracle import OracleBatch

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        s = shard(targets.shape[1], rank, world)
        batch = OracleBatch(model, s.count, 0.005, 10)
        forces = np.zeros((s.count, 3), np.float32)
        start = time.perf_counter()
        for step in range(targets.shape[0]):
            batch.step(targets[step, s.first:s.stop], forces, 4, 20.0, 2.0)
        elapsed = time.perf_counter() - start + 0.05 * rank   # rank 1 is "slower"
        slowest = max_over_ranks(elapsed)
        np.save(os.path.join(out_dir, f"bodies{rank}.npy"), batch.state()[0])
        np.save(os.path.join(out_dir, f"slowest{rank}.npy"), np.array([elapsed, slowest]))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_match_single_process(tmp_path, biped_model, biped_meta):
    from oracle.oracle import OracleBatch

    envs, steps, world = 6, 8, 2
    rng = np.random.default_rng(5)
    home = np.asarray(biped_meta["home"], np.float32)
    targets = (home + rng.normal(0, 0.05, (steps, envs, home.size))).astype(np.float32)
    mp.start_processes(_rank_main, args=(world, free_port(), str(biped_model), home, targets, str(tmp_path)),
                       nprocs=world, start_method="spawn", join=True)
    single = OracleBatch(biped_model, envs, 0.005, 10)
    for step in range(steps):
        single.step(targets[step], np.zeros((envs, 3), np.float32), 4, 20.0, 2.0)
    combined = np.concatenate([np.load(tmp_path / f"bodies{r}.npy") for r in range(world)])
    np.testing.assert_array_equal(combined, single.state()[0])
    times = [np.load(tmp_path / f"slowest{r}.npy") for r in range(world)]
    assert times[0][1] == times[1][1] == max(t[0] for t in times)
