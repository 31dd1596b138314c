"""Multi-rank ragged sharding on CPU (gloo, world size 2): every rank computes
the same LPT partition, runs its graphs (the oracle stands in for the GPU
compute here) and one all_gather returns all per-graph results in order."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from rapidalign_b200.shard import graph_costs, lpt_partition


def test_lpt_partition_covers_and_balances():
    rng = np.random.default_rng(0)
    n = rng.integers(32, 2049, 4096)
    m = n + rng.integers(-64, 65, 4096)
    cost = graph_costs(n, m)
    for world in (1, 2, 3, 8):
        parts = lpt_partition(cost, world)
        allidx = np.sort(np.concatenate(parts))
        assert np.array_equal(allidx, np.arange(4096))
        loads = np.array([cost[p].sum() for p in parts])
        # LPT bound: max load <= mean + largest job
        assert loads.max() <= loads.mean() + cost.max() + 1e-9
        assert loads.max() / loads.mean() < 1.002
    # deterministic
    assert all(np.array_equal(a, b) for a, b in zip(lpt_partition(cost, 4),
                                                    lpt_partition(cost, 4)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, sizes, out_dir):
    import torch.distributed as dist
    from oracle import oracle as O
    from rapidalign_b200.shard import sharded_pair_results
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    sizes = np.asarray(sizes)

    def graph(g):
        rng = np.random.default_rng([7, int(g)])
        n, m = sizes[g]
        x = rng.standard_normal((n, 3))
        y = rng.standard_normal((m, 3))
        return x, y

    def compute(ids):
        rows = []
        for g in ids:
            x, y = graph(g)
            r = O.kde_mmd_loss(x, y, sigma=0.3)
            rows.append([r.loss, r.Kxx, r.Kyy, r.Kxy])
        return torch.tensor(np.array(rows, dtype=np.float64).reshape(-1, 4))

    cost = graph_costs(sizes[:, 0], sizes[:, 1])
    res = sharded_pair_results(len(sizes), cost, compute)
    np.save(os.path.join(out_dir, f"rank{rank}.npy"), res.numpy())
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_gather_matches_single_process(tmp_path):
    from oracle import oracle as O
    rng = np.random.default_rng(1)
    sizes = np.stack([rng.integers(1, 60, 13), rng.integers(1, 60, 13)], axis=1)
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), sizes.tolist(), str(tmp_path)),
                       nprocs=world, join=True, start_method="spawn")
    full = []
    for g in range(len(sizes)):
        r = np.random.default_rng([7, g])
        x = r.standard_normal((sizes[g][0], 3))
        y = r.standard_normal((sizes[g][1], 3))
        o = O.kde_mmd_loss(x, y, sigma=0.3)
        full.append([o.loss, o.Kxx, o.Kyy, o.Kxy])
    full = np.array(full)
    for rank in range(world):
        got = np.load(tmp_path / f"rank{rank}.npy")
        np.testing.assert_allclose(got, full, rtol=0, atol=0)


def _packed_worker(rank, world, port, out_dir):
    import datetime
    import torch.distributed as dist
    from rapidalign_b200.shard import _sharded, packed_all_reduce
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    # one collective over a float64 and a float32 buffer
    f64 = torch.arange(5, dtype=torch.float64) * (rank + 1) + 0.25
    f32 = torch.full((7,), 0.5 * (rank + 1), dtype=torch.float32)
    packed_all_reduce(f64, f32)
    # sharded per-graph results: values of every graph on every rank,
    # gradients only into this rank's graphs
    w = torch.ones(6, dtype=torch.float64, requires_grad=True)

    def compute(ids):
        ids_t = torch.as_tensor(ids, dtype=torch.long)
        v = w.index_select(0, ids_t) * (ids_t.to(torch.float64) + 1.0)
        return v, 2 * v, 3 * v, 4 * v

    costs = [5.0, 1.0, 4.0, 2.0, 3.0, 6.0]
    outs = _sharded(6, costs, compute, None)
    outs[0].sum().backward()
    np.savez(os.path.join(out_dir, f"packed{rank}.npz"), f64=f64.numpy(), f32=f32.numpy(),
             outs=torch.stack([o.detach() for o in outs]).numpy(), grad=w.grad.numpy())
    dist.barrier()
    dist.destroy_process_group()


def test_packed_all_reduce_and_sharded_results(tmp_path):
    world = 2
    mp.start_processes(_packed_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    costs = [5.0, 1.0, 4.0, 2.0, 3.0, 6.0]
    parts = lpt_partition(costs, world)
    for rank in range(world):
        z = np.load(tmp_path / f"packed{rank}.npz")
        np.testing.assert_array_equal(z["f64"], np.arange(5) * 3.0 + 0.5)
        np.testing.assert_array_equal(z["f32"], np.full(7, 1.5, dtype=np.float32))
        g = np.arange(6) + 1.0
        np.testing.assert_array_equal(z["outs"], np.stack([g, 2 * g, 3 * g, 4 * g]))
        grad = np.zeros(6)
        grad[parts[rank]] = g[parts[rank]]
        np.testing.assert_array_equal(z["grad"], grad)
