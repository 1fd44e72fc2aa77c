"""The multi-rank path on CPU: two `gloo` ranks shard C5-shaped segments with `ShardPlan`, check that
every segment runs on exactly one rank with balanced load, gather per-segment outputs back to rank 0
in segment order, and take the max of step timings over the ranks (bench.py's reduction)."""

import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _lengths():
    # C5: 400 segments of U[120,300] frames.
    return np.random.default_rng(5000).integers(120, 301, size=400).tolist()


def _rank(rank, world, port, out_dir):
    import torch.distributed as dist
    from wavo_b200.runner import ShardPlan, encoder_cost, gather_in_order, max_over_ranks, split_rows

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    try:
        lengths = _lengths()
        plan = ShardPlan.for_lengths(lengths, world, lambda t: encoder_cost(t, 1024, 24))
        mine = plan.mine(rank)

        # Every rank derived the same plan on its own.
        plans = [None] * world
        dist.all_gather_object(plans, plan.assign)
        assert all(p == plan.assign for p in plans)
        seen = [None] * world
        dist.all_gather_object(seen, mine)
        flat = sorted(i for s in seen for i in s)
        assert flat == list(range(len(lengths))), "a segment ran on no rank or on two"

        # This rank's "device output": its segments packed one after another in launch order
        # (costliest first, as the varlen launches take them), each row tagged with its segment
        # and row index.
        order = plan.launch_order(rank)
        assert sorted(order) == mine
        costs = [plan.costs[i] for i in order]
        assert costs == sorted(costs, reverse=True)
        packed = np.concatenate([np.stack([np.full(lengths[i], i, np.float32),
                                           np.arange(lengths[i], dtype=np.float32)], 1)
                                 for i in order])
        ordered = gather_in_order(plan, rank, split_rows(packed, [lengths[i] for i in order]),
                                  order=order)
        if rank == 0:
            assert len(ordered) == len(lengths)
            for i, o in enumerate(ordered):
                assert o.shape == (lengths[i], 2)
                assert (o[:, 0] == i).all() and (o[:, 1] == np.arange(lengths[i])).all()
        else:
            assert ordered is None

        # The same outputs through the node-wide shared host buffer: each rank writes its own
        # segments' rows to their places; rank 0 reads them all in segment order.
        from wavo_b200.runner import HostGather
        import torch
        hg = HostGather(plan, lengths, 2, rank, order=order)
        assert hg.available
        hg.copy_from(torch.from_numpy(packed))
        hg.wait()
        if rank == 0:
            for i, t in enumerate(lengths):
                seg = hg.segment(i).numpy()
                assert (seg[:, 0] == i).all() and (seg[:, 1] == np.arange(t)).all(), i
        dist.barrier()
        hg.close()

        # Step timing: the slowest rank sets the time.
        got = max_over_ranks([1.0 + rank, 10.0 - rank])
        assert got == [float(world), 10.0]

        loads = plan.loads()
        with open(os.path.join(out_dir, f"rank{rank}"), "w") as f:
            f.write(f"{len(mine)} {max(loads) / (sum(loads) / world)}\n")
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_shard_and_gather_segments(tmp_path):
    mp.spawn(_rank, args=(WORLD, _free_port(), str(tmp_path)), nprocs=WORLD, join=True)
    counts, imbalance = [], []
    for r in range(WORLD):
        n, imb = open(tmp_path / f"rank{r}").read().split()
        counts.append(int(n))
        imbalance.append(float(imb))
    assert sum(counts) == 400
    assert max(imbalance) < 1.01  # LPT over 400 segments: within 1 % of an even split


def test_plan_single_rank_keeps_everything_in_order():
    from wavo_b200.runner import ShardPlan, gather_in_order
    plan = ShardPlan([5, 3, 9], 1)
    assert plan.mine(0) == [0, 1, 2]
    assert plan.launch_order(0) == [2, 0, 1]
    assert gather_in_order(plan, 0, ["a", "b", "c"]) == ["a", "b", "c"]
    assert gather_in_order(plan, 0, ["c", "a", "b"], order=[2, 0, 1]) == ["a", "b", "c"]
    with pytest.raises(ValueError):
        plan.mine(1)
    with pytest.raises(ValueError):
        gather_in_order(plan, 0, ["a"])
    with pytest.raises(ValueError):
        gather_in_order(plan, 0, ["a", "b", "c"], order=[0, 1, 1])


def test_split_rows_rejects_a_wrong_total():
    from wavo_b200.runner import split_rows
    rows = np.zeros((10, 3))
    assert [p.shape[0] for p in split_rows(rows, [4, 6])] == [4, 6]
    with pytest.raises(ValueError):
        split_rows(rows, [4, 5])
