"""Multi-process host logic of the utterance-sharded decoder stream, on CPU
with the gloo backend (world size 2).  The GPU path adds no collective on
the data path, so what N > 1 changes is host-side: which utterances a rank
owns, the max-over-ranks timing, and a failing rank being noticed by the
others.  Sharding must not change any utterance's result."""
import os
import socket
import warnings

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from bt_b200 import shard


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=60):
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=timeout_s))


def _sharded_worker(rank, world, port, per_rank, t0, result_dir, total=None):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, here)
    from golden import cases as C
    from oracle.ops import OracleRuntime
    from bt_b200.decoder import build_stream
    _init(rank, world, port)
    try:
        # weak scaling: per_rank utterances each; strong: a fixed total split
        if total is None:
            start, count = shard.utterance_range(per_rank, rank)
            total = per_rank * world
        else:
            start, count = shard.split_utterances(total, world, rank)
        ranges = [None] * world
        dist.all_gather_object(ranges, (start, count))
        slowest = shard.max_over_ranks(0.25 + rank)
        assert shard.sum_over_ranks(count) == total
        # this rank's utterances, cut from the job-wide inputs
        full = build_stream(total, t0=t0)
        env_all = C.c5_small_inputs(full, seed=11)
        mine = build_stream(count, t0=t0)
        assert mine.consts.keys() == full.consts.keys()
        env = {k: v for k, v in mine.consts.items()}
        for name in mine.inputs:
            env[name] = env_all[name][start:start + count]
        with warnings.catch_warnings():
            warnings.simplefilter("ignore")
            OracleRuntime().run_nodes(mine.nodes, env)
        outs = [None] * world
        dist.all_gather_object(outs, {n: env[n] for n in mine.stage_outputs()})
        shard.barrier()
        if rank == 0:
            np.savez(os.path.join(result_dir, "sharded.npz"),
                     ranges=np.array(ranges), slowest=np.array(slowest),
                     **{f"r{r}_{i}": o[n] for r, o in enumerate(outs)
                        for i, n in enumerate(mine.stage_outputs())})
    finally:
        dist.destroy_process_group()


def _failing_worker(rank, world, port, result_dir):
    _init(rank, world, port, timeout_s=20)
    if rank == 1:
        raise SystemExit(3)              # leaves between steps, before the collective
    err = "none"
    try:
        shard.barrier()
    except Exception as e:              # noqa: BLE001 - any backend error counts as detection
        err = type(e).__name__
    with open(os.path.join(result_dir, "rank0.txt"), "w") as f:
        f.write(err)


def test_utterance_ranges_are_disjoint_and_cover():
    per, world = 8, 4
    seen = []
    for r in range(world):
        s, n = shard.utterance_range(per, r)
        seen.extend(range(s, s + n))
    assert seen == list(range(per * world))
    for total in (0, 1, 7, 64, 65):
        for world in (1, 2, 3, 8):
            got = []
            for r in range(world):
                s, n = shard.split_utterances(total, world, r)
                got.extend(range(s, s + n))
            assert got == list(range(total))
    with pytest.raises(ValueError):
        shard.split_utterances(4, 2, 2)
    assert shard.rank_seed(100, 3) == 103


def test_single_process_helpers_without_a_group():
    assert shard.world_and_rank() == (1, 0)
    assert shard.max_over_ranks(2.5) == 2.5
    assert shard.sum_over_ranks(2.5) == 2.5
    shard.barrier()


@pytest.mark.timeout(300)
@pytest.mark.parametrize("scaling", ["weak", "strong"])
def test_two_gloo_ranks_shard_utterances_exactly(tmp_path, scaling):
    """Two ranks run their own utterances through the oracle; the gathered
    results equal one process running all of them, bit for bit, and the job
    time is the slower rank's.  weak: two utterances per rank; strong: one
    fixed batch of three split 2 + 1 (the split bench.py --gpus N uses for
    the BASELINE batch of 64)."""
    import sys
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    from golden import cases as C
    from oracle.ops import OracleRuntime
    from bt_b200.decoder import build_stream
    per_rank, world, t0 = 2, 2, 8
    total = None if scaling == "weak" else 3
    mp.start_processes(_sharded_worker, args=(world, _free_port(), per_rank, t0, str(tmp_path), total),
                       nprocs=world, start_method="spawn", join=True)
    got = np.load(os.path.join(tmp_path, "sharded.npz"))
    assert got["ranges"].tolist() == ([[0, 2], [2, 2]] if total is None else [[0, 2], [2, 1]])
    assert float(got["slowest"]) == 1.25
    full = build_stream(per_rank * world if total is None else total, t0=t0)
    env = C.c5_small_inputs(full, seed=11)
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        OracleRuntime().run_nodes(full.nodes, env)
    for i, name in enumerate(full.stage_outputs()):
        joined = np.concatenate([got[f"r{r}_{i}"] for r in range(world)], axis=0)
        want = env[name]
        assert joined.dtype == want.dtype and joined.shape == want.shape
        assert np.array_equal(joined.view(np.uint32), want.view(np.uint32)), name


@pytest.mark.timeout(120)
def test_failed_rank_is_noticed_not_waited_for(tmp_path):
    """A rank that leaves before the collective makes the other rank's
    barrier fail within the group's timeout instead of hanging."""
    import multiprocessing
    ctx = multiprocessing.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=90)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank was still waiting after 90 s"
    assert procs[1].exitcode == 3
    with open(os.path.join(tmp_path, "rank0.txt")) as f:
        assert f.read() != "none"
