"""The benchmark's job layout, on the CPU: how one batch of 64 utterances is
split over N GPUs (strong scaling) and over concurrent decoder streams on
each GPU, and the config block the JSON line reports for it."""
import types

import bench


def test_rank_batches_split_one_batch_of_64():
    for n, want in ((1, [64]), (2, [32, 32]), (4, [16] * 4), (8, [8] * 8)):
        assert bench.rank_batches(64, n) == want
    assert bench.rank_batches(3, 2) == [2, 1]


def test_stream_groups_two_for_small_rank_batches():
    assert bench.stream_groups(64, 0) == 1
    assert bench.stream_groups(33, 0) == 1
    for b in (32, 16, 8, 2):
        assert bench.stream_groups(b, 0) == 2
    assert bench.stream_groups(1, 0) == 1
    # an explicit count, never more groups than utterances
    assert bench.stream_groups(8, 1) == 1
    assert bench.stream_groups(8, 4) == 4
    assert bench.stream_groups(2, 4) == 2


def test_config_names_the_split_and_the_streams():
    args = types.SimpleNamespace(batch=64, t0=400, streams=0)
    c1 = bench.config(args, 1)
    assert c1["batch_split"] == [64] and c1["streams_per_gpu"] == 1 and c1["launches_per_step"] == 49
    c8 = bench.config(args, 8)
    assert c8["batch_split"] == [8] * 8 and c8["streams_per_gpu"] == 2 and c8["launches_per_step"] == 98
    assert "strong scaling" in c8["parallelism"] and "2 concurrent stream(s)" in c8["parallelism"]
    pinned = bench.config(types.SimpleNamespace(batch=16, t0=400, streams=1), 1)
    assert pinned["streams_per_gpu"] == 1 and pinned["launches_per_step"] == 49
