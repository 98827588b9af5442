"""The N>1 bench path on CPU: two gloo ranks reduce their timings with MAX
(the slowest rank sets the time); the strong-scaling line splits one batch
into contiguous per-rank ranges balanced by tokens, and the weak figure
counts every rank's whole batch (no data-path collective)."""
import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    import datetime
    import bench

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        dev_ms, wall = bench.reduce_max([100.0 + 50 * rank, 300.0 - rank], dist, "cpu")
        a, b = bench.shard([512] * 64, world, rank)
        q.put((rank, dev_ms, wall, bench.throughput(64, world, 10, dev_ms), (a, b)))
    finally:
        dist.destroy_process_group()


def test_two_rank_max_reduction_and_weak_throughput():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    got = sorted(q.get(timeout=10) for _ in range(2))
    for rank, dev_ms, wall, tput, _ in got:
        assert dev_ms == 150.0 and wall == 300.0  # max over ranks on every rank
        assert tput == pytest.approx(64 * 2 * 10 / 0.150)
    assert [g[4] for g in got] == [(0, 32), (32, 64)]  # one 64-request batch, split


def test_single_process_reduction_is_identity():
    import bench

    assert bench.reduce_max([1.5, 2.5], None, "cpu") == [1.5, 2.5]
    assert bench.throughput(64, 1, 10, 1000.0) == pytest.approx(640.0)


@pytest.mark.parametrize("world", [1, 2, 4, 8, 3])
def test_shard_ranges_cover_the_batch_in_order(world):
    import bench

    lengths = [512] * 64
    ranges = [bench.shard(lengths, world, r) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == 64
    assert all(ranges[i][1] == ranges[i + 1][0] for i in range(world - 1))
    if 64 % world == 0:
        assert all(b - a == 64 // world for a, b in ranges)
    # ragged lengths: balanced by tokens, not by count
    ragged = [1000] + [100] * 10
    assert bench.shard(ragged, 2, 0) == (0, 1) and bench.shard(ragged, 2, 1) == (1, 11)


def test_cfg0q8_workload_is_cfg0s_request_on_the_q8_decoder():
    # the auxiliary line that times the Q8_0-block GEMMs runs cfg0's request
    # (one 256-token check over 2 candidates) on the cfg1 Q8_0 decoder
    import bench
    from laya_goish_b200 import synth

    cname, requests, tokens, qdesc, _ = bench.AUX["cfg0q8"]
    assert (cname, requests, tokens) == ("cfg1", 1, 256)
    assert bench.AUX["cfg0"][1:4] == (requests, tokens, qdesc)
    assert synth.CONFIGS[cname].quant == "q8_0"
    a, na = bench.aux_questions("cfg0q8", 32000)
    b, nb = bench.aux_questions("cfg0", 32000)
    assert na == nb == 0
    assert [[x.tolist() for x in q.arrays()[1:]] for q in a] == [[x.tolist() for x in q.arrays()[1:]] for q in b]
