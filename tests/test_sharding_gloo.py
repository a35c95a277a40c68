"""Host-side plumbing of the multi-GPU path (image sharding, max-over-ranks
timing, final gather) as world-size-2 gloo ranks on the CPU."""
import os
import socket

import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

from vestra_kernels.sharding import gather_images, image_shard, max_over_ranks  # noqa: E402


@pytest.mark.parametrize("total,world", [(64, 1), (64, 2), (64, 8), (16, 8), (13, 4), (3, 8), (0, 2)])
def test_image_shards_partition_the_batch(total, world):
    covered = []
    for r in range(world):
        first, count = image_shard(total, r, world)
        covered.extend(range(first, first + count))
    assert covered == list(range(total))
    counts = [image_shard(total, r, world)[1] for r in range(world)]
    assert max(counts) - min(counts) <= (1 if total else 0)


def test_image_shard_rejects_bad_rank():
    with pytest.raises(ValueError):
        image_shard(8, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, total, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        first, count = image_shard(total, rank, world)
        # each rank "encodes" its own images: a value that names the image
        local = torch.arange(first, first + count, dtype=torch.float32).view(-1, 1, 1).expand(-1, 3, 2).contiguous()
        slowest = max_over_ranks(10.0 + rank)
        full = gather_images(local, total)
        q.put((rank, slowest, None if full is None else full[:, 0, 0].tolist()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("total", [64, 5])
def test_two_gloo_ranks_shard_time_and_gather(total):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, total, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, slowest, full = q.get(timeout=120)
        results[rank] = (slowest, full)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(s == 10.0 + world - 1 for s, _ in results.values())
    assert results[0][1] == [float(i) for i in range(total)]
    assert results[1][1] is None
