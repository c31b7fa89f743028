"""CPU: the batch-sharding host logic of the multi-GPU model path, with world-size-2 gloo ranks
(the same code runs over NCCL on GPU ranks in bench.py)."""
import os
import socket

import numpy as np
import pytest

from acfun_b200.shard import shard_bounds


@pytest.mark.parametrize("n,world", [(256, 1), (256, 2), (256, 8), (10, 3), (3, 4), (0, 2)])
def test_shard_bounds_cover_every_image_once(n, world):
    seen = []
    for r in range(world):
        b, e = shard_bounds(n, world, r)
        assert 0 <= b <= e <= n
        seen += list(range(b, e))
    assert seen == list(range(n))
    sizes = [shard_bounds(n, world, r)[1] - shard_bounds(n, world, r)[0] for r in range(world)]
    assert max(sizes) - min(sizes) <= 1


def test_shard_bounds_rejects_bad_rank():
    with pytest.raises(ValueError):
        shard_bounds(8, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, n, q):
    import torch
    import torch.distributed as dist

    from acfun_b200.shard import gather_outputs, shard_bounds
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        b, e = shard_bounds(n, world, rank)
        # the "model": a per-image function of the image index, so order errors show up
        local = torch.arange(b, e, dtype=torch.float32).unsqueeze(1).repeat(1, 5) * 10 + torch.arange(5)
        full = gather_outputs(dist, local, n, world)
        q.put((rank, full.numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n", [256, 7])
def test_gather_outputs_gloo_world2(n):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, n, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want = np.arange(n, dtype=np.float32)[:, None] * 10 + np.arange(5, dtype=np.float32)
    for _, arr in got:
        np.testing.assert_array_equal(arr, want)
