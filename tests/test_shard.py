"""Multi-GPU sharding logic on CPU: ``gloo`` ranks, world size 2 (no GPU).

Each rank decodes its contiguous share of the clips through the facade (a
fake device backend runs the fp32 oracle), and the host-side gather returns
every clip in input order on every rank, equal to a one-process decode.
"""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from fast_audiovae import shard
from fast_audiovae import weights as W


def test_shard_range_partitions_contiguously():
    for n in (0, 1, 5, 64, 4096):
        for world in (1, 2, 3, 8):
            ranges = [shard.shard_range(n, world, r) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
            sizes = [b - a for a, b in ranges]
            assert max(sizes) - min(sizes) <= 1
    assert shard.shard_range(4096, 8, 3) == (1536, 2048)  # 512 streams per GPU
    with pytest.raises(ValueError):
        shard.shard_range(4, 2, 2)


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def rank_main(rank, world, port, clips, out_dir):
    import datetime

    import torch.distributed as dist

    from fast_audiovae import cuda as C
    from tests.test_facade import FakeBackend

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        weights = W.seeded_weights(0)
        decoder = C.CUDADecoder(weights, {"device": "cuda"}, "batch", backend=FakeBackend(weights))
        audio = shard.decode_clips(decoder, clips)
        local = shard.decode_clips(decoder, clips, gather=False)
        longest = shard.max_over_ranks(float(rank + 1))
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), *audio, n_local=len(local), longest=longest)
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_decode_disjoint_shards(tmp_path):
    clips = [W.seeded_latents(300 + i, 1 + i % 3) for i in range(5)]
    world = 2
    mp.start_processes(rank_main, args=(world, free_port(), clips, str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    from fast_audiovae import cuda as C
    from tests.test_facade import FakeBackend
    weights = W.seeded_weights(0)
    one = C.CUDADecoder(weights, {"device": "cuda"}, "batch", backend=FakeBackend(weights))
    single = [one.decode(c) for c in clips]
    for rank in range(world):
        with np.load(tmp_path / f"rank{rank}.npz") as got:
            assert int(got["n_local"]) == (3 if rank == 0 else 2)
            assert float(got["longest"]) == 2.0
            for i, want in enumerate(single):
                assert np.array_equal(got[f"arr_{i}"], want), (rank, i)
