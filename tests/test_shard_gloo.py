"""Multi-process (gloo, world size 2, CPU) test of the batch-sharded path: every rank computes its
own slice of the batch with no exchange on the data path; gathering the slices afterwards must
reproduce the full-batch result, and the max-over-ranks timing reduction must agree across
ranks. The per-rank compute here is the CPU oracle (this runs without a GPU)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from dcnv2_b200.shard import shard_batch, shard_range


def test_shard_range_partitions():
    for n in (0, 1, 5, 64, 65, 127, 128):
        for w in (1, 2, 3, 4, 8):
            ranges = [shard_range(n, w, r) for r in range(w)]
            assert ranges[0][0] == 0 and ranges[-1][1] == n
            for (a0, b0), (a1, b1) in zip(ranges, ranges[1:]):
                assert b0 == a1
            sizes = [b - a for a, b in ranges]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, tmpdir):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "oracle"))
    sys.path.insert(0, os.path.join(root, "tensorrt-dcnv2-plugin_b200"))
    import oracle
    from dcnv2_b200.shard import shard_batch
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(5)
        n, c, o, h, w = 5, 8, 6, 9, 7
        x = torch.randn(n, c, h, w, generator=g)
        off = torch.randn(n, 18, h, w, generator=g)
        msk = torch.sigmoid(torch.randn(n, 9, h, w, generator=g))
        wt = torch.randn(o, c, 3, 3, generator=g) * 0.1
        b = torch.randn(o, generator=g) * 0.1
        (xs, offs, ms), (a, bnd) = shard_batch([x, off, msk], world, rank)
        y_local = oracle.forward_ref(xs.numpy(), offs.numpy(), ms.numpy(), wt.numpy(), b.numpy(),
                                     threads=1) if bnd > a else np.zeros((0, o, h, w), np.float32)
        # reassemble (a test-side gather; the sharded path itself exchanges nothing)
        sizes = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(sizes, torch.tensor([bnd - a], dtype=torch.int64))
        maxn = int(max(s.item() for s in sizes))
        pad = torch.zeros(maxn, o, h, w)
        pad[: bnd - a] = torch.from_numpy(y_local)
        parts = [torch.zeros(maxn, o, h, w) for _ in range(world)]
        dist.all_gather(parts, pad)
        y_all = torch.cat([p[: int(s.item())] for p, s in zip(parts, sizes)])
        y_full = oracle.forward_ref(x.numpy(), off.numpy(), msk.numpy(), wt.numpy(), b.numpy(),
                                    threads=1)
        ok = np.array_equal(y_all.numpy(), y_full)
        # max-over-ranks timing reduction (what bench.py does with its per-rank step times)
        t = torch.tensor([1.0 + rank], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ok = ok and float(t.item()) == float(world)
        with open(os.path.join(tmpdir, f"rank{rank}.txt"), "w") as f:
            f.write("ok" if ok else "mismatch")
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_batch_shard(tmp_path):
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    for r in range(world):
        assert (tmp_path / f"rank{r}.txt").read_text() == "ok"
