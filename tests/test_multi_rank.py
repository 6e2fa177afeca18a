"""The multi-GPU row split's host logic on CPU: world-size-2 gloo ranks on
127.0.0.1, each computing its rows with the oracle (standing in for the
device matvec); a gloo all-gather stands in for the device's NCCL one, and
purebee_b200.thread_pool.assemble_rows cuts the gathered slices to y."""
import os
import socket

import numpy as np
import pytest

from purebee_b200.thread_pool import row_split, rows_per_rank


def test_row_split_properties():
    for n in [1, 7, 8, 9, 100, 2048, 3072, 128256, 49152]:
        for world in [1, 2, 3, 4, 8]:
            parts = row_split(n, world)
            assert len(parts) == world
            assert parts[0][0] == 0 and parts[-1][1] == n
            per = rows_per_rank(n, world)
            for r, (lo, hi) in enumerate(parts):
                assert lo <= hi and (lo % 8 == 0 or lo == hi == n)  # empty trailing ranks sit at n
                if r:
                    assert lo == parts[r - 1][1]
                assert hi - lo <= per
                if hi < n:
                    assert hi - lo == per  # only the last rank may be short
    with pytest.raises(ValueError):
        row_split(0, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank(rank, world, port, n, k, seed, outdir):
    import sys
    import torch
    import torch.distributed as dist
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    sys.path.insert(0, os.path.join(root, "oracle"))
    import oracle as O
    from purebee_b200.thread_pool import assemble_rows, row_split, rows_per_rank
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(seed)
        x = rng.standard_normal(k).astype(np.float32)
        raw = rng.integers(0, 256, n * (k // 32) * 18, dtype=np.uint8)
        raw.reshape(-1, 18)[:, :2] = (rng.standard_normal(n * (k // 32)) * 0.01).astype(np.float16).view(
            np.uint8).reshape(-1, 2)
        lo, hi = row_split(n, world)[rank]
        rb = (k // 32) * 18
        y_local = torch.zeros(rows_per_rank(n, world), dtype=torch.float32)
        if hi > lo:
            y_local[:hi - lo] = torch.from_numpy(O.q4_0_matvec(x, raw[lo * rb:hi * rb], hi - lo, k))
        parts = [torch.zeros_like(y_local) for _ in range(world)]
        dist.all_gather(parts, y_local)
        y = assemble_rows([p.numpy() for p in parts], n)
        np.save(os.path.join(outdir, f"y{rank}.npy"), y)
        if rank == 0:
            np.save(os.path.join(outdir, "full.npy"), O.q4_0_matvec(x, raw, n, k))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n,k", [(100, 64), (1000, 256)])
def test_gathered_rows_equal_one_device(tmp_path, n, k, oracle):
    import torch.multiprocessing as mp
    world = 2
    mp.spawn(_rank, args=(world, _free_port(), n, k, 5, str(tmp_path)), nprocs=world, join=True)
    full = np.load(tmp_path / "full.npy")
    for r in range(world):
        y = np.load(tmp_path / f"y{r}.npy")
        assert np.array_equal(y.view(np.uint32), full.view(np.uint32))
