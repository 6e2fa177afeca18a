"""Row-split matvec across GPUs (thread-pool.js:165-246 with GPUs as the
workers): every rank's gathered y equals the one-device matvec bit for bit.
One process per GPU; the slices are all-gathered by the library's own NCCL
communicator (pb_comm_allgather), torch.distributed only carries its id.
The one-GPU case runs a world-size-1 communicator."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _case(n, k, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal(k).astype(np.float32)
    raw = rng.integers(0, 256, n * (k // 32) * 18, dtype=np.uint8)
    raw.reshape(-1, 18)[:, :2] = (rng.standard_normal(n * (k // 32)) * 0.01).astype(np.float16).view(
        np.uint8).reshape(-1, 2)
    return x, raw


def _rank(rank, world, port, n, k, outdir):
    import sys
    from datetime import timedelta
    import torch
    import torch.distributed as dist
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    from purebee_b200 import _native as N
    from purebee_b200.thread_pool import AtomicsThreadPool, NcclComm, RowSplitMatvec
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    ctx = N.Context(rank)
    ctx.set_matvec_mode(N.MATVEC_EXACT)  # the row split against the reference's bits
    comm = None
    try:
        comm = NcclComm.from_torch(ctx)
        x, raw = _case(n, k, 3)
        rs = RowSplitMatvec(ctx, raw, N.TYPE_Q4_0, n, k, comm)
        xd = ctx.to_device(x)
        y = rs.matvec(xd.ptr).download(np.float32, rs.world * rs.per)[:n]
        np.save(os.path.join(outdir, f"y{rank}.npy"), y)
        rs.free()
        y2 = AtomicsThreadPool(ctx, comm).matvec(x, raw, N.TYPE_Q4_0, n, k)
        np.save(os.path.join(outdir, f"z{rank}.npy"), y2)
        dist.barrier()
    finally:
        if comm is not None:
            comm.free()
        ctx.close()
        dist.destroy_process_group()


def _run(world, n, k, tmp_path, oracle):
    import torch.multiprocessing as mp
    mp.spawn(_rank, args=(world, _free_port(), n, k, str(tmp_path)), nprocs=world, join=True)
    x, raw = _case(n, k, 3)
    want = oracle.q4_0_matvec(x, raw, n, k)
    for r in range(world):
        for tag in "yz":
            got = np.load(tmp_path / f"{tag}{r}.npy")
            assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (tag, r)


def test_row_split_one_gpu(tmp_path, oracle):
    _run(1, 1000, 512, tmp_path, oracle)


def test_row_split_two_gpus(tmp_path, oracle):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    _run(2, 4100, 2048, tmp_path, oracle)
