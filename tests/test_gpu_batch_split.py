"""Row split of the batched configuration over ranks (thread-pool.js:165-246's
row split, one GPU per rank): every rank's tokens and logits have the same
bits as the unsplit batch.

The group form runs all ranks of a split in one process on one GPU, with
device copies in place of the all-gathers (pb_batch_create_group); the NCCL
form runs one process per GPU (pb_batch_create_split) when the box has two."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def make(native, ctx, seed=11, **kw):
    from purebee_b200.runtime import LlamaConfig, StreamingLlamaRuntime
    cfg = dict(dim=512, hiddenDim=1024, nLayers=2, nHeads=8, nKvHeads=4, vocabSize=1000, seqLen=400, headDim=64,
               ropeTheta=10000.0)
    cfg.update(kw)
    rt = StreamingLlamaRuntime(LlamaConfig(**cfg), ctx=ctx, emb_type=native.TYPE_Q4_0)
    rt.loadSynthetic(seed, 0.05)
    return rt


def run_batch(rt, prompts, steps, **kw):
    from purebee_b200.runtime import BatchedLlamaRuntime
    bt = BatchedLlamaRuntime(rt, prompts.shape[0], **kw)
    nxt, lg = bt.prefill(prompts, want_logits=True)
    toks, lgd = bt.decode(steps, want_logits=True)
    bt.free()
    return nxt, lg, toks, lgd


def same_bits(a, b):
    a, b = np.ascontiguousarray(a), np.ascontiguousarray(b)
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


@pytest.mark.parametrize("world,n_seqs,n_prompt,shape", [
    (2, 3, 9, "hd64"), (4, 3, 9, "hd64"), (2, 2, 300, "hd64"), (4, 2, 300, "hd64"), (8, 2, 17, "kv8"),
    (2, 3, 9, "hd32"), (4, 2, 260, "hd32"), (2, 16, 256, "hd64")])
def test_group_split_same_bits(native, ctx, world, n_seqs, n_prompt, shape):
    """27 / 34 prompt rows take the fused-dequant GEMM, 520 / 600 the TMA
    one (chunked f16 operands through a 3-d tensor map); head_dim 64 takes the
    tensor-core prefill attention, 32 the per-query kernel; decode steps split
    K over CTAs with the whole matrix's plan.  4096 rows take the prefill-size
    RMSNorm over chunked and row-major x, and the unsplit batch's attention
    writes the wo operand as hi/lo pairs where the split converts its f32
    rows: the same bits either way."""
    kw = {"hd64": {}, "kv8": dict(nKvHeads=8), "hd32": dict(dim=256, hiddenDim=512, headDim=32, nHeads=8,
                                                               nKvHeads=4)}[shape]
    rt = make(native, ctx, **kw)
    rng = np.random.default_rng(world * 1000 + n_prompt)
    prompts = rng.integers(1, 1000, (n_seqs, n_prompt)).astype(np.int32)
    want = run_batch(rt, prompts, 4)
    got = run_batch(rt, prompts, 4, group=world)
    names = ["prefill tokens", "prefill logits", "decode tokens", "decode logits"]
    for name, g, w in zip(names, got, want):
        if g.dtype == np.float32:
            assert same_bits(g, w), f"{name} differ (max abs {np.max(np.abs(g - w)):.3e})"
        else:
            assert np.array_equal(g, w), f"{name}: {g} != {w}"
    rt.shutdown()


def test_group_split_rejects(native, ctx):
    from purebee_b200.runtime import BatchedLlamaRuntime
    rt = make(native, ctx)
    for world in (3, 8, 16):  # kv heads 4; dim 512 = 64 * 8 but 4 kv heads do not split 8 ways
        with pytest.raises(native.PureBeeError):
            BatchedLlamaRuntime(rt, 2, group=world)
    rt.shutdown()


def test_peer_exchange_wait_is_bounded(native, ctx):
    """The peer exchange kernel's wait gives up: a two-rank exchange on this
    device whose peer never signals raises PB_DEVERR_WAIT after the limit,
    and the context keeps working."""
    import ctypes
    import time
    code = ctypes.c_int()
    t0 = time.perf_counter()
    ctx._check(native.lib().pb_comm_selftest_wait(ctx.h, 200, ctypes.byref(code)))
    dt = time.perf_counter() - t0
    assert code.value == 2, f"expected PB_DEVERR_WAIT, got {code.value}"
    assert 0.15 < dt < 5.0
    rt = make(native, ctx)  # the context still runs work
    rt.shutdown()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, outdir):
    import sys
    from datetime import timedelta
    import torch
    import torch.distributed as dist
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    from purebee_b200 import _native as N
    from purebee_b200.thread_pool import NcclComm
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    ctx = N.Context(rank)
    ctx.set_timeout_ms(60000)
    comm = None
    try:
        rt = make(N, ctx)
        rng = np.random.default_rng(7)
        prompts = rng.integers(1, 1000, (3, 300)).astype(np.int32)
        want = run_batch(rt, prompts, 5)
        for kind in ("p2p", "nccl"):
            if kind == "nccl":
                os.environ["PB_NO_P2P"] = "1"
            comm = NcclComm.from_torch(ctx)
            with open(os.path.join(outdir, f"{kind}{rank}.txt"), "w") as f:
                f.write(str(int(comm.peer_access)))
            got = run_batch(rt, prompts, 5, comm=comm)
            comm.free()
            comm = None
            for i, (g, w) in enumerate(zip(got, want)):
                np.save(os.path.join(outdir, f"{kind}{rank}_{i}.npy"), g)
                np.save(os.path.join(outdir, f"w{rank}_{i}.npy"), w)
        rt.shutdown()
        dist.barrier()
    finally:
        if comm is not None:
            comm.free()
        ctx.close()
        dist.destroy_process_group()


def test_nccl_split_two_gpus(tmp_path):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    mp.spawn(_rank, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        assert open(tmp_path / f"p2p{r}.txt").read() == "1"  # NVLink peers: the peer exchange
        assert open(tmp_path / f"nccl{r}.txt").read() == "0"  # PB_NO_P2P=1: NCCL all-gathers
    for i in range(4):
        w0 = np.load(tmp_path / f"w0_{i}.npy")
        for r in range(2):
            assert np.array_equal(np.load(tmp_path / f"w{r}_{i}.npy"), w0)  # the unsplit batch on each GPU
            for kind in ("p2p", "nccl"):
                got = np.load(tmp_path / f"{kind}{r}_{i}.npy")
                assert got.shape == w0.shape and np.array_equal(got.view(np.uint32), w0.view(np.uint32)), \
                    f"{kind} rank {r} output {i} differs from the unsplit batch"
