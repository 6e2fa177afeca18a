"""Host side of the row-split batch on CPU: the split plan (pb_batch_split_plan)
covers every row of every projection and of the vocab exactly once, and the
NCCL unique id reaches every rank of a world-size-2 gloo group unchanged."""
import os
import socket

import pytest

from purebee_b200 import _native as N
from purebee_b200.runtime import LlamaConfig
from purebee_b200.thread_pool import NcclComm, split_plan

LLAMA_1B = LlamaConfig(dim=2048, hiddenDim=8192, nLayers=16, nHeads=32, nKvHeads=8, vocabSize=128256, seqLen=1024,
                       headDim=64, ropeTheta=500000.0)
SMOL = LlamaConfig(dim=576, hiddenDim=1536, nLayers=30, nHeads=9, nKvHeads=3, vocabSize=49152, seqLen=512,
                   headDim=64, ropeTheta=10000.0)


@pytest.mark.parametrize("cfg,worlds", [(LLAMA_1B, [1, 2, 4, 8]), (SMOL, [1, 3])])
def test_plan_covers_rows(cfg, worlds):
    hd, kv = cfg.headDim, cfg.nKvHeads * cfg.headDim
    for world in worlds:
        q, k, v, o, g, vocab = set(), set(), set(), set(), set(), set()
        for r in range(world):
            p = split_plan(cfg, world, r)
            assert (p.world, p.rank) == (world, r)
            assert p.n_heads * world == cfg.nHeads and p.n_kv_heads * world == cfg.nKvHeads
            assert p.qkv_rows == (p.n_heads + 2 * p.n_kv_heads) * hd
            q |= set(range(p.q_row0, p.q_row0 + p.n_heads * hd))
            k |= set(range(p.k_row0, p.k_row0 + p.n_kv_heads * hd))
            v |= set(range(p.v_row0, p.v_row0 + p.n_kv_heads * hd))
            o |= set(range(r * p.dim_chunk, (r + 1) * p.dim_chunk))
            g |= set(range(r * p.hidden_chunk, (r + 1) * p.hidden_chunk))
            assert p.vocab_chunk % 32 == 0 or world == 1
            assert p.vocab_row0 == r * p.vocab_chunk and 0 < p.vocab_rows <= p.vocab_chunk
            vocab |= set(range(p.vocab_row0, p.vocab_row0 + p.vocab_rows))
            # the query heads of a rank's kv heads stay with it (GQA groups are whole)
            assert p.q_row0 // hd // (cfg.nHeads // cfg.nKvHeads) == (p.k_row0 - cfg.dim) // hd
        assert q == set(range(cfg.dim)) and k == set(range(cfg.dim, cfg.dim + kv))
        assert v == set(range(cfg.dim + kv, cfg.dim + 2 * kv))
        assert o == set(range(cfg.dim)) and g == set(range(cfg.hiddenDim)) and vocab == set(range(cfg.vocabSize))


def test_plan_rejects():
    for world, rank in [(16, 0), (3, 0), (0, 0), (2, 2), (2, -1)]:
        with pytest.raises(ValueError):
            split_plan(LLAMA_1B, world, rank)
    with pytest.raises(ValueError):  # 3 kv heads do not split 2 ways
        split_plan(SMOL, 2, 0)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, outdir):
    import sys
    from datetime import timedelta
    import torch.distributed as dist
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from purebee_b200.thread_pool import NcclComm
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    try:
        uid = NcclComm.exchange_id()
        with open(os.path.join(outdir, f"id{rank}"), "wb") as f:
            f.write(uid)
    finally:
        dist.destroy_process_group()


def test_comm_id_exchange(tmp_path):
    import torch.multiprocessing as mp
    assert len(NcclComm.new_id()) == N.COMM_ID_BYTES
    mp.spawn(_rank, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    a, b = (open(tmp_path / f"id{r}", "rb").read() for r in range(2))
    assert len(a) == N.COMM_ID_BYTES and a == b
