"""Host side of tensor parallelism, on CPU: the NCCL-id hand-out of bench.py
across ranks (gloo, world size 2) and the engine's argument checks."""
import os
import socket

import numpy as np
import pytest

import torch.multiprocessing as tmp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, tp, out):
    import datetime

    import torch.distributed as dist

    import bench
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    got = bench.tp_group_id(dist, world, tp, rank, lambda: f"id-of-{rank}".encode())
    out[rank] = got
    dist.destroy_process_group()


@pytest.mark.parametrize("tp", [1, 2])
def test_tp_group_id_gloo(tp):
    world = 2
    mgr = tmp.get_context("spawn").Manager()
    out = mgr.dict()
    tmp.start_processes(_rank, args=(world, _free_port(), tp, out), nprocs=world, join=True,
                        start_method="spawn")
    if tp == 2:
        assert out[0] == out[1] == b"id-of-0"
    else:
        assert out[0] == b"id-of-0" and out[1] == b"id-of-1"


@pytest.mark.parametrize("tp,rank", [(3, 0), (2, 2), (4, 0)])
def test_engine_rejects_unsplittable_tp(sb, workdir, tp, rank):
    """kv heads, vocabulary, FFN/256 and heads*hd/256 must divide by tp; the check
    happens before any device work."""
    path = os.path.join(str(workdir), "tp_reject.gguf")
    if not os.path.exists(path):
        # 8 heads / 2 kv heads (tp 4 splits no kv head pair), vocab 1000, ffn 1024
        sb.synth_gguf(path, n_layers=1, d_model=512, ffn_hidden=1024, n_heads=8, n_kv_heads=2,
                      vocab=1000, max_seq=64, q4k=True, seed=3)
    with pytest.raises(RuntimeError, match="tensor parallel"):
        sb.LlamaBatch(path, tp_size=tp, tp_rank=rank, tp_id=b"\0" * 128)
