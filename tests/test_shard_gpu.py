"""Token sharding on several GPUs (one process per GPU, NCCL): each rank runs the
CUDA operator on its contiguous rows, the shards are all-gathered, and the result
must equal the one-GPU run of the whole batch bit for bit (from 8192 rows per
shard the split-K plan depends on K only).  Skipped with fewer than two GPUs."""
from __future__ import annotations

import os
import socket
from datetime import timedelta

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_path):
    import torch.distributed as dist
    import mhcpre_review_b200 as mp
    from mhcpre_review_b200.configs import CONFIGS, make_inputs, with_shape
    from mhcpre_review_b200.shard import gather_outputs, shard_range
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        cfg = with_shape(CONFIGS["c4"], batch=2 * world)  # 8192 rows per shard
        inp = make_inputs(cfg)
        M, n, D = cfg.M, cfg.n, cfg.D
        start, rows = shard_range(M, world, rank)
        xs = inp["x"].reshape(M, n, D)[start:start + rows].reshape(1, rows, n, D).contiguous()
        ex = mp.MhcPre(1, rows, n, D, xs.dtype, cfg.gamma)
        ex.prepare(inp["phi"], inp["gamma"])
        hin, post, res = ex(xs, inp["alpha"], inp["bias"])
        full = gather_outputs((hin.reshape(rows, D), post.reshape(rows, n), res.reshape(rows, n, n)), M)
        ok = mp.device_status() == 0
        if rank == 0:
            one = mp.mhc_pre(inp["x"], inp["phi"], inp["alpha"], inp["bias"], inp["gamma"])
            torch.cuda.synchronize()
            ok = ok and torch.equal(full[0].view(torch.int16), one[0].reshape(M, D).view(torch.int16))
            ok = ok and torch.equal(full[1], one[1].reshape(M, n)) and torch.equal(full[2], one[2].reshape(M, n, n))
            with open(result_path, "w") as f:
                f.write("ok" if ok else "mismatch")
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_sharded_run_on_two_gpus_equals_one_gpu_run(tmp_path):
    import torch.multiprocessing as tmp
    out = tmp_path / "result.txt"
    tmp.spawn(_worker, args=(2, _free_port(), str(out)), nprocs=2, join=True)
    assert out.read_text() == "ok"
