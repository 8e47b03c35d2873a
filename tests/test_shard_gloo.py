"""Token sharding across ranks, on CPU with the gloo backend (two processes).

The host-side logic of the multi-GPU path is tested here without a GPU: the shard
partition, the all-gather of per-rank output shards (padding, trimming, empty
shards, 16-bit outputs) and the max-over-ranks reduction.  The per-shard compute in
these tests is the CPU oracle (the device kernels are covered by the GPU tests);
gathering the shards must reproduce the unsharded oracle run bit for bit, because
rows are independent.
"""
from __future__ import annotations

import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mhcpre_review_b200.shard import gather_outputs, max_over_ranks, shard_range


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("M,world", [(1, 1), (7, 2), (8, 2), (1, 2), (65536, 8), (10, 4), (3, 8)])
def test_shard_range_partitions_rows(M, world):
    ranges = [shard_range(M, world, r) for r in range(world)]
    assert sum(c for _, c in ranges) == M
    pos = 0
    for start, count in ranges:
        assert count >= 0
        if count:
            assert start == pos
        pos += count
    sizes = [c for _, c in ranges]
    assert max(sizes) - min(sizes) <= -(-M // world)
    assert sizes == sorted(sizes, reverse=True)  # ceil-div: only the last shards are smaller


def test_shard_range_rejects_bad_rank():
    with pytest.raises(ValueError):
        shard_range(10, 2, 2)


def _inputs(M, n, D, seed):
    from oracle import ref
    rng = np.random.default_rng(seed)
    K, mix = n * D, n * n + 2 * n
    x = ref.from_float(rng.standard_normal((M, K), dtype=np.float32), "bf16")
    phi = (rng.standard_normal((mix, K)) * 0.02).astype(np.float32)
    gamma = (1 + 0.05 * rng.standard_normal(K)).astype(np.float32)
    alpha = (0.5 + rng.random(3)).astype(np.float32)
    bias = (0.1 * rng.standard_normal(mix)).astype(np.float32)
    return x, phi, alpha, bias, gamma


def _worker(rank, world, port, M, n, D):
    from oracle import ref
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        x, phi, alpha, bias, gamma = _inputs(M, n, D, seed=5)  # replicated weights, same x on all ranks
        start, count = shard_range(M, world, rank)
        if count:
            hin, post, res = ref.mhc_pre_ref(x[start:start + count], phi, alpha, bias, gamma, n, D, "bf16")
        else:
            hin = np.zeros((0, D), np.uint16)
            post = np.zeros((0, n), np.float32)
            res = np.zeros((0, n, n), np.float32)
        local = (torch.from_numpy(hin.view(np.int16)).view(torch.bfloat16), torch.from_numpy(post),
                 torch.from_numpy(res))
        g_in, g_post, g_res = gather_outputs(local, M)
        full_in, full_post, full_res = ref.mhc_pre_ref(x, phi, alpha, bias, gamma, n, D, "bf16")
        assert g_in.dtype == torch.bfloat16 and tuple(g_in.shape) == (M, D)
        assert np.array_equal(g_in.view(torch.int16).numpy().view(np.uint16), full_in)
        assert np.array_equal(g_post.numpy(), full_post)
        assert np.array_equal(g_res.numpy(), full_res)
        # the slowest rank's time
        assert max_over_ranks(float(rank) * 1.5) == 1.5 * (world - 1)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("M", [9, 1])
def test_two_gloo_ranks_gather_reproduces_unsharded_run(M):
    # M = 1: rank 1's shard is empty and still takes part in every collective
    mp.spawn(_worker, args=(2, _free_port(), M, 4, 64), nprocs=2, join=True)
