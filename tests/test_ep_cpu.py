"""The expert-parallel exchange on CPU: two gloo ranks pack their routed pairs, swap
segments with all_to_all_single, run their own experts on what they received, swap the
outputs back and scatter them; every (token, slot) must end up with its expert's output
of its token, as one process holding all experts computes it."""
import os
import socket

import numpy as np
import pytest
import torch

from oracle import ep_np


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _expert(e, rows):
    """A stand-in expert: a distinct affine map per expert id."""
    return rows * (1.0 + 0.25 * e) + e


def _worker(rank, world, port, T, H, E, k):
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(10 + rank)
        topk = np.stack([rng.choice(E, k, replace=False) for _ in range(T)])   # distinct experts per token
        x = rng.normal(0, 1, (T, H)).astype(np.float32)
        cap = T * k
        rows, meta = ep_np.pack(topk, x, E, world, cap)
        recv_rows = torch.zeros(world, cap, H)
        recv_meta = torch.zeros(world, cap + 1, dtype=torch.int32)
        dist.all_to_all_single(recv_meta, torch.from_numpy(meta))
        dist.all_to_all_single(recv_rows, torch.from_numpy(rows))
        el = E // world
        local = ep_np.recv_experts(recv_meta.numpy())
        r = recv_rows.numpy().reshape(world * cap, H)
        back = np.zeros_like(r)
        for i, e in enumerate(local):
            if e >= 0:
                back[i] = _expert(rank * el + int(e), r[i])
        recv_back = torch.zeros(world, cap, H)
        dist.all_to_all_single(recv_back, torch.from_numpy(back.reshape(world, cap, H)))
        got = ep_np.scatter(topk, recv_back.numpy(), E, world)
        for t in range(T):
            for s in range(k):
                np.testing.assert_allclose(got[t, s], _expert(int(topk[t, s]), x[t]), rtol=0, atol=0)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("T,E,k", [(16, 16, 4), (5, 8, 8)])
def test_expert_parallel_exchange_gloo(T, E, k):
    import torch.multiprocessing as mp
    mp.spawn(_worker, args=(2, _free_port(), T, 32, E, k), nprocs=2, join=True)


def test_pack_layout():
    topk = np.array([[0, 3], [2, 1]])
    x = np.arange(8, dtype=np.float32).reshape(2, 4)
    rows, meta = ep_np.pack(topk, x, experts=4, ranks=2, cap=4)
    # rank 0 owns experts 0, 1: pairs 0 (e0) and 3 (e1); rank 1 owns 2, 3: pairs 1 (e3) and 2 (e2)
    assert meta[0, 0] == 2 and list(meta[0, 1:3]) == [(0 << 8) | 0, (3 << 8) | 1]
    assert meta[1, 0] == 2 and list(meta[1, 1:3]) == [(1 << 8) | 1, (2 << 8) | 0]
    np.testing.assert_array_equal(rows[0, 1], x[1])
    with pytest.raises(ValueError):
        ep_np.pack(np.zeros((4, 1), int), np.zeros((4, 2), np.float32), experts=4, ranks=2, cap=3)
