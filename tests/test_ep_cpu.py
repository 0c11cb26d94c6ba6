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


def _bf16_bits(a: torch.Tensor) -> np.ndarray:
    return a.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)


def _from_bits(b: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(b).view(np.int16)).view(torch.bfloat16).float()


def _expert(e, rows):
    """A stand-in expert: a distinct affine map per expert id, output rounded to bf16."""
    return _bf16_bits(_from_bits(rows) * (1.0 + 0.25 * e) + e)


def _swap(seg: np.ndarray) -> np.ndarray:
    """all_to_all_single of 16-bit segments (as int32 words: gloo's types)."""
    send = torch.from_numpy(np.ascontiguousarray(seg).view(np.int32))
    recv = torch.empty_like(send)
    import torch.distributed as dist
    dist.all_to_all_single(recv, send)
    return recv.numpy().view(np.uint16)


def _worker(rank, world, port, T, H, E, k):
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(10 + rank)
        topk = np.stack([rng.choice(E, k, replace=False) for _ in range(T)])   # distinct experts per token
        x16 = _bf16_bits(torch.from_numpy(rng.normal(0, 1, (T, H)).astype(np.float32)))
        cap = T * k
        recv = _swap(ep_np.pack(topk, x16, E, world, cap))
        el = E // world
        local = ep_np.recv_experts(recv, cap)
        rows = recv.reshape(world * (cap + 1), H)
        back = np.zeros_like(rows)
        for i, e in enumerate(local):
            if e >= 0:
                back[i] = _expert(rank * el + int(e), rows[i])
        got = ep_np.scatter(topk, _swap(back.reshape(world, cap + 1, H)), E, world)
        for t in range(T):
            for s in range(k):
                np.testing.assert_array_equal(got[t, s], _expert(int(topk[t, s]), x16[t]))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("T,E,k", [(16, 16, 4), (5, 8, 8)])
def test_expert_parallel_exchange_gloo(T, E, k):
    import torch.multiprocessing as mp
    mp.spawn(_worker, args=(2, _free_port(), T, 160, E, k), nprocs=2, join=True)


def test_pack_layout():
    topk = np.array([[0, 3], [2, 1]])
    x16 = np.arange(2 * 16, dtype=np.uint16).reshape(2, 16)
    seg = ep_np.pack(topk, x16, experts=4, ranks=2, cap=4)
    words = ep_np.header_words(seg, 4)
    # rank 0 owns experts 0, 1: pairs 0 (e0) and 3 (e1); rank 1 owns 2, 3: pairs 1 (e3) and 2 (e2)
    assert words[0, 0] == 2 and list(words[0, 1:3]) == [(0 << 8) | 0, (3 << 8) | 1]
    assert words[1, 0] == 2 and list(words[1, 1:3]) == [(1 << 8) | 1, (2 << 8) | 0]
    np.testing.assert_array_equal(seg[0, 2], x16[1])    # pair 3 (token 1) is rank 0's second row
    np.testing.assert_array_equal(ep_np.recv_experts(seg, 4).reshape(2, 5)[:, :3], [[-1, 0, 1], [-1, 1, 0]])
    with pytest.raises(ValueError):
        ep_np.pack(np.zeros((4, 1), int), np.zeros((4, 16), np.uint16), experts=4, ranks=2, cap=3)
