"""The expert-parallel exchange protocol on CPU: two gloo ranks dispatch their routed pairs
(the blocks each would store into the owners' windows, swapped here with all_to_all),
run their own experts on the rows they received, send the outputs back to the pairs'
sources and scatter them; every (token, slot) must end up with its expert's output of
its token, as one process holding all experts computes it."""
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


def _swap(arr: np.ndarray) -> np.ndarray:
    """all_to_all over the leading (rank) axis of a 16- or 32-bit array (gloo: int32)."""
    import torch.distributed as dist
    raw = np.ascontiguousarray(arr)
    send = torch.from_numpy(raw.view(np.int32).copy())
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send)
    return recv.numpy().view(raw.dtype).reshape(raw.shape)


def _worker(rank, world, port, T, H, E, k, shared):
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(10 + rank)
        topk = np.stack([rng.choice(E, k, replace=False) for _ in range(T)])   # distinct experts per token
        x16 = _bf16_bits(torch.from_numpy(rng.normal(0, 1, (T, H)).astype(np.float32)))
        cap, el = T * (k + shared), E // world
        out_blocks = ep_np.dispatch(topk, x16, E, world, rank, bool(shared))
        # what lands in this rank's window: block s = what source s wrote for this rank
        rows = _swap(np.stack([b[0] for b in out_blocks]))
        meta = _swap(np.stack([b[1] for b in out_blocks]))
        count = _swap(np.array([[b[2]] for b in out_blocks], np.int32))[:, 0]
        blocks = [(rows[s], meta[s], int(count[s])) for s in range(world)]
        # local expert el is the shared expert (stand-in id E)
        outputs = {(s, j): _expert(E if le == el else rank * el + le, rows[s, j])
                   for s, j, le in ep_np.received(blocks)}
        back_to, written = ep_np.combine(blocks, outputs, cap, H)
        back = _swap(back_to)              # [d]: the rows rank d wrote into this rank's back
        mask = _swap(written.astype(np.int32))
        assert (mask.sum(0) == 1).all()    # every pair's output arrives exactly once
        mine = np.zeros((cap, H), np.uint16)
        for d in range(world):
            mine[mask[d] == 1] = back[d][mask[d] == 1]
        got = ep_np.scatter(mine, T, k, bool(shared))
        for t in range(T):
            for s in range(k):
                np.testing.assert_array_equal(got[t, s], _expert(int(topk[t, s]), x16[t]))
            if shared:
                np.testing.assert_array_equal(got[t, k], _expert(E, x16[t]))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("T,E,k,shared", [(16, 16, 4, 1), (5, 8, 8, 0)])
def test_expert_parallel_exchange_gloo(T, E, k, shared):
    import torch.multiprocessing as mp
    mp.spawn(_worker, args=(2, _free_port(), T, 160, E, k, shared), nprocs=2, join=True)


def test_dispatch_layout():
    topk = np.array([[0, 3], [2, 1]])
    x16 = np.arange(2 * 16, dtype=np.uint16).reshape(2, 16)
    blocks = ep_np.dispatch(topk, x16, experts=4, ranks=2)
    # rank 0 owns experts 0, 1: pairs 0 (e0) and 3 (e1); rank 1 owns 2, 3: pairs 1 (e3) and 2 (e2)
    (r0, m0, c0), (r1, m1, c1) = blocks
    assert c0 == 2 and list(m0[:2]) == [(0 << 9) | 0, (3 << 9) | 1]
    assert c1 == 2 and list(m1[:2]) == [(1 << 9) | 1, (2 << 9) | 0]
    np.testing.assert_array_equal(r0[1], x16[1])    # pair 3 (token 1) is rank 0's second row
    assert ep_np.received(blocks) == [(0, 0, 0), (0, 1, 1), (1, 0, 1), (1, 1, 0)]
    # with the shared expert (local expert 2 of rank 1): tokens 0, 1 after rank 1's pairs
    (_, m0, c0), (r1, m1, c1) = ep_np.dispatch(topk, x16, experts=4, ranks=2, rank=1, shared=True)
    assert c0 == 2 and c1 == 4 and list(m1[2:4]) == [(4 << 9) | 2, (5 << 9) | 2]
    np.testing.assert_array_equal(r1[3], x16[1])
