"""Expert parallelism on 2 GPUs (kernel stores into the peers' windows over NVLink): the
sharded MoE layer equals the one-GPU MoE bit for bit on every rank's tokens, over
repeated exchanges, and a whole engine with sharded experts (eager and replayed as a
CUDA graph) gives every rank the single-GPU engine's predictions and features.  Needs
two GPUs; skipped otherwise."""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _moe_cases(rank, world, so, cases):
    from qwen35_dflash_b200 import ep, lib, w4
    import torch.distributed as dist
    # the expert-parallel receiver runs the grouped kernels only: compare with the
    # one-GPU kernels without the tensor-core dense path (same bits)
    prev = so.qw_moe_dense_threshold(0)
    for (t, h, e, k, inter, g) in cases:
        gen = torch.Generator().manual_seed(1000 + t + e)       # weights: the same on every rank
        qgu = torch.randint(-8, 8, (e, 2 * inter, h), dtype=torch.int8, generator=gen)
        sgu = (torch.rand(e, 2 * inter, h // g, generator=gen) * 0.015 + 0.005).to(torch.bfloat16)
        qdn = torch.randint(-8, 8, (e, h, inter), dtype=torch.int8, generator=gen)
        sdn = (torch.rand(e, h, inter // g, generator=gen) * 0.015 + 0.005).to(torch.bfloat16)
        qsgu = torch.randint(-8, 8, (2 * inter, h), dtype=torch.int8, generator=gen)
        ssgu = (torch.rand(2 * inter, h // g, generator=gen) * 0.015 + 0.005).to(torch.bfloat16)
        qsdn = torch.randint(-8, 8, (h, inter), dtype=torch.int8, generator=gen)
        ssdn = (torch.rand(h, inter // g, generator=gen) * 0.015 + 0.005).to(torch.bfloat16)
        gu = w4.pack_w4(qgu.cuda(), sgu.cuda(), g)
        dn = w4.pack_w4(qdn.cuda(), sdn.cuda(), g)
        shgu = w4.pack_w4(qsgu.cuda(), ssgu.cuda(), g)
        shdn = w4.pack_w4(qsdn.cuda(), ssdn.cuda(), g)
        moe = ep.ExpertParallelMoE(dist.group.WORLD, tokens=t, hidden=h, experts=e, inter=inter, top_k=k,
                                   quant_group=g, device="cuda")
        gu_l, dn_l = moe.local_banks(gu, dn, shgu, shdn)
        st = lib.stream_ptr()
        nbytes = so.qw_moe_workspace_bytes(t, h, e, inter, k)
        try:
            for rep in range(3):   # repeated exchanges: the epochs advance, the windows are reused
                xgen = torch.Generator().manual_seed(7 * rank + t + 100 * rep)   # tokens: each rank its own
                x = torch.randn(t, h, generator=xgen).to(torch.bfloat16).cuda()
                logits = torch.randn(t, e + 1, generator=xgen).to(torch.bfloat16).cuda()
                if rep == 2:   # skewed routing: every token prefers rank 0's experts
                    logits[:, : e // world] += 4.0
                ws1 = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
                out1 = torch.empty(t, h, dtype=torch.bfloat16, device="cuda")
                lib.check(so.qw_moe_route(logits.data_ptr(), lib.QW_BF16, e + 1, t, e, k, e, lib.QW_BF16,
                                          ws1.data_ptr(), st))
                lib.check(so.qw_moe_experts_w4(x.data_ptr(), gu.data_ptr(), dn.data_ptr(), shgu.data_ptr(),
                                               shdn.data_ptr(), t, h, e, inter, k, g, ws1.data_ptr(), st))
                lib.check(so.qw_moe_combine(ws1.data_ptr(), out1.data_ptr(), 0, t, h, e, inter, k, 1, st))
                ws2 = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
                out2 = torch.empty(t, h, dtype=torch.bfloat16, device="cuda")
                lib.check(so.qw_moe_route(logits.data_ptr(), lib.QW_BF16, e + 1, t, e, k, e, lib.QW_BF16,
                                          ws2.data_ptr(), st))
                moe.experts(x, ws2, gu_l, dn_l)
                lib.check(so.qw_moe_combine(ws2.data_ptr(), out2.data_ptr(), 0, t, h, e, inter, k, 1, st))
                lib.check(so.qw_check_wait_status(1, st), "ep waits")
                if not torch.equal(out1, out2):
                    bad = (out1 != out2).sum().item()
                    raise AssertionError(f"rank {rank} case {(t, h, e, k, inter, g)} rep {rep}: {bad} elements differ")
        finally:
            moe.close()
    so.qw_moe_dense_threshold(prev)


def _engine_case(rank, world):
    """The tiny target with its 16 experts sharded 8 + 8 against the one-GPU engine."""
    import torch.distributed as dist
    from qwen35_dflash_b200 import config, engine as E, synthetic
    cfg = config.TINY
    raw = synthetic.init_weights(cfg, seed=21)
    one = E.TargetEngine(cfg, E.weights_from_arrays(cfg, raw), batch=2, block=16, capacity=128)
    sh = E.TargetEngine(cfg, E.weights_from_arrays(cfg, raw), batch=2, block=16, capacity=128,
                        ep_group=dist.group.WORLD)
    try:
        for e in (one, sh):
            e.set_random_context(30, seed=9 + rank)
        gen = torch.Generator().manual_seed(50 + rank)
        for it in range(2):
            props = torch.randint(0, cfg.vocab_size, (32,), generator=gen, dtype=torch.int32).cuda()
            for e in (one, sh):
                e.tokens.copy_(props)
                e.step()
            torch.cuda.synchronize()
            assert torch.equal(one.top1, sh.top1) and torch.equal(one.features, sh.features), (rank, it)
            assert torch.equal(one.state, sh.state) and torch.equal(one.qpos, sh.qpos), (rank, it)
        sh.capture()
        one.capture()
        for it in range(3):
            props = torch.randint(0, cfg.vocab_size, (32,), generator=gen, dtype=torch.int32).cuda()
            for e in (one, sh):
                e.tokens.copy_(props)
                e.replay()
            torch.cuda.synchronize()
            assert torch.equal(one.top1, sh.top1) and torch.equal(one.features, sh.features), (rank, "graph", it)
        assert int(sh.wait_status.item()) == 0
    finally:
        sh.close()
        one.close()


def _worker(rank, world, port, cases):
    import torch.distributed as dist
    import __graft_entry__
    __graft_entry__.load_package()
    from qwen35_dflash_b200 import lib
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank))
    try:
        so = lib.load()
        _moe_cases(rank, world, so, cases)
        _engine_case(rank, world)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_expert_parallel_moe_equals_single_gpu():
    import torch.multiprocessing as mp
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    cases = [(16, 2048, 256, 8, 512, 128), (5, 512, 16, 4, 256, 64), (128, 2048, 256, 8, 512, 128)]
    mp.spawn(_worker, args=(2, _free_port(), cases), nprocs=2, join=True)
