"""Expert parallelism on 2 GPUs (NCCL): the sharded MoE layer equals the one-GPU MoE bit
for bit on every rank's tokens.  Needs two GPUs; skipped otherwise."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, cases):
    import torch.distributed as dist
    import __graft_entry__
    __graft_entry__.load_package()
    from qwen35_dflash_b200 import ep, lib, w4
    from oracle import ep_np
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        so = lib.load()
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
            xgen = torch.Generator().manual_seed(7 * rank + t)       # tokens: each rank its own
            x = torch.randn(t, h, generator=xgen).to(torch.bfloat16).cuda()
            logits = torch.randn(t, e + 1, generator=xgen).to(torch.bfloat16).cuda()
            st = lib.stream_ptr()
            nbytes = so.qw_moe_workspace_bytes(t, h, e, inter, k)

            # one GPU holding every expert
            ws1 = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
            out1 = torch.empty(t, h, dtype=torch.bfloat16, device="cuda")
            lib.check(so.qw_moe_route(logits.data_ptr(), lib.QW_BF16, e + 1, t, e, k, e, lib.QW_BF16,
                                      ws1.data_ptr(), st))
            lib.check(so.qw_moe_experts_w4(x.data_ptr(), gu.data_ptr(), dn.data_ptr(), shgu.data_ptr(),
                                           shdn.data_ptr(), t, h, e, inter, k, g, ws1.data_ptr(), st))
            lib.check(so.qw_moe_combine(ws1.data_ptr(), out1.data_ptr(), 0, t, h, e, inter, k, 1, st))

            # experts sharded over the group
            gu_l = ep.local_expert_streams(gu, e, world, rank)
            dn_l = ep.local_expert_streams(dn, e, world, rank)
            for overlap in (False, True):   # the shared expert first, or launched behind the dispatch
                moe = ep.ExpertParallelMoE(dist.group.WORLD, tokens=t, hidden=h, experts=e, inter=inter, top_k=k,
                                           quant_group=g, device="cuda", overlap_shared=overlap)
                ws2 = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
                out2 = torch.empty(t, h, dtype=torch.bfloat16, device="cuda")
                for _ in range(2):   # twice: the exchange buffers are reused
                    lib.check(so.qw_moe_route(logits.data_ptr(), lib.QW_BF16, e + 1, t, e, k, e, lib.QW_BF16,
                                              ws2.data_ptr(), st))
                    moe.experts(x, ws2, gu_l, dn_l, shgu, shdn)
                    lib.check(so.qw_moe_combine(ws2.data_ptr(), out2.data_ptr(), 0, t, h, e, inter, k, 1, st))
                    torch.cuda.synchronize()
                    if not torch.equal(out1, out2):
                        bad = (out1 != out2).sum().item()
                        raise AssertionError(f"rank {rank} case {(t, h, e, k, inter, g)} overlap {overlap}: "
                                             f"{bad} elements differ")
            # the packed segments are the protocol's (oracle/ep_np.py)
            topk = ws2[: t * k * 4].view(torch.int32).view(t, k).cpu().numpy()
            x16 = x.cpu().view(torch.int16).numpy().view("uint16")
            want = ep_np.pack(topk, x16, e, world, t * k)
            got = moe.send_seg.cpu().view(torch.int16).numpy().view("uint16")
            ww, gw = ep_np.header_words(want, t * k), ep_np.header_words(got, t * k)
            for d in range(world):
                n = int(ww[d, 0])
                assert (gw[d, : 1 + n] == ww[d, : 1 + n]).all()
                assert (got[d, 1:1 + n] == want[d, 1:1 + n]).all()
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_expert_parallel_moe_equals_single_gpu():
    import torch.multiprocessing as mp
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    cases = [(16, 2048, 256, 8, 512, 128), (5, 512, 16, 4, 256, 64)]
    mp.spawn(_worker, args=(2, _free_port(), cases), nprocs=2, join=True)
