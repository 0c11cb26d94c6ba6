"""Expert parallelism for the routed MoE (the reference's multi-GPU serving plan: experts
sharded over the GPUs, dispatch and combine by all-to-all, attention and GDN replicated
per request).

Rank g of a process group of G ranks owns experts [g E/G, (g+1) E/G).  For one MoE layer
each rank routes its own tokens over all E experts (``qw_moe_route``), then
``ExpertParallelMoE.experts`` computes, into the same workspace, every routed
(token, slot) pair's expert output and the shared expert's, exactly as
``qw_moe_experts_w4`` would on one GPU holding all experts:

1. the shared expert on the rank's own tokens (``qw_moe_experts_w4_range`` with an
   empty routed range);
2. ``qw_moe_ep_pack``: each pair's activation row into the send segment of the rank
   owning its expert (fixed ``cap`` rows per destination, ``cap = tokens * top_k``, so a
   segment cannot overflow), behind a header row of counts and local expert ids;
3. all-to-all of the segments (optionally with the shared expert of step 1 launched
   behind it, running meanwhile);
4. ``qw_moe_ep_recv_route`` + ``qw_moe_ep_experts``: the received rows through the
   rank's own experts (top-1 routing, one expert per row);
5. ``qw_moe_ep_pack_out`` + all-to-all back + ``qw_moe_ep_scatter``: the outputs into the
   source rank's per-(token, slot) slots.

``qw_moe_combine`` / ``qw_moe_combine_norm`` then run unchanged.  The expert kernels give
a row the same bits whatever else is in their launch and outputs travel as bf16 (the
precision the combine reads), so the result equals the single-GPU MoE bit for bit.

The collectives are ``torch.distributed.all_to_all_single`` with equal splits (NCCL over
NVLink on GPUs, gloo in the CPU tests of the exchange).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import lib

BF16 = torch.bfloat16


def expert_range(experts: int, ranks: int, rank: int) -> tuple[int, int]:
    """(first expert, count) owned by ``rank``."""
    if experts % ranks:
        raise ValueError(f"{experts} experts do not split over {ranks} ranks")
    el = experts // ranks
    return rank * el, el


def local_expert_streams(stream: torch.Tensor, experts: int, ranks: int, rank: int) -> torch.Tensor:
    """The rank's slice of a W4 expert bank (streams of ``experts`` equal-size experts,
    concatenated), as its own contiguous tensor."""
    lo, el = expert_range(experts, ranks, rank)
    per = stream.numel() // experts
    return stream.view(-1)[lo * per:(lo + el) * per].clone()


class ExpertParallelMoE:
    """The routed experts of MoE layers of one shape, sharded over ``group``.

    ``tokens`` is the rank's own token count per call (every rank the same).  With
    ``overlap_shared`` the dispatch all-to-all is issued first (on the collective's own
    stream) and the shared expert is launched behind it on the caller's stream, so the
    two run together: the collective's kernel already holds its SMs when the persistent
    expert kernels fill the rest (the default: 8.36 against 8.62 ms per verify step on two
    B200s).  Otherwise the shared expert runs first."""

    def __init__(self, group, *, tokens: int, hidden: int, experts: int, inter: int, top_k: int,
                 quant_group: int, device, overlap_shared: bool = True):
        self.group = group
        self.G = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.T, self.H, self.E, self.I, self.k, self.qg = tokens, hidden, experts, inter, top_k, quant_group
        self.lo, self.el = expert_range(experts, self.G, self.rank)
        self.cap = tokens * top_k
        self.so = lib.load()
        G, cap, H = self.G, self.cap, hidden
        if (cap + 1) * 4 > H * 2:
            raise ValueError("the segment header (cap + 1 int32 words) must fit in one row")
        # segments [G][cap + 1][H]: row 0 the header, rows 1.. the pairs (qw_moe_ep_pack)
        self.send_seg = torch.zeros(G, cap + 1, H, dtype=BF16, device=device)
        self.recv_seg = torch.zeros(G, cap + 1, H, dtype=BF16, device=device)
        self.send_back = torch.zeros(G, cap + 1, H, dtype=BF16, device=device)
        self.recv_back = torch.zeros(G, cap + 1, H, dtype=BF16, device=device)
        nbytes = self.so.qw_moe_ep_recv_workspace_bytes(G, cap, H, experts, inter)
        self.ws_r = torch.zeros(nbytes, dtype=torch.uint8, device=device)
        self.overlap = overlap_shared

    def header(self, seg: torch.Tensor) -> torch.Tensor:
        """int32 header words [G, cap + 1] of a segment buffer."""
        return seg[:, 0].contiguous().view(torch.int32)[:, : self.cap + 1]

    def experts(self, x: torch.Tensor, ws: torch.Tensor, gate_up_local: torch.Tensor, down_local: torch.Tensor,
                shared_gate_up: torch.Tensor | None, shared_down: torch.Tensor | None, stream=None):
        """Routed + shared expert outputs of this rank's tokens ``x`` [tokens, hidden] (bf16)
        into ``ws`` (a MoE workspace already routed by qw_moe_route / qw_moe_route_x) on the
        current stream.  Every rank of the group calls it, with the same shapes, in the same
        order."""
        so = self.so
        cur = torch.cuda.current_stream(x.device)
        st = stream if stream is not None else cur.cuda_stream
        T, H, E, I, k, g, G, cap = self.T, self.H, self.E, self.I, self.k, self.qg, self.G, self.cap
        if tuple(x.shape) != (T, H) or x.dtype != BF16:
            raise ValueError(f"x must be bf16 [{T}, {H}]")
        sgu = shared_gate_up.data_ptr() if shared_gate_up is not None else None
        sdn = shared_down.data_ptr() if shared_down is not None else None

        def shared_expert():   # the shared expert (no routed pairs) on the caller's stream
            lib.check(so.qw_moe_experts_w4_range(x.data_ptr(), gate_up_local.data_ptr(), down_local.data_ptr(),
                                                 sgu, sdn, T, H, E, I, k, g, 0, 0, ws.data_ptr(), st),
                      "ep shared expert")

        if not self.overlap:
            shared_expert()
        # dispatch
        lib.check(so.qw_moe_ep_pack(ws.data_ptr(), x.data_ptr(), T, H, E, k, G, cap, self.send_seg.data_ptr(), st),
                  "ep pack")
        if self.overlap:
            work = dist.all_to_all_single(self.recv_seg, self.send_seg, group=self.group, async_op=True)
            shared_expert()
            work.wait()
        else:
            dist.all_to_all_single(self.recv_seg, self.send_seg, group=self.group)
        # this rank's experts on the rows it received
        lib.check(so.qw_moe_ep_recv_route(self.recv_seg.data_ptr(), G, cap, H, E, self.ws_r.data_ptr(), st),
                  "ep receive routing")
        lib.check(so.qw_moe_ep_experts(self.recv_seg.data_ptr(), gate_up_local.data_ptr(), down_local.data_ptr(),
                                       G, cap, H, E, I, g, self.ws_r.data_ptr(), st), "ep local experts")
        # combine
        lib.check(so.qw_moe_ep_pack_out(self.ws_r.data_ptr(), self.recv_seg.data_ptr(), G, cap, H, E, I,
                                        self.send_back.data_ptr(), st), "ep pack outputs")
        dist.all_to_all_single(self.recv_back, self.send_back, group=self.group)
        lib.check(so.qw_moe_ep_scatter(ws.data_ptr(), self.recv_back.data_ptr(), T, H, E, I, k, G, cap, st),
                  "ep scatter")
