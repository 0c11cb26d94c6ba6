"""Expert parallelism for the routed MoE (the reference's multi-GPU serving plan: experts
sharded over the GPUs, dispatch and combine between them, attention and GDN per request).

Rank g of a process group of G ranks owns experts [g E/G, (g+1) E/G).  For one MoE layer
each rank routes its own tokens over all E experts (``qw_moe_route``), then
``ExpertParallelMoE.experts`` computes, into the same workspace, every routed
(token, slot) pair's expert output and the shared expert's, exactly as
``qw_moe_experts_w4`` would on one GPU holding all experts:

1. ``qw_moe_ep_dispatch``: each pair's activation row straight into the window of the
   rank owning its expert (stores over NVLink from the kernel), then a flag; the shared
   expert is every rank's last local expert, and each token sends it one more row, to
   its own rank, so it runs in the same expert launches as the routed pairs;
2. ``qw_moe_ep_recv_route`` (waits for every rank's rows) + ``qw_moe_ep_experts``: the
   received rows through the rank's own experts, the down projection storing its
   outputs straight into the source ranks' windows, then a flag;
3. either ``qw_moe_ep_scatter`` (waits for every rank's outputs) into the per-(token,
   slot) slots (the shared expert's into slot k), after which ``qw_moe_combine`` /
   ``qw_moe_combine_norm`` run unchanged, or ``qw_moe_ep_combine_norm``, which reads the
   returned rows directly (``combine_norm``).  The expert kernels give
a row the same bits whatever else is in their launch and outputs travel as bf16 (the
precision the combine reads), so the result equals the single-GPU MoE bit for bit.

The process group is used once, at construction, to swap the windows' IPC handles; the
data path is kernels only (no collective library, no host synchronisation), on the
caller's current stream, so it can be captured in a CUDA graph.
"""
from __future__ import annotations

import ctypes

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

    ``tokens`` is the rank's own token count per call (every rank the same).  Construction
    is collective (every rank of the group, same arguments); so is ``close()``."""

    def __init__(self, group, *, tokens: int, hidden: int, experts: int, inter: int, top_k: int,
                 quant_group: int, device, shared: bool = True):
        self.group = group
        self.G = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.T, self.H, self.E, self.I, self.k, self.qg = tokens, hidden, experts, inter, top_k, quant_group
        self.lo, self.el = expert_range(experts, self.G, self.rank)
        self.shared = int(bool(shared))
        self.local = self.el + self.shared          # local experts (the shared one last)
        self.cap = tokens * (top_k + self.shared)
        self.device = torch.device(device)
        self.so = lib.load()
        so, G = self.so, self.G
        nbytes = so.qw_ep_window_bytes(G, self.cap, hidden)
        if nbytes < 0:
            raise ValueError("expert parallelism: unsupported rank count or shape")
        with torch.cuda.device(self.device):
            win = ctypes.c_void_p()
            handle = ctypes.create_string_buffer(64)
            lib.check(so.qw_ep_window_alloc(nbytes, ctypes.byref(win), handle), "ep window")
            self.window = win.value
            handles = [None] * G
            dist.all_gather_object(handles, bytes(handle.raw), group=group)
            self._opened = []
            ptrs = []
            for g, h in enumerate(handles):
                if g == self.rank:
                    ptrs.append(self.window)
                    continue
                peer = ctypes.c_void_p()
                lib.check(so.qw_ep_window_open(ctypes.create_string_buffer(h, 64), ctypes.byref(peer)),
                          f"ep window of rank {g}")
                self._opened.append(peer.value)
                ptrs.append(peer.value)
        self.peers = torch.tensor(ptrs, dtype=torch.int64, device=self.device)
        nbytes = so.qw_moe_ep_recv_workspace_bytes(G, self.cap, hidden, self.local, inter)
        self.ws_r = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
        dist.barrier(group=group)

    def close(self):
        """Unmap the peers' windows and free this rank's (collective)."""
        if self.window is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for p in self._opened:
            lib.check(self.so.qw_ep_window_close(p), "ep window close")
        self._opened = []
        dist.barrier(group=self.group)
        lib.check(self.so.qw_ep_window_free(self.window), "ep window free")
        self.window = None

    def local_banks(self, gate_up: torch.Tensor, down: torch.Tensor, shared_gate_up: torch.Tensor | None = None,
                    shared_down: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
        """This rank's expert streams from full W4 banks (every expert's stream, equal sizes,
        concatenated): its E/G routed experts, then the shared expert when it is exchanged."""
        gu = local_expert_streams(gate_up, self.E, self.G, self.rank)
        dn = local_expert_streams(down, self.E, self.G, self.rank)
        if self.shared:
            if shared_gate_up is None or shared_down is None:
                raise ValueError("the shared expert's streams are needed (shared=True)")
            gu = torch.cat([gu.view(-1), shared_gate_up.reshape(-1)])
            dn = torch.cat([dn.view(-1), shared_down.reshape(-1)])
        return gu, dn

    def experts(self, x: torch.Tensor, ws: torch.Tensor, gate_up_local: torch.Tensor, down_local: torch.Tensor,
                scatter: bool = True):
        """Routed (and shared) expert outputs of this rank's tokens ``x`` [tokens, hidden]
        (bf16) for the routing in ``ws`` (a MoE workspace already routed by qw_moe_route /
        qw_moe_route_x), on the current stream; ``gate_up_local`` / ``down_local`` come from
        ``local_banks``.  With ``scatter`` they land in ``ws``'s per-(token, slot) outputs;
        without, they stay in the window for ``combine_norm``, which must follow.  Every
        rank of the group calls it, with the same shapes, in the same order."""
        so = self.so
        st = torch.cuda.current_stream(x.device).cuda_stream
        T, H, E, I, k, g, G, cap = self.T, self.H, self.E, self.I, self.k, self.qg, self.G, self.cap
        if tuple(x.shape) != (T, H) or x.dtype != BF16:
            raise ValueError(f"x must be bf16 [{T}, {H}]")
        win, peers, L, sh = self.window, self.peers.data_ptr(), self.local, self.shared
        lib.check(so.qw_moe_ep_dispatch(ws.data_ptr(), x.data_ptr(), T, H, E, k, G, self.rank, cap, sh, peers, win,
                                        st), "ep dispatch")
        lib.check(so.qw_moe_ep_recv_route(win, G, cap, H, L, self.ws_r.data_ptr(), st), "ep receive routing")
        lib.check(so.qw_moe_ep_experts(win, gate_up_local.data_ptr(), down_local.data_ptr(), G, self.rank, cap, H, L,
                                       I, g, peers, self.ws_r.data_ptr(), st), "ep local experts")
        if scatter:
            lib.check(so.qw_moe_ep_scatter(ws.data_ptr(), win, T, H, E, I, k, G, cap, sh, st), "ep scatter")

    def combine_norm(self, ws: torch.Tensor, hidden: torch.Tensor, gamma: torch.Tensor, normed: torch.Tensor,
                     eps: float, tap, ldf: int, tap_normed: int):
        """``qw_moe_combine_norm`` over the rows the exchange returned (after
        ``experts(..., scatter=False)``): hidden += MoE, normed = RMSNorm(hidden), the
        optional tap."""
        if not self.shared:
            raise ValueError("combine_norm reads the shared expert's row from the exchange (shared=True)")
        st = torch.cuda.current_stream(hidden.device).cuda_stream
        lib.check(self.so.qw_moe_ep_combine_norm(ws.data_ptr(), self.window, self.G, self.cap, hidden.data_ptr(),
                                                 self.T, self.H, self.E, self.I, self.k, 1, gamma.data_ptr(),
                                                 normed.data_ptr(), eps, tap, ldf, tap_normed, st),
                  "ep combine_norm")
