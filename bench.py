"""Benchmark: Qwen3.5-MoE target block verify (block 16, W4 MoE + GDN) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference] [--ctx 4096]

One "step" is one verify of a 16-token block per sequence through all 40 layers
(30 gated-DeltaNet + 10 full attention, 256 experts top-8 + shared, W4A16 group 128,
vocab 248320), the lm_head argmax, the device-side acceptance and the commit of the
accepted prefix (GDN states, conv tails, KV position) — the benchmark's fourth
configuration: batch 1, 4096 tokens of bf16 paged KV context, random-init weights
N(0, 0.02), seeded synthetic context and proposals.  The step runs as one CUDA graph.

value     verify tok/s = batch * 16 / step time (device time, CUDA events, max over ranks,
          inputs resident in HBM); weights streamed per step (~8.5 GB) exceed L2, so no
          flush is needed between steps.
e2e       the same metric through TargetEngine.serve_step (proposals from pinned host
          memory, accepted counts and next tokens back to the host every step).
roofline  the dominant kernel (routed-expert gate/up), achieved algorithmic bytes per
          launch / its CUDA-event duration against the measured HBM copy bandwidth.
cpu_baseline / --impl reference
          the reference's CPU path (torch on every host core: the restatement of
          reference/fused_ops.py and fused/model.py in oracle/ref_torch.py, bf16 weights):
          one GDN layer, one attention layer and one MoE layer at the same shapes and 1/8
          of the lm_head per sample, a verify step extrapolated as 30*GDN + 10*attention +
          40*MoE + 8*(lm_head/8); the reference arm runs one sample per step.
Multi-GPU (torchrun): expert parallelism -- every rank serves its own requests (the
same per-GPU workload as one GPU, "scaling": "weak") and holds E/N of the routed experts
of every MoE layer; rows go to their experts' ranks and back by kernel stores into the
peers' windows (NVLink), value sums the ranks.  --replicas runs independent replicas.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "verify tok/s & step latency (block 16, W4 MoE+GDN); % HBM roofline"

# DRAM bytes (read + write) of one moe_up_bulk_kernel launch, from one ncu capture of the
# same launch (16 tokens of N(0,1) router logits, seed 17 -> 103 active experts; metrics
# dram__bytes_read.sum + dram__bytes_write.sum): ncu cannot run inside the timed bench
MOE_UP_NCU_TRAFFIC = {"bytes": 112_598_016 + 3_043_840, "active": 103,
                      "source": "ncu capture of moe_up_bulk_kernel on the bench routing (103 active experts), "
                                "dram__bytes_read.sum + dram__bytes_write.sum"}


def _peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 20 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "20"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = max(mx, float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() in ("active", "1"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------- CPU side
def _host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


class CpuReference:
    """The reference's CPU path (torch on the host cores: oracle/ref_torch.py restates
    reference/fused_ops.py and the layer bodies of fused/model.py) at the benchmark's
    config-4 shapes: one gated-DeltaNet layer, one attention layer over 4096 tokens of
    context, one MoE layer (16 tokens, top-8 of 256 + shared) and 1/8 of the lm_head,
    dense bf16 weights N(0, 0.02) (the W4 weights dequantized), fp32 GDN state.  A sample
    times one of each; a verify step is extrapolated as 30 GDN + 10 attention + 40 MoE +
    8 x (1/8 lm_head)."""

    def __init__(self, ctx: int = 4096, seed: int = 7):
        import torch
        self.threads = _host_cores()
        torch.set_num_threads(self.threads)   # torchrun exports OMP_NUM_THREADS=1
        import __graft_entry__
        __graft_entry__.load_package()
        from qwen35_dflash_b200.config import QWEN35_35B_A3B
        self.cfg = c = QWEN35_35B_A3B
        self.ctx = ctx
        gen = torch.Generator().manual_seed(seed)
        bf = torch.bfloat16

        def w(*shape, std=0.02):
            return (torch.randn(*shape, generator=gen) * std).to(bf)

        H, E, I = c.hidden_size, c.num_experts, c.moe_intermediate_size
        D, Hq, Hkv = c.head_dim, c.num_attention_heads, c.num_key_value_heads
        vh, dk, dv = c.linear_num_value_heads, c.linear_key_head_dim, c.linear_value_head_dim
        self.gdn_w = {"qkv": w(c.conv_channels, H), "z": w(c.value_width, H), "b": w(vh, H), "a": w(vh, H),
                      "A_log": torch.log(torch.arange(1, vh + 1, dtype=torch.float32)),
                      "dt_bias": w(vh).float(), "conv": w(c.conv_channels, 1, c.linear_conv_kernel_dim),
                      "norm": torch.ones(dv, dtype=bf), "out": w(H, c.value_width)}
        self.conv_hist = torch.randn(1, c.conv_channels, c.linear_conv_kernel_dim - 1, generator=gen).to(bf)
        self.state = torch.randn(1, vh, dk, dv, generator=gen) * 0.02
        self.attn_w = {"q": w(Hq * 2 * D, H), "k": w(Hkv * D, H), "v": w(Hkv * D, H), "o": w(H, Hq * D),
                       "q_norm": torch.zeros(D, dtype=bf), "k_norm": torch.zeros(D, dtype=bf)}
        self.key = torch.randn(1, Hkv, ctx, D, generator=gen).to(bf)
        self.value = torch.randn(1, Hkv, ctx, D, generator=gen).to(bf)
        self.moe_w = {"router": w(E, H), "shared_gu": w(2 * c.shared_expert_intermediate_size, H),
                      "shared_down": w(H, c.shared_expert_intermediate_size), "shared_gate": w(1, H)}
        self._experts = {}
        self._expert_seed = seed
        self.lm = w(c.vocab_size // 8, H)
        self.x = torch.randn(1, 16, H, generator=gen).to(bf)

    def _expert(self, e):
        import torch
        if e not in self._experts:
            g = torch.Generator().manual_seed(self._expert_seed * 1000 + e)
            H, I = self.cfg.hidden_size, self.cfg.moe_intermediate_size
            self._experts[e] = ((torch.randn(2 * I, H, generator=g) * 0.02).to(torch.bfloat16),
                                (torch.randn(H, I, generator=g) * 0.02).to(torch.bfloat16))
        return self._experts[e]

    def sample(self) -> dict:
        """Seconds of one layer of each kind and of 1/8 of the lm_head."""
        import torch
        import torch.nn.functional as Fn
        from oracle import ref_torch as R
        c, x = self.cfg, self.x
        t = {}
        with torch.inference_mode():
            t0 = time.perf_counter()
            R.gdn_layer(x, self.gdn_w, self.conv_hist, self.state, kh=c.linear_num_key_heads,
                        vh=c.linear_num_value_heads, dk=c.linear_key_head_dim, dv=c.linear_value_head_dim)
            t["gdn"] = time.perf_counter() - t0
            t0 = time.perf_counter()
            R.attention_layer(x, self.attn_w, self.key, self.value, self.ctx, heads=c.num_attention_heads,
                              kv_heads=c.num_key_value_heads, dim=c.head_dim, rot=c.rotary_dim, theta=c.rope_theta)
            t["attn"] = time.perf_counter() - t0
            t0 = time.perf_counter()
            R.moe_layer(x, self.moe_w, self._expert, top_k=c.num_experts_per_tok)
            t["moe"] = time.perf_counter() - t0
            t0 = time.perf_counter()
            Fn.linear(x[0], self.lm)
            t["lm8"] = time.perf_counter() - t0
        t["sample"] = sum(t.values())
        t["step"] = 30 * t["gdn"] + 10 * t["attn"] + 40 * t["moe"] + 8 * t["lm8"]
        return t

    def describe(self, t: dict) -> str:
        return (f"torch CPU restatement of the reference path (oracle/ref_torch.py), bf16 weights, "
                f"{self.threads} threads; per sample one GDN layer {t['gdn']*1e3:.1f} ms, one attention layer "
                f"(ctx {self.ctx}) {t['attn']*1e3:.1f} ms, one MoE layer (16 tokens, top-8 of 256 + shared) "
                f"{t['moe']*1e3:.1f} ms, 1/8 lm_head {t['lm8']*1e3:.1f} ms; verify step extrapolated as "
                f"30 GDN + 10 attention + 40 MoE + 8 x lm_head/8 = {t['step']*1e3:.0f} ms")


def cpu_baseline_leg(samples: int = 5) -> dict:
    """cpu_baseline of the GPU arm: best of ``samples`` after one warm-up sample."""
    ref = CpuReference()
    ref.sample()
    best = min((ref.sample() for _ in range(samples)), key=lambda t: t["step"])
    return {"value": round(16 / best["step"], 4), "unit": "tok/s", "cores": ref.threads, "kind": "port",
            "sample": ref.describe(best) + f" (best of {samples} after 1 warm-up)"}


# ---------------------------------------------------------------------------- GPU side
def print_timeline(prof, detail: bool = False):
    """Per kernel of one graph replay: launches, summed duration and the time it adds to
    the step's critical path (its end minus the latest end before it, in start order).
    detail: also every launch of decoder layers 4-7 in order (start from the step's
    first start, duration, added)."""
    import collections
    evs = sorted(((e.name, e.time_range.start, e.time_range.end) for e in prof.events()
                  if e.device_type.name == "CUDA"), key=lambda x: x[1])
    steps, cur = [], []
    for name, s, e in evs:   # replays are separated by the host-side token copies
        if "qw::" not in name and "nccl" not in name:
            if cur:
                steps.append(cur)
            cur = []
            continue
        cur.append((name, s, e))
    if cur:
        steps.append(cur)
    st = steps[-1]
    cnt, dur, marg = collections.Counter(), collections.Counter(), collections.Counter()
    prev = st[0][1]
    rows = []
    for name, s, e in st:
        n = name.split("<")[0].split("(")[0].replace("void ", "")
        cnt[n] += 1
        dur[n] += e - s
        marg[n] += max(e, prev) - prev
        rows.append((n, s - st[0][1], e - s, max(e, prev) - prev))
        prev = max(prev, e)
    if detail:
        # the launches of layers 4-7: after the embedding norm, 10 per GDN layer and 11 per
        # attention layer (layers 3, 7, ... are attention)
        first = 1 + 4 * 10 + 1
        for n, start, d, added in rows[first:first + 41]:
            print(f"  {n:34s} start {start:9.1f} dur {d:7.2f} added {added:6.2f}")
    print(f"timeline: {len(st)} launches, {st[-1][2] - st[0][1]:.1f} us from first start to last end")
    print(f"{'kernel':40s} {'launches':>8s} {'dur us':>9s} {'added us':>9s} {'per launch':>10s}")
    for n, m in marg.most_common():
        print(f"{n:40s} {cnt[n]:8d} {dur[n]:9.1f} {m:9.1f} {m / cnt[n]:10.2f}")


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    import __graft_entry__
    __graft_entry__.load_package()
    from qwen35_dflash_b200 import engine as E, lib
    from qwen35_dflash_b200.config import QWEN35_35B_A3B

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    cfg = QWEN35_35B_A3B
    S = 16
    if args.requests:
        # benchmark config 5: the requests split evenly over the GPUs
        if args.requests % world:
            raise SystemExit(f"--requests {args.requests} does not split over {world} GPUs")
        args.batch = args.requests // world
    B = args.batch
    total_steps = args.warmup + args.steps
    capacity = args.ctx + S + (total_steps + args.e2e_steps + 8) * S
    capacity = (capacity + 15) // 16 * 16
    t_init = time.perf_counter()
    weights = E.weights_random(cfg, seed=2, device=dev)
    ep = world > 1 and not args.replicas
    eng = E.TargetEngine(cfg, weights, batch=B, block=S, capacity=capacity, device=dev,
                         ep_group=dist.group.WORLD if ep else None)
    eng.set_random_context(args.ctx, seed=3 + rank)
    if args.zipf > 0:
        # routing skew: a per-expert router-logit bias log p_e, p_e ~ rank^-s over a seeded
        # permutation of the experts (the same on every GPU)
        perm = torch.randperm(cfg.num_experts, generator=torch.Generator().manual_seed(3))
        ranks = torch.empty(cfg.num_experts)
        ranks[perm] = torch.arange(1, cfg.num_experts + 1, dtype=torch.float32)
        p = ranks.pow(-args.zipf)
        eng.router_bias = (p / p.sum()).log().to(torch.bfloat16).to(dev)
    torch.cuda.synchronize(dev)
    init_s = time.perf_counter() - t_init

    # algorithmic bytes of one step: routed experts actually selected per layer
    eng.tokens.random_(0, cfg.vocab_size)
    active = {}
    snap = eng.snapshot()
    eng.forward(after_moe_route=lambda l: active.__setitem__(l, eng.active_experts()))
    eng.restore(snap)
    alg = eng.algorithmic_bytes([active[l] for l in range(cfg.num_hidden_layers)])

    eng.capture()
    launches = eng.launches_per_step()
    gen = torch.Generator(device=dev)
    gen.manual_seed(11 + rank)
    props = torch.randint(0, cfg.vocab_size, (total_steps, B * S), generator=gen, device=dev, dtype=torch.int32)

    def step(i):
        eng.tokens.copy_(props[i])
        eng.tokens.view(B, S)[:, 0].copy_(eng.next_token)   # the block starts at the anchor
        eng.replay()

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize(dev)
    if args.timeline:
        # in-graph kernel timeline of the last of two steps (CUPTI through torch.profiler)
        from torch.profiler import profile, ProfilerActivity
        if world > 1:
            dist.barrier()
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            for i in range(2):
                step(args.warmup + i)
            torch.cuda.synchronize(dev)
        if rank == 0:
            print_timeline(prof, detail=args.timeline_detail)
        if world > 1:
            dist.barrier()
        eng.close()
        return None
    if args.profile_step:
        # one step between cudaProfilerStart/Stop (ncu --profile-from-start off)
        torch.cuda.profiler.start()
        step(args.warmup)
        torch.cuda.synchronize(dev)
        torch.cuda.profiler.stop()
        eng.close()
        return None
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clocks:
        ev0.record()
        for i in range(args.steps):
            step(args.warmup + i)
        ev1.record()
        torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    ms = ev0.elapsed_time(ev1) / args.steps
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())

    # end to end through the public serving call (pinned host in/out, sync per step)
    host_in = torch.empty(B * S, dtype=torch.int32).pin_memory()
    host_out = torch.empty(2 * B, dtype=torch.int32).pin_memory()
    host_out[B:] = eng.next_token.cpu()
    hrng = torch.Generator().manual_seed(5 + rank)
    for _ in range(2):
        host_in.copy_(torch.randint(0, cfg.vocab_size, (B * S,), generator=hrng, dtype=torch.int32))
        host_in.view(B, S)[:, 0] = host_out[B:]
        eng.serve_step(host_in, host_out)
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.e2e_steps):
        host_in.copy_(torch.randint(0, cfg.vocab_size, (B * S,), generator=hrng, dtype=torch.int32))
        host_in.view(B, S)[:, 0] = host_out[B:]
        eng.serve_step(host_in, host_out)
    e2e_ms = (time.perf_counter() - t0) * 1e3 / args.e2e_steps
    te = torch.tensor([e2e_ms], device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_ms = float(te.item())

    # dominant kernel: routed-expert gate/up (largest share of the step's HBM bytes)
    rl = time_moe_up(eng, cfg, dev)
    result = None
    if rank == 0:
        hbm, peak_kind = _peaks()
        tok = B * S * world
        rl_achieved = rl["bytes"] / (rl["us"] * 1e-6) / 1e9
        result = {
            "metric": METRIC,
            "value": round(tok / (ms_max * 1e-3), 2),
            "unit": "tok/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_max, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (random-init weights N(0,0.02) W4A16 g128, seeded KV/GDN context and proposals)",
            "config": {"workload": (f"benchmark config 5: {B * world} requests ({B} per GPU), ctx {args.ctx}, "
                                    f"Zipf({args.zipf}) routing skew" if args.requests else
                                    ("full target verify forward, experts sharded over the GPUs "
                                     "(benchmark config 4 per GPU, config 5's expert parallelism)") if ep else
                                    "full target verify forward, 1 GPU per replica (benchmark config 4)"),
                       "model": "Qwen3.5-35B-A3B target (40 layers: 30 GDN + 10 attention)",
                       "global_batch": B * world, "block": S, "ctx": args.ctx, "seq_len": args.ctx + S,
                       "parallelism": (f"ep{world} (experts {cfg.num_experts // world} per GPU; dispatch and "
                                       "combine by kernel stores into the peers' windows over NVLink; "
                                       "attention/GDN per request)") if ep else
                                      f"dp{world} (independent replicas)",
                       "l2": "no flush: each step streams ~8.5 GB of weights, far above the 126 MB L2",
                       "step_alg_bytes": alg["total"], "alg_bytes_parts": alg,
                       "routed_experts_per_layer_mean": round(sum(active.values()) / len(active), 1),
                       "step_hbm_frac_of_measured": round(alg["total"] / (ms_max * 1e-3) / (hbm * 1e9), 4),
                       "init_s": round(init_s, 1)},
            "e2e": {"value": round(tok / (e2e_ms * 1e-3), 2), "unit": "tok/s", "ms_per_step": round(e2e_ms, 4),
                    "h2d_bytes_per_step": B * S * 4, "d2h_bytes_per_step": eng.serve_d2h_bytes(),
                    "api": "TargetEngine.serve_step (pinned host proposals -> graph -> accepted/next tokens "
                           "+ device wait status)"},
            "gpu_launches": launches,
            "roofline": {"bound": "hbm", "kernel": "moe_up_bulk_kernel (routed + shared expert gate/up, W4A16)",
                         "achieved": round(rl_achieved, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(rl_achieved / hbm, 4), "peak_kind": f"{peak_kind} burst copy",
                         "traffic": MOE_UP_NCU_TRAFFIC["bytes"] if rl["active"] == MOE_UP_NCU_TRAFFIC["active"] else None,
                         "traffic_source": MOE_UP_NCU_TRAFFIC["source"],
                         "bytes_per_launch": rl["bytes"], "us_per_launch": round(rl["us"], 2),
                         "active_experts": rl["active"]},
            "clocks": clocks.summary(),
        }
    eng.close()
    return result


def time_moe_up(eng, cfg, dev, iters: int = 50):
    """CUDA-event time of one routed-expert gate/up launch on layer 0's weights with the
    routing of 16 tokens of N(0,1) router logits (the benchmark's MoE statistics)."""
    import torch
    from qwen35_dflash_b200 import lib
    T, H, E, k, I, g = eng.T, cfg.hidden_size, cfg.num_experts, cfg.num_experts_per_tok, \
        cfg.moe_intermediate_size, cfg.quant_group
    lw = eng.layers[0]
    gen = torch.Generator(device=dev)
    gen.manual_seed(17)
    x = torch.randn(T, H, device=dev, generator=gen).to(torch.bfloat16)
    logits = torch.randn(T, eng.nrouter, device=dev, generator=gen).to(torch.bfloat16)
    ws = eng.moe_ws
    st = torch.cuda.current_stream(dev).cuda_stream
    so = eng.lib
    lib.check(so.qw_moe_route_x(logits.data_ptr(), lib.QW_BF16, eng.nrouter, T, E, k, E, lib.QW_BF16,
                                x.data_ptr(), H, g, ws.data_ptr(), st, 0))
    args = (x.data_ptr(), lw.gate_up.data_ptr(), lw.down.data_ptr(), lw.shared_gu.data_ptr(),
            lw.shared_down.data_ptr(), T, H, E, I, k, g, ws.data_ptr(), st)
    for _ in range(5):
        lib.check(so.qw_moe_up_w4(*args))
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    times = []
    for _ in range(iters):
        flush.zero_()  # evict the experts from L2 between launches
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        lib.check(so.qw_moe_up_w4(*args))
        e1.record()
        e1.synchronize()
        times.append(e0.elapsed_time(e1) * 1e3)
    off = so.qw_moe_active_experts(None, T, E, k)
    active = int(ws[off:off + 4].view(torch.int32).item())
    w4b = 2 * I * H // 2 + 2 * I * (H // g) * 2
    nbytes = (active + 1) * w4b + T * H * 2 + (T * k + T) * I * 2
    return {"us": statistics.median(times), "bytes": nbytes, "active": active}


def run_reference(args, rank, world):
    """The reference arm: the reference's CPU path on the host cores, rank 0 only (other
    ranks exit without work).  Each of the W + K steps runs one sample (one layer of each
    kind + 1/8 lm_head; about a tenth of a second); ms_per_step is the timed sample's
    wall time, value the verify tok/s of the step extrapolated from the K samples'
    medians."""
    if rank != 0:
        return None
    ref = CpuReference(ctx=args.ctx)
    for _ in range(args.warmup):
        ref.sample()
    runs = [ref.sample() for _ in range(args.steps)]
    med = {key: statistics.median(r[key] for r in runs) for key in runs[0]}
    med["step"] = 30 * med["gdn"] + 10 * med["attn"] + 40 * med["moe"] + 8 * med["lm8"]
    value = 16 / med["step"]
    desc = ref.describe(med) + f" (medians of {args.steps} samples after {args.warmup} warm-up samples)"
    return {"metric": METRIC, "impl": "reference", "value": round(value, 4), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(med["sample"] * 1e3, 2),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random-init bf16 weights N(0,0.02), seeded context)",
            "config": {"workload": "full target verify forward (benchmark config 4), extrapolated per step "
                                   "from one layer of each kind", "block": 16, "ctx": args.ctx, "global_batch": 1,
                       "ms_per_verify_step_extrapolated": round(med["step"] * 1e3, 1)},
            "cpu_baseline": {"value": round(value, 4), "unit": "tok/s", "cores": ref.threads, "kind": "port",
                             "sample": desc},
            "e2e": {"value": round(value, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def run_kernels(args):
    """Per-kernel CUDA-event timings of the verify step's kernels on a 4-layer model of
    the full width (about 2 GB of weights on the device): each launch cycles through the
    4 layers' weights so successive launches stream from HBM, not L2.  The small case
    for ncu captures (``--kernels --kernel-reps 1``)."""
    import torch
    import __graft_entry__
    __graft_entry__.load_package()
    from qwen35_dflash_b200 import config, engine as E, lib
    cfg = config.with_layers(config.QWEN35_35B_A3B, 4)
    eng = E.TargetEngine(cfg, E.weights_random(cfg, seed=2), batch=1, block=16, capacity=args.ctx + 64)
    eng.set_random_context(args.ctx, seed=3)
    so, T, H = eng.lib, eng.T, cfg.hidden_size
    Ex, k, I, g = cfg.num_experts, cfg.num_experts_per_tok, cfg.moe_intermediate_size, cfg.quant_group
    st = torch.cuda.Stream()
    s = st.cuda_stream
    gen = torch.Generator(device="cuda").manual_seed(17)
    x = torch.randn(T, H, device="cuda", generator=gen).to(torch.bfloat16)
    logits = torch.randn(T, eng.nrouter, device="cuda", generator=gen).to(torch.bfloat16)
    ws = eng.moe_ws
    L = eng.layers
    gl = [lw for lw in L if lw.kind == "linear_attention"]

    def chk(rc):
        lib.check(rc)

    def route():
        chk(so.qw_moe_route_x(logits.data_ptr(), lib.QW_BF16, eng.nrouter, T, Ex, k, Ex, lib.QW_BF16, x.data_ptr(), H,
                              g, ws.data_ptr(), s, 0))

    def up(lw):
        return lambda: chk(so.qw_moe_up_w4(x.data_ptr(), lw.gate_up.data_ptr(), lw.down.data_ptr(),
                                           lw.shared_gu.data_ptr(), lw.shared_down.data_ptr(), T, H, Ex, I, k, g,
                                           ws.data_ptr(), s))

    def down(lw):
        return lambda: chk(so.qw_moe_down_w4(x.data_ptr(), lw.gate_up.data_ptr(), lw.down.data_ptr(),
                                             lw.shared_gu.data_ptr(), lw.shared_down.data_ptr(), T, H, Ex, I, k, g,
                                             ws.data_ptr(), s))

    def qkvz(lw):
        return lambda: chk(so.qw_w4_linear(x.data_ptr(), lw.qkvz.data_ptr(), eng.proj[0].data_ptr(), lib.QW_OUT_BF16,
                                           eng.ldp, T, eng.ldp, H, g, s))

    def gdn(gi):
        return lambda: chk(so.qw_gdn_verify(eng.gdn_dims, eng.gdn_desc.data_ptr(), gi, s))

    def attn(ai):
        D, Hq, Hkv = cfg.head_dim, cfg.num_attention_heads, cfg.num_key_value_heads
        return lambda: chk(so.qw_attn_paged(eng.qout.data_ptr(), eng.k_cache[ai].data_ptr(),
                                            eng.v_cache[ai].data_ptr(), eng.pages.data_ptr(), eng.max_pages, eng.P,
                                            eng.qpos.data_ptr(), eng.capacity, eng.qkv.data_ptr() + D * 2, eng.ldq,
                                            eng.attn_out.data_ptr(), eng.B, eng.S, Hq, Hkv, D, D ** -0.5,
                                            eng.attn_ws.data_ptr(), s))

    def lmhead():
        return lambda: chk(so.qw_lmhead_argmax(x.data_ptr(), eng.glob["lm_head"].data_ptr(), None, eng.keys.data_ptr(),
                                               T, eng.vocab_pad, H, s))

    def combine_norm(lw):
        return lambda: chk(so.qw_moe_combine_norm(ws.data_ptr(), eng.hidden.data_ptr(), T, H, Ex, I, k, 1,
                                                  lw.in_norm.data_ptr(), eng.normed.data_ptr(), cfg.rms_norm_eps,
                                                  None, 0, 0, s))

    with torch.cuda.stream(st):
        route()
        up(L[0])()
        down(L[0])()
    torch.cuda.synchronize()
    active = eng.active_experts()
    w4 = lambda n, kk: n * kk // 2 + n * (kk // g) * 2
    cases = [("route", [route], 0), ("moe_up", [up(lw) for lw in L], (active + 1) * w4(2 * I, H)),
             ("moe_down", [down(lw) for lw in L], (active + 1) * w4(H, I)),
             ("w4_qkvz", [qkvz(lw) for lw in gl], w4(eng.ldp, H)),
             ("gdn_verify", [gdn(i) for i in range(len(gl))], 0),
             ("attn_paged", [attn(i) for i in range(len(eng.k_cache))],
              2 * cfg.num_key_value_heads * (args.ctx + 16) * cfg.head_dim * 2),
             ("lm_head_argmax", [lmhead()], cfg.vocab_size * H * 2),
             ("combine_norm", [combine_norm(lw) for lw in L], T * (k + 1) * H * 4 + 3 * T * H * 2)]
    out = {"kernels": {}, "active_experts": active, "ctx": args.ctx}
    for name, fns, nbytes in cases:
        with torch.cuda.stream(st):
            for f in fns:
                f()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=st):
            for _ in range(args.kernel_reps):
                for f in fns:
                    f()
        graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()           # graph.replay() runs on the current stream
        graph.replay()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / (args.kernel_reps * len(fns))
        entry = {"us": round(us, 2)}
        if nbytes:
            entry.update(bytes=nbytes, gbs=round(nbytes / us / 1e3, 1))
        out["kernels"][name] = entry
        del graph
    print(json.dumps(out), flush=True)


def _event_times(fn, reps: int, flush) -> float:
    """Median CUDA-event time (us) of fn() over reps launches, L2 flushed before each."""
    import torch
    times = []
    for _ in range(reps):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        e1.synchronize()
        times.append(e0.elapsed_time(e1) * 1e3)
    return statistics.median(times)


def run_prefill(args):
    """Prompt prefill of the full target (1 GPU, random weights of the architecture): a
    prompt of --prefill-tokens tokens committed in chunks of 64 tokens per forward (the
    prefill engine) and, for comparison, in verify blocks of 16.  CUDA events around the
    whole prefill (every chunk's forward + accept + commit); prefill tokens/s."""
    import torch
    import __graft_entry__
    __graft_entry__.load_package()
    from qwen35_dflash_b200 import config, engine as E
    dev = torch.device("cuda")
    cfg = config.QWEN35_35B_A3B
    n = args.prefill_tokens
    te = E.TargetEngine(cfg, E.weights_random(cfg, seed=2, device=dev), batch=1, block=16, capacity=n + 128,
                        device=dev)
    gen = torch.Generator().manual_seed(5)
    prompt = torch.randint(0, cfg.vocab_size, (n,), generator=gen, dtype=torch.int32).tolist()
    out = {"metric": "prefill tok/s (1 GPU, Qwen3.5-35B-A3B target, random-init weights)", "prompt_tokens": n}
    for block in (64, 16):
        eng = te if block == 16 else te.prefill_engine(block)
        chunks = [torch.tensor(prompt[i:i + block] + [0] * (block - len(prompt[i:i + block])), dtype=torch.int32)
                  for i in range(0, n, block)]
        counts = [min(block, n - i) for i in range(0, n, block)]

        def run():
            te.qpos.zero_(); te.state.zero_(); te.conv_hist.zero_()
            for c, k in zip(chunks, counts):
                eng.tokens.copy_(c, non_blocking=True)
                eng.forward()
                eng.accept(auto_commit=False)
                eng.accepted.fill_(k)
                eng.commit()
        run()   # warm-up
        torch.cuda.synchronize()
        times = []
        for _ in range(3):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(); run(); e1.record(); e1.synchronize()
            times.append(e0.elapsed_time(e1) / 1e3)
        best = min(times)
        eng.raise_on_wait_timeout()
        out[f"chunk{block}"] = {"s": round(best, 4), "tok_s": round(n / best, 1), "forwards": len(chunks)}
    print(json.dumps(out), flush=True)


def run_dflash(args):
    """The greedy DFlash loop on the full target and the full draft (1 GPU, random weights
    of both architectures): a --ctx-token prompt prefilled in 64-token chunks, then the
    DFlash step -- the draft's proposals, the target's block verify + accept + commit, the
    draft's context extension -- captured as one CUDA graph and replayed --steps times
    after --warmup replays, CUDA events around the replays; then the target's own verify
    step (its graph) timed the same way, so that the difference is the draft's share.
    With random weights the proposals are almost never accepted: the step latency is the
    figure that carries over to trained weights, where a step emits 1 + accepted tokens."""
    import torch
    import __graft_entry__
    __graft_entry__.load_package()
    from qwen35_dflash_b200 import config, engine as E, synthetic
    from qwen35_dflash_b200.dflash import DFlash
    from qwen35_dflash_b200.draft import DraftEngine
    dev = torch.device("cuda")
    cfg, dcfg = config.QWEN35_35B_A3B, config.QWEN35_DFLASH_DRAFT
    n, k, w = args.ctx, args.steps, args.warmup
    cap = n + 16 * (2 * (k + w) + 8) + 128
    te = E.TargetEngine(cfg, E.weights_random(cfg, seed=2, device=dev), batch=1, block=16, capacity=cap, device=dev)
    df = DFlash(te, DraftEngine(dcfg, te, synthetic.init_draft_weights(dcfg), device=dev))
    gen = torch.Generator().manual_seed(5)
    df.prefill(torch.randint(0, cfg.vocab_size, (n,), generator=gen, dtype=torch.int32).tolist())
    df.capture()

    def timed(replay):
        for _ in range(w):
            replay()
        torch.cuda.synchronize()
        q0 = int(te.qpos[0].item())
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(k):
            replay()
        e1.record()
        e1.synchronize()
        te.raise_on_wait_timeout()
        return e0.elapsed_time(e1) / k, (int(te.qpos[0].item()) - q0) / k

    ms, tok = timed(df.graph.replay)
    te.capture()
    ms_verify, _ = timed(te.replay)
    print(json.dumps({
        "metric": "DFlash step latency (draft propose + target block verify/accept/commit + draft extend), 1 GPU",
        "ctx": n, "steps": k, "warmup": w, "ms_per_dflash_step": round(ms, 4),
        "tokens_per_step": round(tok, 3), "tok_s": round(tok / ms * 1e3, 1),
        "ms_per_verify_step": round(ms_verify, 4), "draft_ms_per_step": round(ms - ms_verify, 4),
        "data": "random-init weights of the target and draft architectures: proposals ~never accepted; "
                "a trained draft emits 1 + accepted tokens per step"}), flush=True)


def run_micro(args):
    """Benchmark configs 2 and 3 (one JSON line per point): the W4A16 grouped MoE
    (router logits given, softmax top-8 + shared expert, H 2048, 256 experts, I 512, g128,
    scales U(0.005, 0.02)) at T = 16, 64, 256 -- routing + experts + combine; also with
    skewed routing (config 5's Zipf bias at T = 256 and 1024, and 8 hot experts), each
    timed with the default grouped kernels ("us") and with the tcgen05 dense-expert
    kernels enabled at 128 pairs ("us_tcgen05_dense") -- and the
    gated-DeltaNet verify at B = 1, 8, 32 (16 QK / 32 V heads of 128, block 16) -- verify
    + commit of all 16 tokens.  CUDA events around each launch group, L2 flushed (256 MB
    write) before each; achieved = algorithmic bytes / time against the measured HBM
    copy bandwidth."""
    import torch
    import __graft_entry__
    __graft_entry__.load_package()
    from qwen35_dflash_b200 import lib, w4
    hbm, peak_kind = _peaks()
    so = lib.load()
    dev = torch.device("cuda")
    st = torch.cuda.current_stream().cuda_stream
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    lines = []
    # ---- config 2
    H, E, k, I, g = 2048, 256, 8, 512, 128
    gen = torch.Generator(device=dev).manual_seed(0)

    def bank(n, kk, experts):
        q = torch.randint(-8, 8, (experts, n, kk), dtype=torch.int8, device=dev, generator=gen)
        sc = (torch.rand(experts, n, kk // g, device=dev, generator=gen) * 0.015 + 0.005).to(torch.bfloat16)
        return w4.pack_w4(q, sc, g)

    gu, dn = bank(2 * I, H, E), bank(H, I, E)
    sgu, sdn = bank(2 * I, H, 1), bank(H, I, 1)
    w4b = lambda n, kk: n * kk // 2 + n * (kk // g) * 2   # noqa: E731
    per_expert = w4b(2 * I, H) + w4b(H, I)
    dense_default = so.qw_moe_dense_threshold(-1)
    DENSE_ON = 128   # the tensor-core arm: routed experts with >= 128 pairs, when they fill the GPU
    # (tokens, routing): "random" logits N(0, 1); "zipf" adds the per-expert bias log p_e,
    # p_e ~ rank^-1.1 (benchmark config 5's skew); "hot8" adds +4 to 8 experts (every
    # token's routed pairs land on them: all nine slots are dense contractions)
    perm = torch.randperm(E, generator=torch.Generator().manual_seed(3))
    ranks = torch.empty(E)
    ranks[perm] = torch.arange(1, E + 1, dtype=torch.float32)
    zipf = ranks.pow(-1.1)
    zipf = (zipf / zipf.sum()).log().to(dev)
    cases = ((16, "random"), (64, "random"), (256, "random"), (256, "zipf"), (1024, "zipf"), (256, "hot8"))
    if args.moe_case:
        tok, rt = args.moe_case.split(":")
        cases = ((int(tok), rt),)
    for T, routing in cases:
        x = torch.randn(T, H, device=dev, generator=gen).to(torch.bfloat16)
        logits = torch.randn(T, E + 1, device=dev, generator=gen)
        if routing == "zipf":
            logits[:, :E] += zipf
        elif routing == "hot8":
            logits[:, perm[:8].to(dev)] += 4.0
        logits = logits.to(torch.bfloat16)
        ws = torch.zeros(so.qw_moe_workspace_bytes(T, H, E, I, k), dtype=torch.uint8, device=dev)
        out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)

        def moe():
            lib.check(so.qw_moe_route(logits.data_ptr(), lib.QW_BF16, E + 1, T, E, k, E, lib.QW_BF16, ws.data_ptr(), st))
            lib.check(so.qw_moe_experts_w4(x.data_ptr(), gu.data_ptr(), dn.data_ptr(), sgu.data_ptr(), sdn.data_ptr(),
                                           T, H, E, I, k, g, ws.data_ptr(), st))
            lib.check(so.qw_moe_combine(ws.data_ptr(), out.data_ptr(), 0, T, H, E, I, k, 1, st))

        moe()
        torch.cuda.synchronize()
        off = so.qw_moe_active_experts(None, T, E, k)
        active = int(ws[off:off + 4].view(torch.int32).item())
        na = min(E, T * k)   # room of the active list; the pair offsets follow it
        pair_off = ws[off + 4 * (4 + na):off + 4 * (4 + na + active + 1)].view(torch.int32).cpu()
        counts = (pair_off[1:] - pair_off[:-1]).tolist()
        dense = [c for c in counts if T > 16 and c >= DENSE_ON]
        if sum((c + 127) // 128 for c in dense) * (I // 64) < 128:   # the kernels' fill rule
            dense = []
        us = _event_times(moe, args.kernel_reps, flush)
        so.qw_moe_dense_threshold(DENSE_ON)
        us_dense = _event_times(moe, args.kernel_reps, flush) if dense else us
        so.qw_moe_dense_threshold(dense_default)
        nbytes = (active + 1) * per_expert + T * H * 2 * 2 + T * (E + 1) * 2
        lines.append({"config": "2: W4A16 grouped MoE (route + experts + combine)", "tokens": T,
                      "routing": routing, "active_experts": active, "max_pairs": max(counts),
                      "dense_experts": len(dense), "dense_pairs": sum(dense), "us": round(us, 2),
                      "us_tcgen05_dense": round(us_dense, 2), "alg_bytes": nbytes,
                      "achieved_gbs": round(nbytes / us / 1e3, 1), "peak_gbs": hbm,
                      "frac": round(nbytes / us / 1e3 / hbm, 4), "peak_kind": f"{peak_kind} burst copy",
                      "tflops": round(2 * T * 9 * 3 * I * H / us / 1e6, 2)})
    del gu, dn
    if args.moe_case:
        for line in lines:
            print(json.dumps(line), flush=True)
        return
    # ---- config 3
    kh, vh, d, S = 16, 32, 128, 16
    kw, vw = kh * d, vh * d
    C = 2 * kw + vw
    ldp = C + vw
    for B in (1, 8, 32):
        proj = torch.randn(B * S, ldp, device=dev, generator=gen).to(torch.bfloat16)
        ab = torch.randn(B * S, 2 * vh, device=dev, generator=gen)
        hist = torch.randn(B, C, 3, device=dev, generator=gen).to(torch.bfloat16)
        conv_w = (torch.randn(C, 4, device=dev, generator=gen) * 0.02).to(torch.bfloat16)
        a_log = torch.log(torch.arange(1, vh + 1, dtype=torch.float32, device=dev))
        dt_bias = torch.randn(vh, device=dev, generator=gen) * 0.5
        norm_w = torch.ones(d, device=dev).to(torch.bfloat16)
        state = torch.randn(B, vh, d, d, device=dev, generator=gen) * 0.02
        outp = torch.zeros(B * S, vw, dtype=torch.bfloat16, device=dev)
        slots = torch.arange(B, dtype=torch.int32, device=dev)
        accepted = torch.full((B,), S, dtype=torch.int32, device=dev)
        layer = (lib.GdnLayer * 1)()
        layer[0] = lib.GdnLayer(proj.data_ptr(), ab.data_ptr(), hist.data_ptr(), conv_w.data_ptr(), a_log.data_ptr(),
                                dt_bias.data_ptr(), norm_w.data_ptr(), state.data_ptr(), outp.data_ptr())
        desc = torch.frombuffer(bytearray(bytes(memoryview(layer).cast("B"))), dtype=torch.uint8).to(dev)
        dims = lib.GdnDims(B, S, kh, vh, d, d, C, 4, ldp, 1e-6, slots.data_ptr(), accepted.data_ptr())

        def gdn_verify():
            lib.check(so.qw_gdn_verify(ctypes.byref(dims), desc.data_ptr(), 0, st))

        def gdn_both():
            lib.check(so.qw_gdn_verify(ctypes.byref(dims), desc.data_ptr(), 0, st))
            lib.check(so.qw_gdn_commit(ctypes.byref(dims), desc.data_ptr(), 1, st))

        gdn_both()
        torch.cuda.synchronize()
        us_v = _event_times(gdn_verify, args.kernel_reps, flush)
        us_b = _event_times(gdn_both, args.kernel_reps, flush)
        seq_alg = 2 * 2 * vh * d * d + S * C * 2 + 2 * C * 3 * 2 + S * 2 * vh * 4 + 3 * S * vw * 2
        moved = (3 * vh * d * d * 4 + S * ldp * 2 + S * 2 * vh * 4 + 2 * C * 3 * 2 + S * vw * 2)
        lines.append({"config": "3: gated-DeltaNet verify + commit (block 16)", "batch": B,
                      "us_verify": round(us_v, 2), "us_verify_commit": round(us_b, 2),
                      "alg_bytes": B * seq_alg, "bytes_moved": B * moved,
                      "achieved_gbs": round(B * seq_alg / us_b / 1e3, 1), "peak_gbs": hbm,
                      "frac": round(B * seq_alg / us_b / 1e3 / hbm, 4), "peak_kind": f"{peak_kind} burst copy"})
    for line in lines:
        print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=("ours", "reference"))
    ap.add_argument("--ctx", type=int, default=4096)
    ap.add_argument("--batch", type=int, default=1, help="requests per GPU")
    ap.add_argument("--requests", type=int, default=0,
                    help="total requests, split evenly over the GPUs (benchmark config 5: 64)")
    ap.add_argument("--zipf", type=float, default=0.0,
                    help="routing skew: router-logit bias log p_e, p_e ~ rank^-s (benchmark config 5: 1.1)")
    ap.add_argument("--serving", action="store_true",
                    help="benchmark config 5: --requests 64 --ctx 32768 --zipf 1.1")
    ap.add_argument("--replicas", action="store_true",
                    help="with --gpus > 1: run independent replicas instead of sharding the routed experts")
    ap.add_argument("--e2e-steps", type=int, default=30)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--timeline-detail", action="store_true",
                    help="with --timeline: also each launch of decoder layers 4-7 in order")
    ap.add_argument("--timeline", action="store_true",
                    help="after warm-up, print the in-graph kernel timeline of one step (rank 0) and exit")
    ap.add_argument("--profile-step", action="store_true",
                    help="run warm-up then one step inside cudaProfilerStart/Stop and exit (for ncu)")
    ap.add_argument("--kernels", action="store_true",
                    help="per-kernel timings on a 4-layer model of the full width (the small case for ncu)")
    ap.add_argument("--kernel-reps", type=int, default=5)
    ap.add_argument("--micro", action="store_true",
                    help="benchmark configs 2 (W4A16 MoE, T 16/64/256) and 3 (GDN verify, B 1/8/32), one line each")
    ap.add_argument("--dflash", action="store_true",
                    help="time the DFlash step (draft + verify + extend) on the full target and draft (1 GPU)")
    ap.add_argument("--prefill", action="store_true",
                    help="prompt prefill tok/s: 64-token chunks (prefill engine) against 16-token blocks")
    ap.add_argument("--prefill-tokens", type=int, default=2048)
    ap.add_argument("--moe-case", default="",
                    help="with --micro: only this config-2 case, TOKENS:ROUTING (e.g. 256:hot8; the small case for ncu)")
    args = ap.parse_args()
    if args.serving:
        args.requests = args.requests or 64
        args.ctx = 32768 if args.ctx == 4096 else args.ctx
        args.zipf = args.zipf or 1.1
    if args.kernels:
        run_kernels(args)
        return
    if args.micro:
        args.kernel_reps = max(args.kernel_reps, 20)
        run_micro(args)
        return
    if args.prefill:
        run_prefill(args)
        return
    if args.dflash:
        run_dflash(args)
        return
    if args.warmup < 3:
        args.warmup = 3
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if os.environ.get("NCCL_DEBUG", "VERSION").upper() == "VERSION":
        os.environ["NCCL_DEBUG"] = "WARN"   # the version banner would go to stdout, ahead of the JSON line
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        # the CPU reference needs no process group: rank 0 measures, the others exit
        out = run_reference(args, rank, world)
        if out is not None:
            print(json.dumps(out), flush=True)
        return
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(minutes=10),
                                device_id=torch.device("cuda", local_rank))
    try:
        out = run_ours(args, rank, world, local_rank)
        if out is not None and world == 1 and not args.no_cpu_baseline:
            out["cpu_baseline"] = cpu_baseline_leg()
        if out is not None:
            print(json.dumps(out), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
