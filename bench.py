#!/usr/bin/env python3
"""Benchmark of the sm100 MoM hot path (one JSON line on rank 0).

Default workload: the 300M-class Naylis decoder training
step — 20 layers, d=1024, 16x64 heads, SwiGLU 2816, vocab 32000, RoPE, RMSNorm,
a MoM read (fused router + bucketed read on this package's sm_100a kernels) in
every layer sharing one 8x128x1024 bank, router rank 32, top-2, aux 0.01 —
forward + backward + fused AdamW, bf16 autocast with fp32 master weights, on
B=8 x S=2048 token ids per GPU. At N>1 every rank trains its own 8x2048 batch
(weak scaling) and the gradients are averaged by the bucketed NCCL all-reduce
of naylis_b200.data_parallel, launched from the backward's hooks so it
overlaps the backward. The line also carries the MoM read (fwd+bwd) and the
router forward on BASELINE config 2's geometry, timed alone through the C ABI:
the dominant kernels of this library and their rooflines.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl sm100|reference]
                    [--workload cfg3|cfg2|read-top4of32]

``--workload cfg2`` times one MoM layer forward+backward (config 2) as a CUDA
graph; ``read-top4of32`` the read alone on config 4's geometry.
``--impl reference`` times the CPU restatement of the reference's eager path
(oracle/) on this host's cores for the same workload and metric.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CFG = dict(B=8, S=2048, d=1024, H=16, nb=8, bs=128, top=2, r=32)
CFG3 = dict(B=8, S=2048)
METRIC3 = "Naylis 300M decoder training tokens/s (fwd+bwd+AdamW, all GPUs), BASELINE config 3"
WORKLOAD3 = ("cfg3: 20-layer Naylis decoder (d 1024, 16x64 heads, SwiGLU 2816, vocab 32000, RoPE, RMSNorm, "
             "MoM in every layer sharing one 8x128x1024 bank, rank 32, top-2, aux 0.01), B=8 x S=2048 "
             "token ids per GPU, bf16 autocast, fp32 master weights, AdamW")
METRIC = "MoM layer fwd+bwd tokens/s (router + read + projections), BASELINE config 2"
WORKLOAD = ("cfg2: one MoM layer fwd+bwd per GPU, B=8 S=2048 d=1024, 16x64 heads, "
            "bank 8x128 slots, router rank 32, top-2, bf16 autocast, fp32 master weights")

# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum, MB) per launch of every kernel on
# the read path at config 2, medians of one ncu capture (profiles/read_path_dram_bytes_cfg2.md):
# the roofline's traffic figure covers the whole read, bucketing and row passes included.
READ_TRAFFIC_MB = {"bucket (4 kernels)": 1.26, "permute_rows (q -> plan order)": 33.65,
                   "read_fwd_tc": 39.42, "row_delta (dO copy + delta)": 70.24, "read_bwd_dq_tc": 79.93,
                   "read_bwd_dkdv_tc": 86.34}
READ_TRAFFIC_BYTES = sum(READ_TRAFFIC_MB.values()) * 1e6
# Algorithmic bytes of the read fwd + bwd at config 2 (N = 16384 tokens, H*hd = 1024 bf16,
# bank 1024 slots): forward Q + K + V in, O + lse out; backward Q, K, V, O (for delta), dO,
# lse in, dQ, fp32 dK / dV out.
READ_ALGO_BYTES = ((16384 * 2048) * 2 + 4 * 1024 * 1024 + 16384 * 16 * 4
                   + (16384 * 2048) * 4 + 4 * 1024 * 1024 + 16384 * 16 * 4 + 8 * 1024 * 1024)


def read_flops(N, d, top, bs):
    """Algorithmic read FLOPs, active slots only: fwd 4*N*d*La, bwd 8*N*d*La."""
    La = top * bs
    return 4 * N * d * La, 8 * N * d * La


def router_bytes(N, d, nb, top, r, x_bytes=2):
    """Algorithmic router-forward HBM bytes: read x once, write probs, idx
    (int64), gates and the saved activations."""
    return N * d * x_bytes + N * nb * 4 + N * top * 8 + N * top * 4 + N * r * 2


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return dict(hbm=p["hbm_gbs"], bf16=p["bf16_tflops"], bf16_sust=p["bf16_tflops_sustained"],
                    src="measured")
    return dict(hbm=6650.0, bf16=1590.0, bf16_sust=1400.0, src="fallback")


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi samples (200 ms) taken while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.rows = []
        self.proc = None
        self.window = (0.0, 0.0)

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.gpu)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        self._t = threading.Thread(target=self._read, daemon=True)
        self._t.start()

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append((time.time(), [c.strip() for c in line.split(",")]))

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        t0, t1 = self.window
        rows = [r for t, r in self.rows if t0 <= t <= t1] or [r for _, r in self.rows]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        sm = sorted(float(r[1]) for r in rows if r[1].replace(".", "").isdigit())
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for name, val in zip(names, r[5:9]):
                if val.strip().lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": sm[len(sm) // 2] if sm else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "reasons": sorted(reasons), "samples": len(rows)}


# ------------------------------------------------------------------ GPU arm
def run_layer_cfg2(args):
    import torch
    import torch.distributed as dist
    from naylis_b200 import _lib
    from naylis_b200 import mom_kernels as mk
    from naylis_b200.data_parallel import GradAllReduce
    from naylis_b200.model import MoMLayer

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
    c = CFG
    N = c["B"] * c["S"]
    torch.manual_seed(1234 + rank)
    layer = MoMLayer(c["d"], c["H"], c["nb"] * c["bs"], c["bs"], c["top"], c["r"], use_kernel=True)
    with torch.no_grad():
        for p in layer.parameters():
            p.normal_(0.0, 0.02)
        layer.mom_scale.fill_(1.0)
    layer = layer.to(dev).train()
    layer.noise_scale = 1.0
    M = torch.nn.Parameter(torch.randn(c["nb"], c["bs"] * c["d"], device=dev) * 0.02)
    x = torch.randn(c["B"], c["S"], c["d"], device=dev).to(torch.bfloat16).requires_grad_(True)
    # the layer's output is fp32 (bf16 o_proj output times the fp32 mom_scale,
    # model.py:239), so the upstream gradient is fp32 too
    dout = torch.randn(c["B"], c["S"], c["d"], device=dev)

    holder = torch.nn.Module()
    holder.layer = layer
    holder.M = M
    use_graph = not args.no_graph
    # Data parallel: bucketed all-reduces launched from the backward's hooks
    # (overlapping it) when eager; under a CUDA graph they run after each replay
    # (measured faster than capturing them with the backward, --dp-in-graph: the
    # NCCL kernels then share the SMs with the persistent read kernels).
    dp_in_graph = use_graph and args.dp_in_graph
    dp = (GradAllReduce(holder, bucket_mb=args.bucket_mb, overlap=(not use_graph) or dp_in_graph)
          if world > 1 else None)
    mk.resolve_mode(dev, torch.bfloat16, head_dim=c["d"] // c["H"])
    lib = _lib.load()

    def body(xin, gin, with_exchange=False):
        if dp is not None:
            dp.zero_grad()
        else:
            for p in holder.parameters():
                p.grad = None
        xin.grad = None
        with torch.autocast("cuda", dtype=torch.bfloat16):
            out = layer(xin, M)
        out.backward(gin)
        if with_exchange and dp is not None:
            dp.finish()

    def step(xin, gin):
        body(xin, gin)
        if dp is not None:
            dp.finish()

    graph = None
    launches_per_replay = None
    if use_graph:
        # the whole step (zero grads, forward, backward) as one CUDA graph over
        # static x / dout; warm-up on a side stream first, as capture requires
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(3):
                body(x, dout, with_exchange=True)
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        l0 = lib.mom_kernel_launches()
        with torch.cuda.graph(graph):
            body(x, dout, with_exchange=dp_in_graph)
        launches_per_replay = lib.mom_kernel_launches() - l0

        def step(xin, gin):
            assert xin is x and gin is dout, "the graphed step reads the static x / dout"
            graph.replay()
            if dp is not None and not dp_in_graph:
                dp.finish()

    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)   # 256 MiB > L2
    for _ in range(args.warmup):
        step(x, dout)
    torch.cuda.synchronize()

    clocks = ClockSampler(local) if rank == 0 else None
    if clocks:
        clocks.start()
        time.sleep(0.5)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    launches0 = lib.mom_kernel_launches()
    t_wall0 = time.time()
    for i in range(args.steps):
        flush.fill_(float(i))                       # evict L2 between timed steps (untimed)
        starts[i].record()
        step(x, dout)
        ends[i].record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t_wall1 = time.time()
    launches = lib.mom_kernel_launches() - launches0
    if graph is not None:
        # replays launch the captured kernels without passing through the
        # host-side counter: count what one capture launched, per replay
        launches = launches_per_replay * args.steps
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    total_ms = sum(step_ms)
    if clocks:
        clocks.window = (t_wall0, t_wall1)
    if world > 1:
        t = torch.tensor([total_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
    tokens_per_s = world * N * args.steps / (total_ms / 1e3)

    # ---- dominant kernels: the read (fwd + bwd) and the router, on this rank's data
    extra = {}
    if rank == 0:
        extra = measure_kernels(layer, x, M, dout, dev, args)
    # ---- end to end through the public API with host buffers
    e2e = measure_e2e(step, x, dout, dev, args, world, N)
    if clocks:
        clocks.stop()
    if rank == 0:
        pk = peaks()
        roof = extra["read"]
        line = {
            "metric": METRIC,
            "value": round(tokens_per_s, 1),
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(total_ms / args.steps, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) activations, N(0,0.02) weights and bank)",
            "config": {"workload": WORKLOAD, "global_batch": c["B"] * world, "seq_len": c["S"],
                       "parallelism": f"dp{world}", "l2": "flushed between timed steps (256 MiB write, untimed)",
                       "cuda_graph": ("fwd+bwd captured once, replayed per step"
                                      + (("; bucket all-reduces captured with the backward"
                                          if dp_in_graph else "; bucket all-reduce after replay")
                                         if world > 1 else ""))
                       if graph is not None else "off (eager launches)"},
            "roofline": {"bound": "tensor", "achieved": roof["tflops"], "peak": pk["bf16"],
                         "unit": "TFLOP/s", "frac": round(roof["tflops"] / pk["bf16"], 4),
                         "traffic": READ_TRAFFIC_BYTES,
                         "traffic_note": ("dram__bytes_read.sum + dram__bytes_write.sum summed over every kernel "
                                          "of the read path on config 2 (ncu medians, MB): "
                                          + ", ".join(f"{k} {v}" for k, v in READ_TRAFFIC_MB.items())),
                         "algorithmic_bytes": READ_ALGO_BYTES,
                         "traffic_over_algorithmic": round(READ_TRAFFIC_BYTES / READ_ALGO_BYTES, 2),
                         "kernel": "MoM read fwd+bwd (bucket + fwd + dq + dkdv)",
                         "flops_per_launch": roof["flops"], "ms_per_launch": roof["ms"],
                         "peak_source": f"{pk['src']} bf16 burst (MEASURED_PEAKS.json bf16_tflops)"},
            "router": extra["router"],
            "read": roof,
            "e2e": e2e,
            "gpu_launches": int(launches),
            "gpu_launches_per_step": round(launches / args.steps, 2),
            "clocks": clocks.summary() if clocks else None,
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(samples=args.cpu_samples)
        print(json.dumps(line), flush=True)
    del graph
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_model_cfg3(args):
    """the decoder's training step on every GPU."""
    import torch
    import torch.distributed as dist
    from naylis_b200 import _lib
    from naylis_b200.data_parallel import GradAllReduce
    from naylis_b200.decoder import NaylisConfig, NaylisForCausalLM, flops_per_token, param_count

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    B, S = CFG3["B"], CFG3["S"]
    cfg = NaylisConfig()
    torch.manual_seed(1234)                       # every replica starts from the same weights
    model = NaylisForCausalLM(cfg).to(dev).train()
    comm = torch.bfloat16 if args.bf16_grads else None
    # the step as one CUDA graph, the buckets exchanged by finish() after each replay
    # (measured at 2 GPUs: faster than the eager step whose hooks overlap the all-reduces
    # with the backward); --no-graph launches eagerly with that overlap
    use_graph = not args.no_graph
    dp = GradAllReduce(model, bucket_mb=args.bucket_mb, comm_dtype=comm, overlap=not use_graph)
    if args.optim == "torch":
        opt = torch.optim.AdamW(model.parameters(), lr=3e-4, weight_decay=0.1, fused=True)
    else:
        # one launch over every parameter, writing the bf16 weight copies the next forward reads
        from naylis_b200.optim import AdamW
        opt = AdamW(model.parameters(), lr=3e-4, weight_decay=0.1)
    g = torch.Generator(device=dev).manual_seed(77 + rank)
    ids = torch.randint(0, cfg.vocab_size, (B, S), device=dev, generator=g)
    lib = _lib.load()

    gstep = None
    if use_graph:
        # zero_grad + forward + loss + backward as one CUDA graph (the public helper)
        from naylis_b200.graph_step import GraphedTrainStep
        gstep = GraphedTrainStep(model, dp, ids)

    def step(batch):
        if gstep is not None:
            loss = gstep.step(None if batch is ids else batch)
            opt.step()
            return loss
        dp.zero_grad()
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = model(batch, labels=batch)
        loss.backward()
        dp.finish()
        opt.step()
        return loss

    for _ in range(args.warmup):
        step(ids)
    torch.cuda.synchronize()
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    clocks = ClockSampler(local) if rank == 0 else None
    if clocks:
        clocks.start()
        time.sleep(0.5)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    l0 = lib.mom_kernel_launches()
    t_wall0 = time.time()
    for i in range(args.steps):
        flush.fill_(float(i))                     # evict L2 between timed steps (untimed)
        starts[i].record()
        step(ids)
        ends[i].record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t_wall1 = time.time()
    launches = lib.mom_kernel_launches() - l0
    if gstep is not None:
        launches += gstep.kernels_per_replay * args.steps    # replayed, not counted by the host
    each_ms = sorted(a.elapsed_time(b) for a, b in zip(starts, ends))
    total_ms = sum(each_ms)
    if clocks:
        clocks.window = (t_wall0, t_wall1)
    if world > 1:
        t = torch.tensor([total_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
    tokens_per_s = world * B * S * args.steps / (total_ms / 1e3)

    # end to end through the public API: the token ids travel from pinned host
    # memory every step, the loss comes back every step
    ids_host = ids.cpu().pin_memory()
    loss_host = torch.empty(max(1, min(args.steps, 20)), dtype=torch.float32).pin_memory()
    dev_ids = torch.empty_like(ids)
    n_e2e = loss_host.numel()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    for i in range(n_e2e):
        if gstep is not None:
            loss = step(ids_host)                 # copied from pinned host memory into the graph's input
        else:
            dev_ids.copy_(ids_host, non_blocking=True)
            loss = step(dev_ids)
        loss_host[i:i + 1].copy_(loss.detach().float().reshape(1), non_blocking=True)
    b.record()
    torch.cuda.synchronize()
    e2e_ms = a.elapsed_time(b)
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e = {"value": round(world * B * S * n_e2e / (e2e_ms / 1e3), 1), "unit": "tokens/s",
           "h2d_bytes_per_step": ids_host.numel() * ids_host.element_size(), "d2h_bytes_per_step": 4,
           "loss_last": round(float(loss_host[-1]), 4)}

    extra = {}
    if rank == 0:
        layer, x, M, dout = cfg2_layer_inputs(dev)
        extra = measure_kernels(layer, x, M, dout, dev, args)
    if clocks:
        clocks.stop()
    if rank == 0:
        pk = peaks()
        roof = extra["read"]
        fpt = 3 * flops_per_token(cfg, S, B * S)
        per_gpu = tokens_per_s / world
        line = {
            "metric": METRIC3,
            "value": round(tokens_per_s, 1),
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(total_ms / args.steps, 3),
            "step_ms_rank0": {"min": round(each_ms[0], 3), "median": round(each_ms[len(each_ms) // 2], 3),
                              "max": round(each_ms[-1], 3)},
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (token ids uniform in [0, 32000), seeded per rank; random-init weights as the "
                    "reference initialises them)",
            "config": {"workload": WORKLOAD3, "global_batch": B * world, "seq_len": S, "parallelism": f"dp{world}",
                       "params": param_count(model),
                       "l2": "flushed between timed steps (256 MiB write, untimed); the step's working set "
                             "(weights, optimizer state, activations) is far above L2 as well",
                       "grad_exchange": (f"bucketed NCCL AVG all-reduce ({args.bucket_mb:g} MiB buckets, "
                                         f"{'bf16' if comm is not None else 'fp32'} on the wire) "
                                         + ("after each graph replay" if use_graph else
                                            "launched from the backward's hooks")
                                         if world > 1 else "none (one GPU)"),
                       "cuda_graph": ("zero_grad + forward + loss + backward replayed as one CUDA graph "
                                      "(naylis_b200.graph_step.GraphedTrainStep); AdamW and the exchange outside"
                                      if use_graph else "none (eager launches)")},
            "tokens_per_s_per_gpu": round(per_gpu, 1),
            "model_flops_per_token": fpt,
            "mfu": round(per_gpu * fpt / (pk["bf16_sust"] * 1e12), 4),
            "mfu_peak": f"{pk['src']} bf16 sustained {pk['bf16_sust']} TFLOP/s (MEASURED_PEAKS.json)",
            "roofline": {"bound": "tensor", "achieved": roof["tflops"], "peak": pk["bf16"],
                         "unit": "TFLOP/s", "frac": round(roof["tflops"] / pk["bf16"], 4),
                         "traffic": READ_TRAFFIC_BYTES,
                         "traffic_note": ("dram__bytes_read.sum + dram__bytes_write.sum summed over every kernel "
                                          "of the read path on config 2 (ncu medians, MB): "
                                          + ", ".join(f"{k} {v}" for k, v in READ_TRAFFIC_MB.items())),
                         "algorithmic_bytes": READ_ALGO_BYTES,
                         "traffic_over_algorithmic": round(READ_TRAFFIC_BYTES / READ_ALGO_BYTES, 2),
                         "kernel": "MoM read fwd+bwd on BASELINE config 2 (bucket + fwd + dq + dkdv), C ABI",
                         "flops_per_launch": roof["flops"], "ms_per_launch": roof["ms"],
                         "peak_source": f"{pk['src']} bf16 burst (MEASURED_PEAKS.json bf16_tflops)"},
            "router": extra["router"],
            "read": roof,
            "e2e": e2e,
            "gpu_launches": int(launches),
            "gpu_launches_per_step": round(launches / args.steps, 1),
            "clocks": clocks.summary() if clocks else None,
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline_model(args)
        print(json.dumps(line), flush=True)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def cfg2_layer_inputs(dev, seed=4321):
    """A config-2 MoM layer (N(0, 0.02) weights, bank and mom_scale 1), x and
    an upstream gradient, for timing the library's kernels on their own."""
    import torch
    from naylis_b200.model import MoMLayer
    c = CFG
    torch.manual_seed(seed)
    layer = MoMLayer(c["d"], c["H"], c["nb"] * c["bs"], c["bs"], c["top"], c["r"])
    with torch.no_grad():
        for p in layer.parameters():
            p.normal_(0.0, 0.02)
        layer.mom_scale.fill_(1.0)
    layer = layer.to(dev)
    M = torch.randn(c["nb"], c["bs"] * c["d"], device=dev) * 0.02
    x = torch.randn(c["B"], c["S"], c["d"], device=dev).to(torch.bfloat16)
    dout = torch.randn(c["B"], c["S"], c["d"], device=dev)
    return layer, x, M, dout


def measure_kernels(layer, x, M, dout, dev, args):
    """CUDA-event timing of the read and the router through the C ABI, on the
    launching (current) stream, L2 flushed between iterations."""
    import torch
    from naylis_b200 import _lib
    from naylis_b200 import mom_kernels as mk
    c = CFG
    B, S, d, H, nb, bs, top, r = (c[k] for k in ("B", "S", "d", "H", "nb", "bs", "top", "r"))
    hd = d // H
    N = B * S
    lib = _lib.load()

    def cur():   # the launching stream, looked up at call time (a capture switches it)
        return torch.cuda.current_stream(dev).cuda_stream

    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        probs, idx, gates = mk.mom_route(x, layer.router_down.weight, layer.router_up.weight, top)
        q = layer.q_proj(x).view(B, S, H, hd).contiguous()
        slots = M.view(nb * bs, d)
        k = layer.k_proj(slots).contiguous()
        v = layer.v_proj(slots).contiguous()
    lg = gates.clamp_min(1e-9).log().float().contiguous()
    plan = torch.empty(lib.mom_plan_size(N, nb, top), dtype=torch.uint8, device=dev)
    out = torch.empty_like(q)
    lse = torch.empty(H, N, dtype=torch.float32, device=dev)
    q_rows = torch.empty(N, d, dtype=torch.bfloat16, device=dev)
    dq = torch.empty_like(q)
    dk = torch.empty(nb * bs, d, dtype=torch.float32, device=dev)
    dv = torch.empty_like(dk)
    dlg = torch.empty(N, top, dtype=torch.float32, device=dev)
    ws = torch.empty(lib.mom_read_bwd_workspace_size(B, S, H, hd), dtype=torch.uint8, device=dev)
    do4 = dout.to(torch.bfloat16).view(B, S, H, hd)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)

    def read_once():
        st = cur()
        _lib.call("mom_bucket", idx.data_ptr(), _lib.I64, lg.data_ptr(), N, nb, top, plan.data_ptr(),
                  plan.numel(), st)
        _lib.call("mom_read_fwd", q.data_ptr(), k.data_ptr(), v.data_ptr(), _lib.BF16, B, S, H, hd, nb,
                  bs, top, plan.data_ptr(), out.data_ptr(), lse.data_ptr(), q_rows.data_ptr(), st)
        _lib.call("mom_read_bwd", q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                  do4.data_ptr(), lse.data_ptr(), _lib.BF16, B, S, H, hd, nb, bs, top, plan.data_ptr(),
                  q_rows.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), dlg.data_ptr(),
                  ws.data_ptr(), ws.numel(), st)

    xb = x.detach().contiguous()
    wd = layer.router_down.weight.detach().to(torch.bfloat16).contiguous()
    wu = layer.router_up.weight.detach().to(torch.bfloat16).contiguous()
    probs_o = torch.empty(N, nb, dtype=torch.float32, device=dev)
    idx_o = torch.empty(N, top, dtype=torch.int64, device=dev)
    gates_o = torch.empty(N, top, dtype=torch.float32, device=dev)
    act_o = torch.empty(N, r, dtype=torch.bfloat16, device=dev)
    rws = torch.empty(lib.mom_route_workspace_size(B, S, d, r, nb, _lib.BF16), dtype=torch.uint8, device=dev)

    def route_once(mode=_lib.SCAN_MODES["fp32"]):
        _lib.call("mom_route_fwd", xb.data_ptr(), _lib.BF16, B, S, d, wd.data_ptr(), wu.data_ptr(),
                  _lib.BF16, r, nb, top, None, mode, probs_o.data_ptr(), idx_o.data_ptr(), _lib.I64,
                  gates_o.data_ptr(), None, act_o.data_ptr(), rws.data_ptr(), rws.numel(), cur())

    def timed(fn, iters):
        """One call captured in a CUDA graph (the entry points only launch kernels
        on the stream they are given), replayed per timed iteration after an L2
        flush: the host's launch cost stays outside the events."""
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(3):
                fn()
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            fn()
        for _ in range(3):
            graph.replay()
        times = []
        for i in range(iters):
            flush.fill_(float(i))
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record()
            graph.replay()
            b.record()
            times.append((a, b))
        torch.cuda.synchronize()
        del graph
        return sum(a.elapsed_time(b) for a, b in times) / iters

    iters = max(10, min(100, args.steps))
    t_read = timed(read_once, iters)
    t_route = timed(route_once, iters)
    t_route64 = timed(lambda: route_once(_lib.SCAN_MODES["fp64"]), iters)
    fwd_f, bwd_f = read_flops(N, d, top, bs)
    rb = router_bytes(N, d, nb, top, r)
    pk = peaks()
    return {
        "read": {"ms": round(t_read, 4), "flops": fwd_f + bwd_f,
                 "tflops": round((fwd_f + bwd_f) / (t_read / 1e3) / 1e12, 2),
                 "tokens_per_s": round(N / (t_read / 1e3), 1)},
        "router": {"ms": round(t_route, 4), "bytes": rb,
                   "gbs": round(rb / (t_route / 1e3) / 1e9, 1),
                   "frac_of_hbm": round(rb / (t_route / 1e3) / 1e9 / pk["hbm"], 4),
                   "hbm_peak_gbs": pk["hbm"], "scan_mode": "fp32 (torch CUDA cumsum; the layer default)",
                   "fp64_scan_ms": round(t_route64, 4)},
    }


def measure_e2e(step, x, dout, dev, args, world, N):
    """The same step through the public API with host buffers: every step copies
    its inputs (x, upstream grad) from pinned host memory and its dx back, all
    inside the timed region. The copies are pipelined across steps as a training
    input pipeline would run them: step i+1's inputs travel host -> device on
    one copy stream (into one of two device staging slots) while step i
    computes, and step i's dx travels back on another; the compute stream moves
    a staged slot into the step's own input buffers on the device (static under
    a CUDA graph) and dx out of the step's gradient buffer."""
    import torch
    import torch.distributed as dist
    xh = x.detach().cpu().pin_memory()
    gh = dout.cpu().pin_memory()
    dxh = [torch.empty_like(xh).pin_memory() for _ in range(2)]
    xd, gd = x, dout          # the step's own device input buffers
    xs = [torch.empty_like(xd) for _ in range(2)]
    gs = [torch.empty_like(gd) for _ in range(2)]
    dxs = [torch.empty_like(xd) for _ in range(2)]
    comp = torch.cuda.current_stream()
    h2d = torch.cuda.Stream(device=dev)
    d2h = torch.cuda.Stream(device=dev)
    ev = lambda: [torch.cuda.Event() for _ in range(2)]
    in_ready, in_free, out_ready, out_free = ev(), ev(), ev(), ev()
    iters = max(5, min(50, args.steps))

    def load(i):              # step i's inputs -> staging slot i % 2
        k = i % 2
        with torch.cuda.stream(h2d):
            h2d.wait_event(in_free[k])                # the slot's previous inputs were moved out
            xs[k].copy_(xh, non_blocking=True)
            gs[k].copy_(gh, non_blocking=True)
            in_ready[k].record(h2d)

    def run(i):
        k = i % 2
        comp.wait_event(in_ready[k])
        with torch.no_grad():
            xd.copy_(xs[k])
            gd.copy_(gs[k])
        in_free[k].record(comp)
        step(xd, gd)
        comp.wait_event(out_free[k])                  # the slot's previous dx reached the host
        with torch.no_grad():
            dxs[k].copy_(xd.grad)
        out_ready[k].record(comp)
        with torch.cuda.stream(d2h):
            d2h.wait_event(out_ready[k])
            dxh[k].copy_(dxs[k], non_blocking=True)
            out_free[k].record(d2h)

    def steps(n, start_ev=None):
        if start_ev is not None:
            h2d.wait_event(start_ev)
        load(0)
        for i in range(n):
            if i + 1 < n:
                load(i + 1)
            run(i)
        comp.wait_stream(d2h)                         # the last dx is on the host

    steps(2)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record(comp)
    steps(iters, start_ev=a)
    b.record(comp)
    torch.cuda.synchronize()
    ms = a.elapsed_time(b)
    if world > 1:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return {"value": round(world * N * iters / (ms / 1e3), 1), "unit": "tokens/s",
            "h2d_bytes_per_step": xh.numel() * xh.element_size() + gh.numel() * gh.element_size(),
            "d2h_bytes_per_step": dxh[0].numel() * dxh[0].element_size(),
            "copies": "pipelined across steps (separate host->device and device->host streams)"}


# ------------------------------------------------------------------ CPU arms
def _cpu_step_inputs(S_sample):
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
    import golden_inputs as gi
    import mom_oracle as O
    c = CFG
    geo = dict(B=1, S=S_sample, d=c["d"], H=c["H"], nb=c["nb"], bs=c["bs"], top=c["top"], r=c["r"],
               seed=0, x_std=1.0, m_std=0.02, w_std=0.02, mom_scale=1.0)
    inp = gi.layer_inputs(geo)
    return O, inp["x"].numpy(), gi.oracle_params(inp, geo), gi.upstream_grad(geo).numpy()


def cpu_baseline(samples=3, S_sample=2048):
    """The oracle port of the reference's eager layer step (fp32, dense over
    all L slots) on this host's cores, a bounded sample of the workload."""
    O, x, P, g = _cpu_step_inputs(S_sample)
    c = CFG
    O.layer_step_fp32(x, P, g, c["H"], c["nb"], c["bs"], c["top"])   # warm-up
    t = time.perf_counter()
    for _ in range(samples):
        O.layer_step_fp32(x, P, g, c["H"], c["nb"], c["bs"], c["top"])
    dt = (time.perf_counter() - t) / samples
    return {"value": round(S_sample / dt, 1), "unit": "tokens/s", "cores": os.cpu_count(),
            "kind": "port",
            "sample": f"{samples} x one 1x{S_sample}-token sequence of the cfg2 layer, fwd+bwd, fp32 numpy "
                      f"(oracle/mom_oracle.py layer_step_fp32; BLAS threads = all cores)"}


CPU_SAMPLE3 = dict(B=1, S=512)


def _decoder_oracle():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import decoder_oracle as D
    return D


def cpu_baseline_model(args, samples=3):
    """The oracle's CPU restatement of the reference's decoder training step
    (fwd + bwd + AdamW, fp32, config-3 architecture) on this host's cores, a
    bounded sample of the workload: one 1 x 512-token sequence per step."""
    import torch
    D = _decoder_oracle()
    threads = os.cpu_count()
    torch.set_num_threads(threads)
    B, S = CPU_SAMPLE3["B"], CPU_SAMPLE3["S"]
    step = D.train_step_timer(D.CONFIG3, B, S, threads=threads)
    step()                                            # warm-up
    t = time.perf_counter()
    for _ in range(samples):
        step()
    dt = (time.perf_counter() - t) / samples
    return {"value": round(B * S / dt, 1), "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{samples} steps of one {B}x{S}-token sequence: the config-3 decoder (20 layers, d 1024, "
                      f"vocab 32000) fwd + bwd + AdamW in fp32 torch on the host (oracle/decoder_oracle.py, "
                      f"pinned to the reference's NaylisLlamaForCausalLM)"}


def run_reference_model(args):
    """--impl reference for config 3: the CPU restatement of the reference's
    training step, timed on this host's cores, --warmup then --steps steps of a
    bounded sample (one 1 x 512-token sequence per step). Rank 0 only."""
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    D = _decoder_oracle()
    threads = os.cpu_count()
    torch.set_num_threads(threads)
    B, S = CPU_SAMPLE3["B"], CPU_SAMPLE3["S"]
    step = D.train_step_timer(D.CONFIG3, B, S, threads=threads)
    for _ in range(args.warmup):
        step()
    t = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t) / args.steps
    val = round(B * S / dt, 1)
    sample = (f"one {B}x{S}-token sequence per step: the config-3 decoder fwd + bwd + AdamW in fp32 torch on the "
              f"host (oracle/decoder_oracle.py, the CPU restatement pinned to the reference's "
              f"NaylisLlamaForCausalLM)")
    print(json.dumps({
        "impl": "reference", "metric": METRIC3, "value": val, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 2), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD3, "global_batch": B, "seq_len": S, "parallelism": "cpu",
                   "sample_of": f"{CFG3['B']}x{CFG3['S']} tokens per GPU"},
        "cpu_baseline": {"value": val, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": val, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    S_sample = 2048
    O, x, P, g = _cpu_step_inputs(S_sample)
    c = CFG
    for _ in range(args.warmup):
        O.layer_step_fp32(x, P, g, c["H"], c["nb"], c["bs"], c["top"])
    steps = args.steps
    t = time.perf_counter()
    for _ in range(steps):
        O.layer_step_fp32(x, P, g, c["H"], c["nb"], c["bs"], c["top"])
    dt = (time.perf_counter() - t) / steps
    val = round(S_sample / dt, 1)
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": val, "unit": "tokens/s", "n_gpus": world,
        "steps": steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 2),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": {"workload": WORKLOAD, "global_batch": 1, "seq_len": S_sample,
                                        "parallelism": "cpu"},
        "cpu_baseline": {"value": val, "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
                         "sample": f"one 1x{S_sample}-token sequence per step (the reference's eager "
                                   f"layer math restated in fp32 numpy, oracle/mom_oracle.py)"},
        "e2e": {"value": val, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# ------------------------------------------------------------------ decoder trunk kernels
def run_trunk(args):
    """The decoder trunk's fused kernels (csrc/trunk.cu) alone at BASELINE
    config 3's sizes (B=8 x S=2048 tokens, d=1024, 16x64 heads, SwiGLU 2816),
    each timed with CUDA events on the launching stream over --steps calls
    after --warmup, L2 flushed before each call; achieved = algorithmic bytes
    (each input read once, each output written once) / time, against the
    measured HBM copy bandwidth. These kernels move bytes only."""
    import torch
    from naylis_b200 import _lib
    from naylis_b200.decoder import rope_tables
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    B, S, d, H, f = CFG3["B"], CFG3["S"], 1024, 16, 2816
    hd, N = d // H, B * S
    g = torch.Generator(device=dev).manual_seed(5)
    bf = torch.bfloat16
    qkv = torch.randn(N, 3 * d, generator=g, device=dev).to(bf)
    q, k, v = (torch.empty(N, d, dtype=bf, device=dev) for _ in range(3))
    dqkv = torch.empty_like(qkv)
    cos, sin = rope_tables(S, hd, 500000.0, dev)
    gu = torch.randn(N, 2 * f, generator=g, device=dev).to(bf)
    h = torch.empty(N, f, dtype=bf, device=dev)
    dh = torch.randn(N, f, generator=g, device=dev).to(bf)
    dgu = torch.empty_like(gu)
    x = torch.randn(N, d, generator=g, device=dev)
    delta = torch.randn(N, d, generator=g, device=dev).to(bf)
    w = torch.ones(d, device=dev)
    x_out, dx_in, dx = (torch.empty(N, d, device=dev) for _ in range(3))
    y16, ddelta, dy16 = (torch.empty(N, d, dtype=bf, device=dev) for _ in range(3))
    dy16.normal_()
    dx_in.normal_()
    rstd = torch.empty(N, device=dev)
    dw = torch.empty(d, device=dev)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    st = lambda: torch.cuda.current_stream(dev).cuda_stream
    ops = {
        "rope_qkv_fwd": (lambda: _lib.call("mom_rope_qkv_fwd", qkv.data_ptr(), cos.data_ptr(), sin.data_ptr(), B, S,
                                           H, hd, q.data_ptr(), k.data_ptr(), v.data_ptr(), st()), 6 * N * d * 2),
        "rope_qkv_bwd": (lambda: _lib.call("mom_rope_qkv_bwd", q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                           cos.data_ptr(), sin.data_ptr(), B, S, H, hd, dqkv.data_ptr(), st()),
                         6 * N * d * 2),
        "swiglu_fwd": (lambda: _lib.call("mom_swiglu_fwd", gu.data_ptr(), N, f, h.data_ptr(), st()), 3 * N * f * 2),
        "swiglu_bwd": (lambda: _lib.call("mom_swiglu_bwd", dh.data_ptr(), gu.data_ptr(), N, f, dgu.data_ptr(), st()),
                       5 * N * f * 2),
        "add_rmsnorm_fwd": (lambda: _lib.call("mom_add_rmsnorm_fwd", x.data_ptr(), delta.data_ptr(), _lib.BF16, None,
                                              w.data_ptr(), N, d, 1e-5, x_out.data_ptr(), y16.data_ptr(), None,
                                              rstd.data_ptr(), st()), N * d * 12),
        "add_rmsnorm_bwd": (lambda: _lib.call("mom_add_rmsnorm_bwd", x_out.data_ptr(), rstd.data_ptr(), w.data_ptr(),
                                              delta.data_ptr(), _lib.BF16, None, dy16.data_ptr(), None,
                                              dx_in.data_ptr(), N, d, dx.data_ptr(), ddelta.data_ptr(),
                                              dw.data_ptr(), None, st()), N * d * 16),
    }
    pk = peaks()
    res = {}
    for name, (fn, nbytes) in ops.items():
        for _ in range(args.warmup):
            fn()
        ev = []
        for i in range(args.steps):
            flush.fill_(float(i))
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            ev.append((a, b))
        torch.cuda.synchronize()
        us = sum(a.elapsed_time(b) for a, b in ev) / args.steps * 1e3
        gbs = nbytes / (us / 1e6) / 1e9
        res[name] = {"us": round(us, 2), "bytes": nbytes, "gbs": round(gbs, 1), "frac_of_hbm": round(gbs / pk["hbm"], 4)}
    print(json.dumps({"metric": "decoder trunk kernels, achieved HBM GB/s (BASELINE config 3 sizes)",
                      "unit": "GB/s", "steps": args.steps, "warmup": args.warmup, "kernels": res,
                      "hbm_peak_gbs": pk["hbm"], "peak_source": pk["src"],
                      "config": {"workload": "trunk: N=16384 tokens, d=1024, 16x64 heads, SwiGLU 2816, bf16",
                                 "l2": "flushed before each call (256 MiB write, untimed)"}}), flush=True)


# ------------------------------------------------------------------ config-4 read
CFG4 = dict(B=4, S=4096, H=16, hd=128, nb=32, bs=128, top=4)
METRIC4 = "MoM read fwd+bwd tokens/s, BASELINE config 4 geometry (top-4 of 32 blocks, 16x128 heads)"


def run_read_top4of32(args):
    """The read alone on BASELINE config 4's geometry (configs[3]: x [4, 4096], 16 heads of
    128, bank 32 x 128 slots, top-4): 35,960 block sets, so the door takes the
    block-split read. One step = mom_read forward + backward through the door
    on resident inputs, L2 flushed before each timed step."""
    import torch
    from naylis_b200 import _lib
    from naylis_b200 import mom_kernels as mk
    c = CFG4
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(1234)
    B, S, H, hd, nb, bs, top = c["B"], c["S"], c["H"], c["hd"], c["nb"], c["bs"], c["top"]
    q = (torch.randn(B, S, H, hd, generator=g, device=dev) * 0.7).bfloat16().requires_grad_(True)
    k = (torch.randn(nb * bs, H * hd, generator=g, device=dev) * 0.4).bfloat16().requires_grad_(True)
    v = (torch.randn(nb * bs, H * hd, generator=g, device=dev) * 0.4).bfloat16().requires_grad_(True)
    gates = torch.softmax(torch.randn(B, S, top, generator=g, device=dev), -1).requires_grad_(True)
    idx = torch.argsort(torch.rand(B, S, nb, generator=g, device=dev), -1)[..., :top]
    dout = torch.randn(B, S, H, hd, generator=g, device=dev).bfloat16()
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    lib = _lib.load()

    def step():
        for t in (q, k, v, gates):
            t.grad = None
        out = mk.mom_read(q, k, v, idx, gates, num_blocks=nb, block_size=bs)
        out.backward(dout)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    clocks = ClockSampler(0)
    clocks.start()
    t_wall0 = time.time()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    l0 = lib.mom_kernel_launches()
    for i in range(args.steps):
        flush.zero_()
        starts[i].record()
        step()
        ends[i].record()
    torch.cuda.synchronize()
    launches = lib.mom_kernel_launches() - l0
    clocks.window = (t_wall0, time.time())
    clocks.stop()
    total_ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends))
    N = B * S
    fwd_flops, bwd_flops = read_flops(N, H * hd, top, bs)   # over the selected blocks only
    flops = fwd_flops + bwd_flops
    ms = total_ms / args.steps
    pk = peaks()
    tflops = flops / (ms / 1e3) / 1e12
    print(json.dumps({
        "metric": METRIC4, "value": round(N / (ms / 1e3), 1), "unit": "tokens/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) q/k/v scaled 0.7/0.4/0.4, random distinct top-4 blocks, softmax gates)",
        "config": {"workload": "cfg4-read: mom_read fwd+bwd, B=4 S=4096, 16x128 heads, bank 32x128 slots, top-4 "
                               "(block-split read)", "l2": "flushed between timed steps (256 MiB write, untimed)"},
        "roofline": {"bound": "tensor", "achieved": round(tflops, 2), "peak": pk["bf16"], "unit": "TFLOP/s",
                     "frac": round(tflops / pk["bf16"], 4), "traffic": None,
                     "kernel": "MoM read fwd+bwd, block-split (bucket, row passes, fwd, dq, dkdv, combine)",
                     "peak_source": f"{pk['src']} bf16 burst (MEASURED_PEAKS.json bf16_tflops)"},
        "gpu_launches": int(launches), "clocks": clocks.summary(),
    }), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="sm100", choices=["sm100", "reference"])
    ap.add_argument("--cpu-samples", type=int, default=3)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-graph", action="store_true", help="launch the step eagerly, no CUDA graph")
    ap.add_argument("--dp-in-graph", action="store_true",
                    help="N>1 with a graph: capture the bucket all-reduces with the backward")
    ap.add_argument("--bucket-mb", type=float, default=32.0, help="gradient bucket size for N>1 (MiB)")
    ap.add_argument("--optim", default="naylis", choices=["naylis", "torch"],
                    help="cfg3 optimizer: this package's one-launch AdamW (default) or torch's fused AdamW")
    ap.add_argument("--workload", default="cfg3", choices=["cfg3", "cfg2", "read-top4of32", "trunk"],
                    help="cfg3: the decoder training step (default); cfg2: one MoM layer step; "
                         "read-top4of32: the read alone on config 4's geometry; trunk: the decoder's fused "
                         "trunk kernels alone")
    ap.add_argument("--bf16-grads", action="store_true", help="N>1: all-reduce the gradient buckets in bf16")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference_model(args) if args.workload == "cfg3" else run_reference(args)
    elif args.workload == "read-top4of32":
        run_read_top4of32(args)
    elif args.workload == "trunk":
        run_trunk(args)
    elif args.workload == "cfg2":
        run_layer_cfg2(args)
    else:
        run_model_cfg3(args)


if __name__ == "__main__":
    main()
