#!/usr/bin/env python
"""lfm2moe MoE-FFN throughput on B200 (tokens/s), against the reference CPU path.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--config C] [--impl ours|reference]

A step is one MoE-FFN layer forward over one batch of T tokens (config 2 by
default: the T=8 speculative-verify batch, D=2048, E=32, top-4, I=1792, Q4_K
experts).  Weights are generated on the device from the seeded synthetic
generator.  Consecutive steps cycle through a ring of distinct layers whose
weights total more than the 126 MB L2, so no step re-reads weights the
previous steps left in L2.

Printed JSON (one line, rank 0):
  value      tokens/s over all ranks, inputs resident in HBM, device-timed (CUDA
             events on the launch stream, max over ranks);
  e2e        the same metric through the public host-buffer API
             (lfm_gpu_moe_forward with host x: H2D + layer + D2H per step);
  roofline   the dominant kernel's algorithmic bytes per launch / its mean
             event-timed duration, against MEASURED_PEAKS.json's HBM copy rate;
  cpu_baseline  the reference's own CPU path (oracle/_ref, built from the
             reference sources) on this host's cores, on a bounded sample.
Multi-GPU (torchrun): each rank runs its own replica of the step on its own
tokens ("scaling": "weak"); no collective is on the data path yet.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

Q4K = 144
METRIC = "MoE-FFN tok/s: decode %HBM roofline, prefill %int8 TC peak, 1/2/4/8 B200"


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "src": "fallback"}


class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.lines = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "--query-gpu=" + self.FIELDS, "--format=csv,noheader,nounits",
                                          "-lms", "100", "-i", str(self.device)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except (OSError, ValueError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_setup():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def config_dict(cfg_id, cfg, ring, extra=None):
    experts = "Q4_K gate/up and Q6_K down experts" if cfg.get("down_q6k") else "Q4_K experts"
    d = {"workload": f"cfg{cfg_id}: {cfg['name']} (lfm2moe FFN layer, D={cfg['D']} E={cfg['E']} top-{cfg['K']} "
                     f"I={cfg['I']}, {experts}, T={cfg['T']} tokens per step)",
         "tokens_per_step": cfg["T"], "D": cfg["D"], "E": cfg["E"], "K": cfg["K"], "I": cfg["I"],
         "layers_in_ring": ring,
         "l2": f"steps cycle a ring of {ring} distinct layers "
               f"({ring * expert_bytes(cfg) * cfg['E'] / 1e9:.2f} GB of expert weights > 126 MB L2); "
               "no step re-reads weights of the previous steps"}
    if extra:
        d.update(extra)
    return d


def down_block_bytes(cfg):
    return 210 if cfg.get("down_q6k") else Q4K  # Q6_K or Q4_K super-block of the down tensor


def expert_bytes(cfg):
    D, I = cfg["D"], cfg["I"]
    return 2 * I * (D // 256) * Q4K + D * (I // 256) * down_block_bytes(cfg)


def layer_seeds(layer):
    from laii_b200 import synth
    return [synth.layer_seed(s, layer) for s in (synth.SEED_GATE, synth.SEED_UP, synth.SEED_DOWN,
                                                   synth.SEED_ROUTER, synth.SEED_BIAS)]


def zipf_bias_for(cfg, layer):
    """exp_probs_b giving Zipf(s) expert popularity for the seeded router of `layer` (config 3)."""
    from types import SimpleNamespace
    from laii_b200 import synth
    D, E = cfg["D"], cfg["E"]
    router = synth.normal_f32(E * D, synth.layer_seed(synth.SEED_ROUTER, layer), std=0.02).reshape(E, D)
    return synth.zipf_bias(SimpleNamespace(E=E, K=cfg["K"], D=D, eps=1e-5, router_w=router), s=cfg["zipf"])


def cpu_baseline(cfg, seconds=12.0, threads=0):
    """The reference's CPU MoE FFN (built from its sources) on this host, bounded sample."""
    from laii_b200 import synth
    from oracle.oracle import REF_SO, Oracle, Reference
    L = synth.make_moe_layer(cfg["D"], cfg["E"], cfg["K"], cfg["I"], layer=0,
                             down_type=14 if cfg.get("down_q6k") else 12)
    T = cfg["T"]
    x = synth.make_hidden(T, cfg["D"], seed_offset=0)
    if os.path.exists(REF_SO):
        R = Reference(threads)
        kind, cores, fwd = "reference", R.n_threads, (lambda xx: R.moe_forward(L, xx, capture=False))
        label = f"{R.isa}; {R.cpu}"
    else:
        O = Oracle()
        kind, cores, fwd = "port", 1, (lambda xx: O.moe_forward(L, xx))
        label = "scalar oracle port"
    fwd(x)  # warm
    n, t0 = 0, time.perf_counter()
    while True:
        fwd(x)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    tok_s = n * T / el
    return {"value": tok_s, "unit": "tok/s", "cores": cores, "kind": kind,
            "sample": f"{n} calls x {T} tokens (cfg layer 0 weights, one lfm2_forward_moe_ffn_1x4 call per token), "
                      f"{el:.1f} s; {label}; nproc={os.cpu_count()}"}


def run_reference(args, cfg):
    ws, rank, _ = dist_setup()
    if rank != 0:
        return
    from laii_b200 import synth
    from oracle.oracle import REF_SO, Oracle, Reference
    L = synth.make_moe_layer(cfg["D"], cfg["E"], cfg["K"], cfg["I"], layer=0,
                             down_type=14 if cfg.get("down_q6k") else 12)
    T = cfg["T"]
    x = synth.make_hidden(T, cfg["D"], seed_offset=0)
    if os.path.exists(REF_SO):
        R = Reference(0)
        kind, cores = "reference", R.n_threads
        fwd = lambda xx: R.moe_forward(L, xx, capture=False)  # noqa: E731
        label = f"{R.isa}; {R.cpu}"
    else:
        O = Oracle()
        kind, cores = "port", 1
        fwd = lambda xx: O.moe_forward(L, xx)  # noqa: E731
        label = "scalar oracle port"
    for _ in range(args.warmup):
        fwd(x)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        fwd(x)
    el = time.perf_counter() - t0
    v = T * args.steps / el
    out = {"impl": "reference", "metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": ws, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": el * 1e3 / args.steps, "higher_is_better": True, "scaling": "weak",
           "vs_baseline": None, "dtype": "q4_k x q8_k int, fp32 accum", "data": "synthetic (seeded)",
           "config": config_dict(args.config, cfg, 1),
           "cpu_baseline": {"value": v, "unit": "tok/s", "cores": cores, "kind": kind,
                            "sample": f"{args.steps} steps x {T} tokens, one lfm2_forward_moe_ffn_1x4 call per "
                                      f"token; {label}; nproc={os.cpu_count()}"},
           "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


def run_ours(args, cfg):
    import torch
    ws, rank, local = dist_setup()
    if ws > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    torch.cuda.set_device(local)
    from laii_b200 import synth
    from laii_b200.moe import GpuMoE

    D, E, K, I, T = cfg["D"], cfg["E"], cfg["K"], cfg["I"], cfg["T"]
    R = args.ring
    g = GpuMoE(local)
    if cfg.get("down_q6k"):  # host-made layers (Q6_K down from our own quantiser), fewer of them
        R = min(R, 2)
        for l in range(R):
            g.upload_layer(l, synth.make_moe_layer(D, E, K, I, layer=l, down_type=14))
    for l in range(0 if cfg.get("down_q6k") else R):
        bias = zipf_bias_for(cfg, l) if cfg.get("zipf") else None
        g.synth_layer(l, D, E, K, I, layer_seeds(l), bias=bias)
    g.reserve(T)
    x0 = synth.make_hidden(T, D, seed_offset=rank * T)
    x = torch.from_numpy(x0.copy()).cuda()
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream

    def step(i):
        g.forward_device(i % R, x.data_ptr(), T, stream=sp)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    st0 = g.last_stats()
    if ws > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        step(i)
    e1.record(stream)
    torch.cuda.synchronize()
    if ws > 1:
        torch.distributed.barrier()
    ms = e0.elapsed_time(e1)
    clk = clocks.stop()
    st1 = g.last_stats()
    loads = st1["expert_loads"] - st0["expert_loads"]
    kernels_per_step = st1["kernels_launched"]
    if ws > 1:
        t = torch.tensor([ms], device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    ms_step = ms / args.steps
    value = ws * T * args.steps / (ms / 1e3)

    # algorithmic bytes: active experts' gate/up/down + router + x in/out
    eb = expert_bytes(cfg)
    layer_bytes = loads * eb + args.steps * (E * D * 4 + 2 * T * D * 4)
    pk = peaks()
    layer_frac = layer_bytes / (ms / 1e3) / (pk["hbm_gbs"] * 1e9)

    # per-kernel pass (event-bracketed launches inside the library) for the roofline of the dominant kernel
    g.profile(True)
    stp = g.last_stats()
    for i in range(args.steps):
        step(i)
    torch.cuda.synchronize()
    prof = g.profile_read()
    g.profile(False)
    stq = g.last_stats()
    ploads = stq["expert_loads"] - stp["expert_loads"]
    # dominant kernel among those whose algorithmic work is counted below
    known = [k for k in prof if k in ("gateup", "down", "moe_layer", "gemm_gate", "gemm_up", "gemm_down", "gemm_gateup")]
    dom = max(known or list(prof), key=lambda k: prof[k][1])
    n_launch, tot_ms = prof[dom]
    gu_bytes = 2 * I * (D // 256) * Q4K
    dn_bytes = D * (I // 256) * down_block_bytes(cfg)
    # algorithmic bytes per launch: the active experts' Q4_K bytes (each read once) plus, for the
    # fused layer, the router rows and x in/out; Q8_K activations at 292/256 bytes per value
    per_launch_bytes = {"gateup": ploads * gu_bytes / n_launch + T * D * 1.140625,
                        "down": ploads * dn_bytes / n_launch + T * K * I * 1.140625 + T * K * D * 4,
                        "moe_layer": ploads * (gu_bytes + dn_bytes) / n_launch + E * D * 4 + 2 * T * D * 4}
    tensor_bound = dom.startswith("gemm_")
    if tensor_bound:
        # int8 ops of one GEMM launch: 2 * (T*K rows) * rows_out * cols (each matrix once)
        gemm_ops = {"gemm_gate": 2.0 * T * K * I * D, "gemm_up": 2.0 * T * K * I * D, "gemm_down": 2.0 * T * K * D * I,
                    "gemm_gateup": 4.0 * T * K * I * D}
        ach = gemm_ops[dom] / (tot_ms / n_launch / 1e3) / 1e12
    else:
        ach = per_launch_bytes.get(dom, 0.0) / (tot_ms / n_launch / 1e3) / 1e9
    total_prof = sum(v[1] for v in prof.values())
    traffic = None
    tfile = os.path.join(ROOT, "profiles", f"traffic_{dom}_cfg{args.config}.json")
    if os.path.exists(tfile):
        traffic = json.load(open(tfile)).get("dram_bytes_per_launch")

    # end to end through the public host-buffer API (H2D + forward + D2H per call)
    pinned = torch.empty((T, D), dtype=torch.float32, pin_memory=True)
    xh = pinned.numpy()
    xh[:] = x0
    n_e2e = max(10, min(args.steps, 500))
    for i in range(3):
        g.forward(i % R, xh)
    if ws > 1:
        torch.distributed.barrier()
    t0 = time.perf_counter()
    for i in range(n_e2e):
        g.forward(i % R, xh)
    e2e_s = time.perf_counter() - t0
    if ws > 1:
        t = torch.tensor([e2e_s], device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e = ws * T * n_e2e / e2e_s

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(cfg, seconds=args.cpu_seconds)

    if rank == 0:
        out = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": ws, "steps": args.steps,
               "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
               "vs_baseline": None, "data": "synthetic (seeded)",
               "dtype": ("u8 x s8 -> s32 (q4_k x q8_k; down q6_k x q8_k), fp32 accum" if cfg.get("down_q6k")
                         else "u8 x s8 -> s32 (q4_k x q8_k), fp32 accum"),
               "config": config_dict(args.config, cfg, R, {"parallelism": f"replicas x{ws}" if ws > 1 else "single",
                                                           "layer_hbm_frac": round(layer_frac, 4),
                                                           "unique_experts_per_step": loads / args.steps}),
               "roofline": ({"bound": "tensor", "kernel": dom, "achieved": ach, "peak": 4500.0, "unit": "TOP/s (int8)",
                             "frac": ach / 4500.0, "traffic": traffic,
                             "peak_src": "nominal dense int8 4.5 POPS (MEASURED_PEAKS.json holds no int8 figure)"}
                            if tensor_bound else
                            {"bound": "hbm", "kernel": dom, "achieved": ach, "peak": pk["hbm_gbs"], "unit": "GB/s",
                             "frac": ach / pk["hbm_gbs"], "traffic": traffic, "peak_src": pk["src"] + " (burst copy)"}) | {
                            "share": tot_ms / total_prof,
                            "kernel_ms": {k: round(v[1] / v[0] * 1e3, 2) for k, v in prof.items()},
                            "kernel_ms_unit": "us per launch"},
               "cpu_baseline": cpu,
               "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": T * D * 4, "d2h_bytes_per_step": T * D * 4},
               "gpu_launches": kernels_per_step * args.steps,
               "clocks": clk}
        print(json.dumps(out), flush=True)
    if ws > 1:
        torch.distributed.barrier()  # no rank frees its arena while another may still write into it
    g.close()
    if ws > 1:
        torch.distributed.destroy_process_group()


def stack_layers(cfg):
    """(kind, layer index) of a stack config: dense layers first, then MoE layers."""
    return [("dense", l) for l in range(cfg.get("dense", 0))] + \
           [("moe", cfg.get("dense", 0) + m) for m in range(cfg["layers"])]


def stack_cpu_baseline(cfg, seconds, threads=0):
    """The reference's CPU path per (token, layer), timed on one MoE (and one dense) layer over a bounded
    sample and extrapolated to the stack: tok/s = 1 / sum over layers of the per-token layer time."""
    from laii_b200 import synth
    from oracle.oracle import REF_SO, Reference
    if not os.path.exists(REF_SO):
        return None
    R = Reference(threads)
    D = cfg["D"]
    L = synth.make_moe_layer(D, cfg["E"], cfg["K"], cfg["I"], layer=cfg.get("dense", 0))
    per_layer = {}
    layers = [("moe", L)]
    if cfg.get("dense", 0):
        layers.append(("dense", synth.make_dense_layer(D, cfg["dense_I"], layer=0)))
    for kind, lay in layers:
        x = synth.make_hidden(8, D, seed_offset=0)
        fwd = (lambda xx: R.moe_forward(lay, xx, capture=False)) if kind == "moe" else (lambda xx: R.dense_forward(lay, xx))
        fwd(x)
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < seconds / len(layers):
            fwd(x)
            n += 1
        per_layer[kind] = (time.perf_counter() - t0) / (n * 8)
    t_tok = cfg["layers"] * per_layer["moe"] + cfg.get("dense", 0) * per_layer.get("dense", 0.0)
    return {"value": 1.0 / t_tok, "unit": "tok/s", "cores": R.n_threads, "kind": "reference",
            "sample": f"per-token layer time of the reference (one call per token, 8-token batches) on one MoE layer "
                      f"({per_layer['moe'] * 1e6:.0f} us)" + (f" and one dense layer ({per_layer['dense'] * 1e6:.0f} us)"
                                                              if "dense" in per_layer else "") +
                      f", extrapolated to the {len(stack_layers(cfg))}-layer stack; {R.isa}; nproc={os.cpu_count()}"}


KERNEL_NAMES = ("route", "gateup", "quant_h", "down", "combine", "moe_layer", "gemm_plan", "gemm_gate", "gemm_up",
                "swiglu_q8", "gemm_down", "xt_gather", "gemm_gateup", "ep_publish", "ep_plan")


def run_stack(args, cfg):
    """Configs 4 and 5: a stack of FFN layers, T tokens in total per step (strong scaling over ranks).
    One GPU: the stack as one captured forward.  N GPUs with --ep: experts sharded across ranks,
    each rank's T/N tokens routed and exchanged by the library's peer-memory kernels (--ep-comm p2p,
    the default) or NCCL all-to-all driven from Python (--ep-comm nccl, laii_b200.ep.ep_forward)."""
    import torch
    ws, rank, local = dist_setup()
    torch.cuda.set_device(local)
    if ws > 1:
        import torch.distributed as dist
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=torch.device("cuda", local), timeout=timedelta(seconds=300))
    from laii_b200 import ep, synth
    from laii_b200.moe import GpuMoE

    D, E, K, I, T = cfg["D"], cfg["E"], cfg["K"], cfg["I"], cfg["T"]
    use_ep = args.ep and ws > 1
    if T % ws:
        raise SystemExit(f"T={T} does not split over {ws} ranks")
    Tl = T // ws
    g = GpuMoE(local)
    layers = stack_layers(cfg)
    first, count = ep.shard_of(E, ws, rank) if use_ep else (0, E)
    for kind, l in layers:
        if kind == "dense":
            g.upload_dense(l, synth.make_dense_layer(D, cfg["dense_I"], layer=l))
        elif use_ep:
            g.synth_layer_shard(l, D, E, K, I, layer_seeds(l), first, count)
        else:
            g.synth_layer(l, D, E, K, I, layer_seeds(l))
    g.reserve(max(Tl * K if use_ep else Tl, Tl))
    p2p = use_ep and args.ep_comm == "p2p"
    if p2p:  # the library's own exchange kernels over peer memory; torch.distributed carries the IPC handles
        ep.p2p_connect(g, Tl, D, E, K, I)
    x0 = synth.make_hidden(Tl, D, seed_offset=rank * Tl)
    x = torch.from_numpy(x0.copy()).cuda()
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    comm = ep.TorchComm() if use_ep and not p2p else None
    ops = ep.GpuOps(g, D, K) if use_ep else None

    def step():
        if not use_ep:
            g.forward_device(0, x.data_ptr(), Tl, stream=sp, n_layers=len(layers))
            return
        if p2p:  # the whole stack in one call: a captured CUDA graph after the first step
            g.ep_p2p_forward_stack(0, len(layers), x.data_ptr(), Tl, sp)
            ops.launches += g.last_stats()["kernels_launched"]
            return
        for kind, l in layers:
            if kind == "dense":
                g.forward_device(l, x.data_ptr(), Tl, stream=sp)
            else:
                ep.ep_forward(ops, comm, l, x, E, K)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    # kernels one step launches: the library's own count (graph replay on one GPU, per call with EP)
    if use_ep:
        l0 = ops.launches
        step()
        launches_per_step = ops.launches - l0
    else:
        step()
        launches_per_step = g.last_stats()["kernels_launched"]
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    st0 = g.last_stats()
    if ws > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    if ws > 1:
        torch.distributed.barrier()
    ms = e0.elapsed_time(e1)
    clk = clocks.stop()
    st1 = g.last_stats()
    loads = float(st1["expert_loads"] - st0["expert_loads"])
    if ws > 1:
        t = torch.tensor([ms, loads], device="cuda", dtype=torch.float64)
        mx = t.clone()
        torch.distributed.all_reduce(mx, op=torch.distributed.ReduceOp.MAX)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.SUM)
        ms, loads = float(mx[0].item()), float(t[1].item())
    ms_step = ms / args.steps
    value = T * args.steps / (ms / 1e3)
    pk = peaks()
    n_moe, n_dense = cfg["layers"], cfg.get("dense", 0)
    if T <= 64:  # decode: HBM-bound on the active experts' bytes
        dense_bytes = n_dense * 3 * cfg.get("dense_I", 0) * D * Q4K // 256
        step_bytes = loads / args.steps * expert_bytes(cfg) + n_moe * E * D * 4 + dense_bytes + 2 * T * D * 4
        ach = step_bytes / (ms_step / 1e3) / 1e9
        roof = {"bound": "hbm", "kernel": "stack step", "achieved": ach, "peak": pk["hbm_gbs"], "unit": "GB/s",
                "frac": ach / pk["hbm_gbs"], "traffic": None, "peak_src": pk["src"] + " (burst copy)",
                "algorithmic_bytes_per_step": step_bytes}
    else:  # prefill: int8 tensor-op bound
        ops_step = 2.0 * T * K * 3 * I * D * n_moe
        ach = ops_step / (ms_step / 1e3) / 1e12
        roof = {"bound": "tensor", "kernel": "stack step", "achieved": ach, "peak": 4500.0, "unit": "TOP/s (int8)",
                "frac": ach / 4500.0, "traffic": None,
                "peak_src": "nominal dense int8 4.5 POPS (MEASURED_PEAKS.json holds no int8 figure)",
                "algorithmic_ops_per_step": ops_step}
    # end to end through the public API with host buffers: this rank's tokens copied in from pinned
    # host memory, the whole stack, the result copied back, every step; wall clock, max over ranks
    pinned = torch.empty((Tl, D), dtype=torch.float32, pin_memory=True)
    pinned.numpy()[:] = x0
    n_e2e = max(3, min(args.steps, 20))

    def e2e_step():
        if not use_ep:
            g.forward_stack(0, len(layers), pinned.numpy())
            return
        x.copy_(pinned, non_blocking=True)
        step()
        pinned.copy_(x, non_blocking=True)
        torch.cuda.current_stream().synchronize()

    e2e_step()
    if ws > 1:
        torch.distributed.barrier()
    t0 = time.perf_counter()
    for _ in range(n_e2e):
        e2e_step()
    e2e_s = time.perf_counter() - t0
    if ws > 1:
        t = torch.tensor([e2e_s], device="cuda", dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e = T * n_e2e / e2e_s

    kprof = None
    if args.kernel_profile:  # after the timed region: events around every launch (no graphs), mean us per launch
        g.profile(True)
        for _ in range(max(1, min(args.steps, 5))):
            if p2p:
                for kind, l in layers:
                    if kind == "dense":
                        g.forward_device(l, x.data_ptr(), Tl, stream=sp)
                    else:
                        g.ep_p2p_forward(l, x.data_ptr(), Tl, sp)
            else:
                step()
        torch.cuda.synchronize()
        prof = g.profile_read()
        g.profile(False)
        names = sorted(KERNEL_NAMES)
        mean = torch.tensor([prof[n][1] / prof[n][0] * 1e3 if n in prof else 0.0 for n in names], dtype=torch.float64,
                            device="cuda")
        if ws > 1:  # the slowest rank's figure per kernel
            torch.distributed.all_reduce(mean, op=torch.distributed.ReduceOp.MAX)
        kprof = {n: round(float(v), 1) for n, v in zip(names, mean.tolist()) if v > 0}

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        cpu = stack_cpu_baseline(cfg, args.cpu_seconds)
    if rank == 0:
        out = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": ws, "steps": args.steps,
               "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
               "vs_baseline": None, "dtype": "u8 x s8 -> s32 (q4_k x q8_k), fp32 accum", "data": "synthetic (seeded)",
               "config": {"workload": f"cfg{args.config}: {cfg['name']} ({n_dense} dense + {n_moe} lfm2moe FFN layers, "
                                      f"D={D} E={E} top-{K} I={I}, {T} tokens per step in total)",
                          "tokens_per_step": T, "layers": len(layers),
                          "parallelism": (f"expert-parallel x{ws} (E/{ws} experts per rank, "
                                          + ("exchange kernels over NVLink peer memory)" if p2p else "NCCL all-to-all)"))
                          if use_ep else ("single" if ws == 1 else f"replicas x{ws}"),
                          "l2": "the stack's weights exceed the 126 MB L2; every step streams them from HBM",
                          "unique_experts_per_moe_layer": loads / args.steps / n_moe},
               "roofline": roof, "cpu_baseline": cpu,
               "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": T * D * 4, "d2h_bytes_per_step": T * D * 4},
               "gpu_launches": launches_per_step * args.steps, "clocks": clk}
        if kprof is not None:
            out["kernel_profile"] = {"us_per_launch_max_over_ranks": kprof,
                                     "how": "library event profile after the timed region, eager launches"}
        print(json.dumps(out), flush=True)
    if ws > 1:
        torch.distributed.barrier()  # no rank frees its arena while another may still write into it
    g.close()
    if ws > 1:
        torch.distributed.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--config", type=int, default=2, choices=[1, 2, 3, 4, 5])
    ap.add_argument("--ep", action="store_true", help="configs 4/5 under torchrun: expert parallelism")
    ap.add_argument("--kernel-profile", action="store_true",
                    help="stack configs: add per-kernel event times (max over ranks) to the JSON line")
    ap.add_argument("--ep-comm", default="p2p", choices=["p2p", "nccl"],
                    help="--ep exchange: the library's peer-memory kernels (p2p) or torch all_to_all over NCCL")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--ring", type=int, default=8)
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--down-q6k", action="store_true",
                    help="configs 1-3: the layers' ffn_down_exps in Q6_K (as Q4_K_M checkpoints store some)")
    args = ap.parse_args()
    from laii_b200.synth import CONFIGS
    cfg = dict(CONFIGS[args.config])
    if args.down_q6k:
        if args.config >= 4:
            raise SystemExit("--down-q6k: single-layer configs 1-3 only")
        cfg["down_q6k"] = True
    if args.impl == "reference":
        run_reference(args, cfg)
    elif args.config >= 4:
        run_stack(args, cfg)
    else:
        run_ours(args, cfg)


if __name__ == "__main__":
    main()
