#!/usr/bin/env python
"""lfm2moe MoE-FFN throughput on B200 (tokens/s), against the reference CPU path.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--config C] [--impl ours|reference]

Default workload: config 4, the LFM2-8B-A1B-shaped decode stack -- 2 dense
SwiGLU FFN layers (I=7168) then 22 lfm2moe layers (D=2048, E=32, top-4,
I=1792, Q4_K), 64 tokens (one per sequence) per step.  A step is one forward of
the whole stack over the step's tokens.  Under torchrun (N ranks) the stack
runs expert-parallel: every rank holds the routers and dense layers and E/N of
each layer's experts, takes T/N of the tokens, and the library's own kernels
exchange the rows over NVLink peer memory (strong scaling: T is the total).

The same line carries a "prefill" block: config 5, the 24B-A2B-scale stack
(38 lfm2moe layers, E=64, I=1536) over T=4096 tokens, on the same ranks.

Printed JSON (one line, rank 0):
  value      tokens/s over all ranks, inputs resident in HBM, device-timed (CUDA
             events on the launch stream, max over ranks);
  e2e        the same metric through the public host-buffer API: each step
             copies the tokens in from pinned host memory, runs the stack and
             copies the result back (wall clock, max over ranks);
  roofline   the dominant kernel: its algorithmic bytes (decode) or int8 ops
             (prefill) per launch over its mean event-timed launch, against
             MEASURED_PEAKS.json's HBM copy rate or an int8 GEMM peak measured
             in this run (torch._int_mm); "step" holds the whole-step figure;
  parity     every rank re-runs a token subset layer by layer and compares each
             layer's rows with the reference CPU path (oracle/_ref) run on the
             same input rows: ids, Q8_K, weights, rel-L2 and max-abs; a miss
             makes the run exit non-zero;
  cpu_baseline  the reference's own CPU path on this host's cores (rank 0, N=1).
--impl reference times the reference's CPU path (oracle/_ref, built from the
reference sources) on the same workload and prints the same config.
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
Q8K_PER_VALUE = 292 / 256
METRIC = "MoE-FFN tok/s: decode %HBM roofline, prefill %int8 TC peak, 1/2/4/8 B200"
NOMINAL_INT8_TOPS = 4500.0
SPARE_SLOT = 63  # layer slot used to rebuild a full layer for the parity check of an expert shard


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "src": "fallback"}


def measure_int8_peak(torch, n=8192, reps=10):
    """Dense int8 tensor-core throughput of this GPU: torch._int_mm (cuBLASLt) on n^3, best of reps."""
    try:
        a = torch.randint(-128, 127, (n, n), dtype=torch.int8, device="cuda")
        b = torch.randint(-128, 127, (n, n), dtype=torch.int8, device="cuda").t().contiguous().t()
        for _ in range(3):
            torch._int_mm(a, b)
        best = float("inf")
        for _ in range(reps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            torch._int_mm(a, b)
            e1.record()
            e1.synchronize()
            best = min(best, e0.elapsed_time(e1))
        del a, b
        torch.cuda.empty_cache()
        return {"tops": 2.0 * n ** 3 / (best / 1e3) / 1e12,
                "src": f"measured in this run: torch._int_mm int8 {n}^3, best of {reps}"}
    except Exception as ex:  # noqa: BLE001 -- report the nominal figure instead
        return {"tops": NOMINAL_INT8_TOPS, "src": f"nominal dense int8 (measurement failed: {ex})"}


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


# ---------------------------------------------------------------------------
# workload descriptions (identical in both arms)
# ---------------------------------------------------------------------------

def down_block_bytes(cfg):
    return 210 if cfg.get("down_q6k") else Q4K  # Q6_K or Q4_K super-block of the down tensor


def expert_bytes(cfg):
    D, I = cfg["D"], cfg["I"]
    return 2 * I * (D // 256) * Q4K + D * (I // 256) * down_block_bytes(cfg)


def dense_bytes(cfg):
    return 3 * cfg.get("dense_I", 0) * cfg["D"] // 256 * Q4K


def stack_layers(cfg):
    """(kind, layer index) of a config: dense layers first, then MoE layers."""
    return [("dense", l) for l in range(cfg.get("dense", 0))] + \
           [("moe", cfg.get("dense", 0) + m) for m in range(cfg["layers"])]


def workload(cfg_id, cfg):
    """The workload as both arms name it: the config's shapes, nothing about how it is run."""
    n_moe, n_dense = cfg["layers"], cfg.get("dense", 0)
    experts = "Q4_K gate/up and Q6_K down experts" if cfg.get("down_q6k") else "Q4_K experts"
    wbytes = n_moe * cfg["E"] * expert_bytes(cfg) + n_dense * dense_bytes(cfg)
    d = {"workload": f"cfg{cfg_id}: {cfg['name']} ({n_dense} dense + {n_moe} lfm2moe FFN layers, D={cfg['D']} "
                     f"E={cfg['E']} top-{cfg['K']} I={cfg['I']}, {experts}, {cfg['T']} tokens per step)",
         "tokens_per_step": cfg["T"], "layers": n_moe + n_dense, "moe_layers": n_moe, "dense_layers": n_dense,
         "D": cfg["D"], "E": cfg["E"], "K": cfg["K"], "I": cfg["I"]}
    if n_dense:
        d["dense_I"] = cfg["dense_I"]
    if cfg.get("zipf"):
        d["routing"] = f"exp_probs_b calibrated to Zipf({cfg['zipf']}) expert popularity"
    if n_moe + n_dense > 1:
        d["l2"] = (f"inputs larger than L2: the stack's {wbytes / 1e9:.2f} GB of FFN weights exceed the 126 MB L2, "
                   "so every step streams them from HBM")
    else:
        d["l2"] = ("inputs larger than L2: consecutive steps cycle a ring of distinct layers whose expert weights "
                   "exceed the 126 MB L2")
    return d


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


def host_layer(cfg, kind, l):
    """Host copy of layer l of a config (the CPU arms; the GPU arm fills the same bytes on the device)."""
    from laii_b200 import synth
    if kind == "dense":
        return synth.make_dense_layer(cfg["D"], cfg["dense_I"], layer=l)
    bias = zipf_bias_for(cfg, l) if cfg.get("zipf") else None
    return synth.make_moe_layer(cfg["D"], cfg["E"], cfg["K"], cfg["I"], layer=l, bias=bias,
                                down_type=14 if cfg.get("down_q6k") else 12)


# ---------------------------------------------------------------------------
# the reference's CPU path (oracle/_ref): cpu_baseline leg and --impl reference
# ---------------------------------------------------------------------------

def _cpu_forward(R, kind, L, x):
    return R.moe_forward(L, x, capture=False)[0] if kind == "moe" else R.dense_forward(L, x)


def cpu_baseline(cfg, seconds=12.0, threads=0):
    """The reference's CPU path (built from its sources) on this host over a bounded sample: the
    per-token time of one MoE (and one dense) layer, extrapolated to the config's stack
    (tok/s = 1 / sum over layers of the per-token layer time).  The reference has no batched MoE:
    one lfm2_forward_moe_ffn_1x4 call per token."""
    from laii_b200 import synth
    from oracle.oracle import REF_SO, Oracle, Reference
    kinds = ["moe"] + (["dense"] if cfg.get("dense") else [])
    if os.path.exists(REF_SO):
        R = Reference(threads)
        kind_s, cores, label = "reference", R.n_threads, f"{R.isa}; {R.cpu}"
    else:
        R = Oracle()
        kind_s, cores, label = "port", 1, "scalar oracle port"
    per_tok = {}
    T = min(cfg["T"], 8)
    for kind in kinds:
        L = host_layer(cfg, kind, 0 if kind == "dense" else cfg.get("dense", 0))
        x = synth.make_hidden(T, cfg["D"], seed_offset=0)
        _cpu_forward(R, kind, L, x)
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < seconds / len(kinds):
            _cpu_forward(R, kind, L, x)
            n += 1
        per_tok[kind] = (time.perf_counter() - t0) / (n * T)
    t_tok = cfg["layers"] * per_tok["moe"] + cfg.get("dense", 0) * per_tok.get("dense", 0.0)
    n_layers = cfg["layers"] + cfg.get("dense", 0)
    return {"value": 1.0 / t_tok, "unit": "tok/s", "cores": cores, "kind": kind_s,
            "sample": f"per-token time of the reference ({T}-token calls, one lfm2_forward_moe_ffn_1x4 per token) on "
                      f"one MoE layer ({per_tok['moe'] * 1e6:.0f} us)"
                      + (f" and one dense layer ({per_tok['dense'] * 1e6:.0f} us)" if "dense" in per_tok else "")
                      + (f", extrapolated to the {n_layers}-layer stack" if n_layers > 1 else "")
                      + f"; {label}; nproc={os.cpu_count()}"}


def run_reference(args, cfg_id, cfg):
    """--impl reference: the reference's own CPU path (oracle/_ref) on the same workload.  A step is
    the config's whole stack over its T tokens, one lfm2_forward_moe_ffn_1x4 call per token and
    layer (dense layers: lfm2_forward_ffn_fused_1x4's path); all host threads but one (the reference
    pool's default).  Inputs come from the oracle's own build of the seeded generator."""
    ws, rank, _ = dist_setup()
    if rank != 0:
        return
    from laii_b200 import synth
    from oracle.oracle import GEN_SO, REF_SO, Oracle, Reference
    if os.path.exists(GEN_SO):
        synth.use_generator_library(GEN_SO)
    if os.path.exists(REF_SO):
        R = Reference(0)
        kind, cores, label = "reference", R.n_threads, f"{R.isa}; {R.cpu}"
    else:
        R = Oracle()
        kind, cores, label = "port", 1, "scalar oracle port"
    layers = stack_layers(cfg)
    host = [(k, host_layer(cfg, k, l)) for k, l in layers]
    T = cfg["T"]
    x0 = synth.make_hidden(T, cfg["D"], seed_offset=0)

    def step():
        x = x0
        for k, L in host:
            x = _cpu_forward(R, k, L, x)
        return x

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    el = time.perf_counter() - t0
    v = T * args.steps / el
    out = {"impl": "reference", "metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": ws, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": el * 1e3 / args.steps, "higher_is_better": True,
           "scaling": "strong" if len(layers) > 1 else "weak", "vs_baseline": None,
           "dtype": "u8 x s8 -> s32 (q4_k x q8_k), fp32 accum", "data": "synthetic (seeded)",
           "config": workload(cfg_id, cfg),
           "cpu_baseline": {"value": v, "unit": "tok/s", "cores": cores, "kind": kind,
                            "sample": f"{args.steps} steps x {T} tokens through all {len(layers)} layers, one "
                                      f"reference call per token and layer; {label}; nproc={os.cpu_count()}"},
           "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    del host
    if args.prefill_config and cfg_id != args.prefill_config:
        out["prefill"] = reference_prefill_sample(args.prefill_config, R, label, cores, kind)
    print(json.dumps(out), flush=True)


def reference_prefill_sample(cfg_id, R, label, cores, kind, tokens=32, n_layers=4):
    """The prefill stack on the reference CPU path, as a bounded sample: `tokens` tokens through
    `n_layers` of its layers, extrapolated to the whole stack (every layer has the same shape and
    the reference's cost per token and layer does not depend on T: it loops over tokens)."""
    from laii_b200 import synth
    from laii_b200.synth import CONFIGS
    cfg = dict(CONFIGS[cfg_id])
    layers = stack_layers(cfg)[:n_layers]
    host = [(k, host_layer(cfg, k, l)) for k, l in layers]
    x = synth.make_hidden(tokens, cfg["D"], seed_offset=0)
    for k, L in host[:1]:
        _cpu_forward(R, k, L, x[:2])
    t0 = time.perf_counter()
    for k, L in host:
        x = _cpu_forward(R, k, L, x)
    el = time.perf_counter() - t0
    per_tok_layer = el / (tokens * len(host))
    v = 1.0 / (per_tok_layer * (cfg["layers"] + cfg.get("dense", 0)))
    return {"config": workload(cfg_id, cfg), "value": v, "unit": "tok/s",
            "ms_per_step": cfg["T"] / v * 1e3,
            "cpu_baseline": {"value": v, "unit": "tok/s", "cores": cores, "kind": kind,
                             "sample": f"{tokens} tokens through {len(host)} of the {len(stack_layers(cfg))} layers "
                                       f"({el:.1f} s), extrapolated to the stack; {label}"},
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


# ---------------------------------------------------------------------------
# the GPU arm
# ---------------------------------------------------------------------------

class StackRun:
    """One config on this rank: layers on the device, the timed step, the per-kernel profile, the
    end-to-end pass and the parity check.  use_ep: experts sharded across the ranks."""

    def __init__(self, cfg_id, cfg, ws, rank, local, use_ep, ep_comm):
        import torch
        from laii_b200 import ep, synth
        from laii_b200.moe import GpuMoE
        self.torch, self.ep, self.synth = torch, ep, synth
        self.cfg_id, self.cfg, self.ws, self.rank, self.local = cfg_id, cfg, ws, rank, local
        D, E, K, I, T = cfg["D"], cfg["E"], cfg["K"], cfg["I"], cfg["T"]
        self.layers = stack_layers(cfg)
        self.single = len(self.layers) == 1
        self.use_ep = use_ep and ws > 1 and not self.single  # single-layer configs run as replicas
        if self.use_ep and T % ws:
            raise SystemExit(f"T={T} does not split over {ws} ranks")
        self.Tl = T // ws if self.use_ep else T
        self.ring = 1
        self.g = g = GpuMoE(local)
        self.dense_host = {}
        self.first, self.count = ep.shard_of(E, ws, rank) if self.use_ep else (0, E)
        if self.single:  # one layer: steps cycle a ring of distinct copies (weights > L2)
            self.ring = max(1, min(args_ring(), 8))
            for l in range(self.ring):
                if cfg.get("down_q6k"):
                    g.upload_layer(l, synth.make_moe_layer(D, E, K, I, layer=l, down_type=14))
                else:
                    g.synth_layer(l, D, E, K, I, layer_seeds(l),
                                  bias=zipf_bias_for(cfg, l) if cfg.get("zipf") else None)
        else:
            for kind, l in self.layers:
                if kind == "dense":
                    self.dense_host[l] = synth.make_dense_layer(D, cfg["dense_I"], layer=l)
                    g.upload_dense(l, self.dense_host[l])
                elif self.use_ep:
                    g.synth_layer_shard(l, D, E, K, I, layer_seeds(l), self.first, self.count)
                else:
                    g.synth_layer(l, D, E, K, I, layer_seeds(l))
        g.reserve(max(self.Tl * K if self.use_ep else self.Tl, self.Tl))
        self.p2p = self.use_ep and ep_comm == "p2p"
        if self.p2p:  # the library's own exchange kernels over peer memory; torch.distributed carries the handles
            ep.p2p_connect(g, self.Tl, D, E, K, I)
        self.x0 = synth.make_hidden(self.Tl, D, seed_offset=rank * self.Tl)
        self.x = torch.from_numpy(self.x0.copy()).cuda()
        self.stream = torch.cuda.current_stream()
        self.sp = self.stream.cuda_stream
        self.comm = ep.TorchComm() if self.use_ep and not self.p2p else None
        self.ops = ep.GpuOps(g, D, K) if self.use_ep else None
        self.i = 0

    # -- one step --------------------------------------------------------
    def step(self):
        g, x = self.g, self.x
        if self.single:
            g.forward_device(self.i % self.ring, x.data_ptr(), self.Tl, stream=self.sp)
            self.i += 1
        elif not self.use_ep:
            g.forward_device(0, x.data_ptr(), self.Tl, stream=self.sp, n_layers=len(self.layers))
        elif self.p2p:  # the whole stack in one call: a captured CUDA graph after the first step
            g.ep_p2p_forward_stack(0, len(self.layers), x.data_ptr(), self.Tl, self.sp)
            self.ops.launches += g.last_stats()["kernels_launched"]
        else:
            for kind, l in self.layers:
                if kind == "dense":
                    g.forward_device(l, x.data_ptr(), self.Tl, stream=self.sp)
                else:
                    self.ep.ep_forward(self.ops, self.comm, l, x, self.cfg["E"], self.cfg["K"])

    def layer_eager(self, kind, l):
        """One layer of the stack on the device (every rank calls the same layers in the same order)."""
        g, x = self.g, self.x
        if kind == "dense" or not self.use_ep:
            g.forward_device(l, x.data_ptr(), self.Tl, stream=self.sp)
        elif self.p2p:
            g.ep_p2p_forward(l, x.data_ptr(), self.Tl, self.sp)
        else:
            self.ep.ep_forward(self.ops, self.comm, l, x, self.cfg["E"], self.cfg["K"])

    def barrier(self):
        if self.ws > 1:
            self.torch.distributed.barrier()

    def allreduce(self, vals, op):
        if self.ws == 1:
            return [float(v) for v in vals]
        t = self.torch.tensor([float(v) for v in vals], device="cuda", dtype=self.torch.float64)
        self.torch.distributed.all_reduce(t, op=op)
        return [float(v) for v in t.tolist()]

    # -- timing ----------------------------------------------------------
    def timed(self, steps, warmup):
        torch = self.torch
        for _ in range(warmup):
            self.step()
        torch.cuda.synchronize()
        if self.use_ep:  # kernels one step launches: the library's own counts
            l0 = self.ops.launches
            self.step()
            launches = self.ops.launches - l0
        else:
            self.step()
            launches = self.g.last_stats()["kernels_launched"]
        torch.cuda.synchronize()
        clocks = ClockSampler(self.local)
        clocks.start()
        time.sleep(0.3)
        st0 = self.g.last_stats()
        self.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(self.stream)
        for _ in range(steps):
            self.step()
        e1.record(self.stream)
        torch.cuda.synchronize()
        self.barrier()
        ms = e0.elapsed_time(e1)
        clk = clocks.stop()
        st1 = self.g.last_stats()
        loads = st1["expert_loads"] - st0["expert_loads"]
        runs = st1["layer_runs"] - st0["layer_runs"]
        R = self.torch.distributed.ReduceOp if self.ws > 1 else None
        ms = self.allreduce([ms], R.MAX if R else None)[0]
        loads, = self.allreduce([loads], R.SUM if R else None)
        return {"ms": ms, "launches_per_step": launches, "loads": loads, "runs": runs, "clocks": clk}

    def kernel_profile(self, steps):
        """Events around every launch (eager, no graphs): {kernel: (launches, us per launch max over
        ranks)} and the expert loads (summed over ranks) of the profiled steps."""
        torch = self.torch
        g = self.g
        st0 = g.last_stats()
        g.profile(True)
        for _ in range(steps):
            if self.single or not self.use_ep:
                self.step()
            else:
                for kind, l in self.layers:
                    self.layer_eager(kind, l)
        torch.cuda.synchronize()
        prof = g.profile_read()
        g.profile(False)
        st1 = g.last_stats()
        names = sorted(set(KERNEL_NAMES))
        launches = [prof[n][0] if n in prof else 0 for n in names]
        us = [prof[n][1] / prof[n][0] * 1e3 if n in prof and prof[n][0] else 0.0 for n in names]
        R = torch.distributed.ReduceOp if self.ws > 1 else None
        us = self.allreduce(us, R.MAX if R else None)
        launches = self.allreduce(launches, R.MAX if R else None)
        loads, = self.allreduce([st1["expert_loads"] - st0["expert_loads"]], R.SUM if R else None)
        return {n: (int(c), u) for n, c, u in zip(names, launches, us) if u > 0}, loads

    def e2e(self, n):
        """Wall-clock seconds for n steps through the public API with host buffers, max over ranks."""
        torch = self.torch
        pinned = torch.empty((self.Tl, self.cfg["D"]), dtype=torch.float32, pin_memory=True)
        pinned.numpy()[:] = self.x0
        g = self.g

        def one():
            if self.single:
                g.forward(self.i % self.ring, pinned.numpy())
                self.i += 1
            elif not self.use_ep:
                g.forward_stack(0, len(self.layers), pinned.numpy())
            else:
                self.x.copy_(pinned, non_blocking=True)
                self.step()
                pinned.copy_(self.x, non_blocking=True)
                torch.cuda.current_stream().synchronize()

        one()
        self.barrier()
        t0 = time.perf_counter()
        for _ in range(n):
            one()
        s = time.perf_counter() - t0
        R = torch.distributed.ReduceOp if self.ws > 1 else None
        return self.allreduce([s], R.MAX if R else None)[0]

    # -- parity ------------------------------------------------------------
    def parity(self, n_tok):
        """Layer-by-layer check of a token subset of this rank against the reference CPU path
        (oracle/stack_check.py).  Returns the summary merged over ranks."""
        torch = self.torch
        from oracle.stack_check import StackChecker, summarise
        g, cfg = self.g, self.cfg
        D, E, K, I = cfg["D"], cfg["E"], cfg["K"], cfg["I"]
        n_tok = max(1, min(n_tok, self.Tl))
        sub = np.unique(np.linspace(0, self.Tl - 1, n_tok).astype(np.int64))
        layers = [("moe", 0)] if self.single else self.layers
        # 1. the device path, layer by layer, from this rank's step input
        self.x.copy_(torch.from_numpy(self.x0))
        rows = []
        for kind, l in layers:
            xin = self.x.cpu().numpy()[sub]
            self.layer_eager(kind, l)
            torch.cuda.synchronize()
            rows.append((kind, l, xin, self.x.cpu().numpy()[sub]))
        eager_final = self.x.cpu().numpy()
        # 2. the timed path (graphs) from the same input: the same kernels, so the same bits
        graph_equal = True
        if not self.single:
            self.x.copy_(torch.from_numpy(self.x0))
            self.step()
            torch.cuda.synchronize()
            graph_equal = bool(np.array_equal(self.x.cpu().numpy(), eager_final))
        g.sync()
        # 3. every layer on the CPU from the device's own input rows
        checker = StackChecker(max(1, (os.cpu_count() or 2) // self.ws - 1))
        per_layer = []
        for kind, l, xin, xout in rows:
            if kind == "dense":
                per_layer.append(checker.check_dense(self.dense_host[l], xin, xout))
                continue
            slot = l
            full = not (self.use_ep and self.count != E)
            if not full:  # an expert shard: rebuild the full layer in a spare slot to read the experts
                slot = SPARE_SLOT
                g.synth_layer(slot, D, E, K, I, layer_seeds(l))

            def read(which, off, nb, slot=slot):
                return g.read_layer(slot, which, nb, offset=off)

            Lh, sel, _ = checker.host_moe_layer(read, D, E, K, I, xin, down_type=14 if cfg.get("down_q6k") else 12)
            route = g.debug_route(l, np.ascontiguousarray(xin))
            per_layer.append(checker.check_moe(Lh, sel, xin, xout, route))
        s = summarise(per_layer)
        s["graph_equals_eager"] = graph_equal
        R = torch.distributed.ReduceOp if self.ws > 1 else None
        mx = self.allreduce([s["rel_l2"], s["max_abs"]], R.MAX if R else None)
        bad, ties, toks = self.allreduce([0 if (s["ok"] and graph_equal) else 1, s["near_ties"], len(sub)],
                                         R.SUM if R else None)
        q8_ok, ids_ok = self.allreduce([1 if s["q8_exact"] else 0, 1 if s["ids_match"] else 0],
                                       R.MIN if R else None)
        return {"ok": bad == 0, "rel_l2": mx[0], "max_abs": mx[1], "ids_match": ids_ok == 1,
                "q8_exact": q8_ok == 1, "near_ties": int(ties), "graph_equals_eager": bad == 0 or graph_equal,
                "tokens": int(toks), "layers": len(per_layer), "ranks_failed": int(bad),
                "checker": checker.kind,
                "how": "each rank's token subset re-run layer by layer on the CPU from the device's input rows; "
                       "bars rel-L2 <= 1e-3, max-abs <= 5e-3, ids equal except near-ties (< 1e-6), Q8_K bit-exact"}

    def close(self):
        self.barrier()  # no rank frees its arena while another may still write into it
        self.g.close()


KERNEL_NAMES = ("route", "gateup", "quant_h", "down", "combine", "moe_layer", "gemm_plan", "gemm_gate", "gemm_up",
                "swiglu_q8", "gemm_down", "xt_gather", "gemm_gateup", "ep_publish", "ep_plan")


def is_prefill(cfg):
    """Prefill sizes: at least 32 routed rows per expert on average (the tcgen05 GEMMs' prefill
    arrangement); below that the expert GEMMs stream weights and are HBM-bound."""
    return cfg["T"] * cfg["K"] >= 32 * cfg["E"]

_ARGS = None


def args_ring():
    return _ARGS.ring if _ARGS is not None else 8


def roofline(cfg, prof, loads_prof, prof_steps, ws, hbm, int8):
    """The dominant kernel's achieved rate.  Work per launch is counted for the whole job (all ranks'
    experts and rows), its time is the slowest rank's mean launch, and the rate is per GPU
    (job rate / ws, ws = the ranks sharing the job's work: N with expert parallelism, else 1).  Decode sizes are HBM-bound on the active experts' bytes; prefill sizes
    (T*K rows well above the expert count x 128) are int8-op bound."""
    D, E, K, I, T = cfg["D"], cfg["E"], cfg["K"], cfg["I"], cfg["T"]
    n_moe = cfg["layers"]
    runs = max(1, prof_steps * n_moe)
    U = loads_prof / runs  # distinct experts a MoE layer runs (all ranks together)
    rows = T * K
    gu_w, dn_w = 2 * I * (D // 256) * Q4K, D * (I // 256) * down_block_bytes(cfg)
    moe_kernels = {"gemm_gateup": ("gu", 2), "gemm_gate": ("gu", 1), "gemm_up": ("gu", 1), "gemm_down": ("dn", 1),
                   "gateup": ("gu", 2), "down": ("dn", 1), "q6k_down": ("dn", 1), "moe_layer": ("all", 1)}
    cands = {k: v for k, v in prof.items() if k in moe_kernels}
    if not cands:
        return None
    dom = max(cands, key=lambda k: cands[k][0] * cands[k][1])
    launches, us = cands[dom]
    total_us = sum(c * u for c, u in prof.values())
    share = launches * us / total_us if total_us else None
    which, mats = moe_kernels[dom]
    per_launch_layers = 1  # every one of these kernels covers one MoE layer a launch
    if is_prefill(cfg) and dom.startswith("gemm_"):
        ops = {"gu": 2.0 * rows * I * D * mats, "dn": 2.0 * rows * D * I, "all": 6.0 * rows * I * D}[which]
        ach = ops * per_launch_layers / (us / 1e6) / 1e12 / ws
        return {"bound": "tensor", "kernel": dom, "achieved": ach, "peak": int8["tops"], "unit": "TOP/s (int8)",
                "frac": ach / int8["tops"], "traffic": None, "peak_src": int8["src"],
                "work_per_launch": f"{ops:.4g} int8 ops (2*T*K*rows*cols over the layer's {rows} routed rows)",
                "us_per_launch": us, "share": share}
    wbytes = {"gu": U * gu_w / 2 * mats, "dn": U * dn_w, "all": U * (gu_w + dn_w) + E * D * 4}[which]
    act = {"gu": rows * D * Q8K_PER_VALUE + mats * rows * I * 4, "dn": rows * I * Q8K_PER_VALUE + rows * D * 4,
           "all": 2 * T * D * 4}[which]
    b = wbytes + act
    ach = b / (us / 1e6) / 1e9 / ws
    return {"bound": "hbm", "kernel": dom, "achieved": ach, "peak": hbm["hbm_gbs"], "unit": "GB/s",
            "frac": ach / hbm["hbm_gbs"], "traffic": None, "peak_src": hbm["src"] + " (burst copy)",
            "work_per_launch": f"{b / 1e6:.2f} MB: {U:.2f} active experts' Q4_K bytes + Q8_K rows in + fp32 rows out",
            "us_per_launch": us, "share": share}


def step_roofline(cfg, ms_step, loads_step, ws, hbm, int8):
    D, E, K, I, T = cfg["D"], cfg["E"], cfg["K"], cfg["I"], cfg["T"]
    n_moe, n_dense = cfg["layers"], cfg.get("dense", 0)
    if is_prefill(cfg):  # int8 ops of the step
        ops = 2.0 * T * K * 3 * I * D * n_moe
        ach = ops / (ms_step / 1e3) / 1e12 / ws
        return {"bound": "tensor", "achieved": ach, "peak": int8["tops"], "unit": "TOP/s (int8) per GPU",
                "frac": ach / int8["tops"], "algorithmic_ops_per_step": ops}
    b = loads_step * expert_bytes(cfg) + n_moe * E * D * 4 + n_dense * dense_bytes(cfg) + 2 * T * D * 4
    ach = b / (ms_step / 1e3) / 1e9 / ws
    return {"bound": "hbm", "achieved": ach, "peak": hbm["hbm_gbs"], "unit": "GB/s per GPU",
            "frac": ach / hbm["hbm_gbs"], "algorithmic_bytes_per_step": b,
            "unique_experts_per_moe_layer": loads_step / max(n_moe, 1)}


def measure(cfg_id, cfg, args, ws, rank, local, use_ep, hbm, int8, steps, warmup, cpu=True):
    """All figures of one config on this rank; returns the JSON fields (rank 0's view)."""
    import torch
    run = StackRun(cfg_id, cfg, ws, rank, local, use_ep, args.ep_comm)
    t = run.timed(steps, warmup)
    T = cfg["T"]
    ms_step = t["ms"] / steps
    share = ws if run.use_ep else 1           # ranks sharing one job's work
    tok_job = T if run.use_ep else ws * T     # tokens all ranks process per step
    value = tok_job * steps / (t["ms"] / 1e3)
    prof_steps = max(1, min(steps, 3))
    prof, loads_prof = run.kernel_profile(prof_steps)
    if not run.use_ep:  # replicas: every rank runs the whole job; count one rank's experts
        loads_prof /= ws
        t["loads"] /= ws
    roof = roofline(cfg, prof, loads_prof, prof_steps, share, hbm, int8)
    sroof = step_roofline(cfg, ms_step, t["loads"] / steps, share, hbm, int8)
    n_e2e = max(3, min(steps, 20))
    e2e_s = run.e2e(n_e2e)
    e2e = tok_job * n_e2e / e2e_s
    par = None if args.no_parity else run.parity(args.parity_tokens)
    out = {"value": value, "ms_per_step": ms_step, "config": workload(cfg_id, cfg),
           "run": {"parallelism": (f"expert-parallel x{ws} (E/{ws} experts and T/{ws} tokens per rank, exchange "
                                   + ("kernels over NVLink peer memory)" if run.p2p else "by NCCL all-to-all)"))
                   if run.use_ep else ("single GPU" if ws == 1 else f"replicas x{ws}"),
                   "tokens_per_rank": run.Tl, "unique_experts_per_moe_layer": t["loads"] / steps / max(cfg["layers"], 1),
                   "layers_in_ring": run.ring if run.single else None},
           "roofline": dict(roof or {}, step=sroof) if roof else sroof,
           "kernel_us_per_launch": {k: round(u, 2) for k, (_, u) in prof.items()},
           "limiting_kernel": limiting_kernel(prof),
           "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": run.Tl * cfg["D"] * 4 * ws,
                   "d2h_bytes_per_step": run.Tl * cfg["D"] * 4 * ws},
           "gpu_launches": t["launches_per_step"] * steps, "clocks": t["clocks"],
           "scaling": "weak" if (run.single or args.replicas) else "strong"}
    if par is not None:
        out["parity"] = par
    run.close()
    del run
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    if cpu and rank == 0 and ws == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline(cfg, seconds=args.cpu_seconds)
    return out


def limiting_kernel(prof):
    """The kernel with the most device time a layer in the per-kernel profile (the slowest rank's
    mean per launch times its launches), and its share of the profiled kernel time."""
    if not prof:
        return None
    tot = {k: n * u for k, (n, u) in prof.items()}
    k = max(tot, key=tot.get)
    return {"kernel": k, "us_per_launch": round(prof[k][1], 2), "share": round(tot[k] / max(sum(tot.values()), 1e-9), 3)}


def run_ours(args, cfg_id, cfg):
    import torch
    ws, rank, local = dist_setup()
    torch.cuda.set_device(local)
    if ws > 1:
        import torch.distributed as dist
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=torch.device("cuda", local), timeout=timedelta(seconds=300))
    hbm = peaks()
    int8 = measure_int8_peak(torch)
    if ws > 1:  # one int8 figure for the job: the slowest rank's
        t = torch.tensor([int8["tops"]], device="cuda", dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MIN)
        int8["tops"] = float(t.item())
    use_ep = ws > 1 and not args.replicas
    m = measure(cfg_id, cfg, args, ws, rank, local, use_ep, hbm, int8, args.steps, args.warmup)
    pre = None
    if args.prefill_config and args.prefill_config != cfg_id:
        from laii_b200.synth import CONFIGS
        pcfg = dict(CONFIGS[args.prefill_config])
        psteps = max(3, min(args.steps, 10))
        pre = measure(args.prefill_config, pcfg, args, ws, rank, local, use_ep, hbm, int8, psteps,
                      max(3, min(args.warmup, 3)), cpu=True)
        pre["steps"], pre["warmup"] = psteps, max(3, min(args.warmup, 3))
    ok = all(b is None or "parity" not in b or b["parity"]["ok"] for b in (m, pre))
    if rank == 0:
        out = {"metric": METRIC, "value": m["value"], "unit": "tok/s", "n_gpus": ws, "steps": args.steps,
               "warmup": args.warmup, "ms_per_step": m["ms_per_step"], "higher_is_better": True,
               "scaling": m["scaling"], "vs_baseline": None, "data": "synthetic (seeded)",
               "dtype": ("u8 x s8 -> s32 (q4_k x q8_k; down q6_k x q8_k), fp32 accum" if cfg.get("down_q6k")
                         else "u8 x s8 -> s32 (q4_k x q8_k), fp32 accum"),
               "config": m["config"], "run": m["run"], "roofline": m["roofline"],
               "cpu_baseline": m.get("cpu_baseline"), "e2e": m["e2e"], "gpu_launches": m["gpu_launches"],
               "clocks": m["clocks"], "kernel_us_per_launch": m["kernel_us_per_launch"],
               "limiting_kernel": m["limiting_kernel"]}
        if "parity" in m:
            out["parity"] = m["parity"]
        if pre is not None:
            out["prefill"] = {k: pre[k] for k in ("config", "run", "value", "ms_per_step", "steps", "warmup",
                                                  "roofline", "e2e", "gpu_launches", "clocks", "kernel_us_per_launch",
                                                  "limiting_kernel", "cpu_baseline", "parity") if k in pre}
            out["prefill"]["unit"] = "tok/s"
        print(json.dumps(out), flush=True)
    if ws > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    if not ok:
        sys.stderr.write("parity check failed\n")
        sys.exit(3)


def main():
    global _ARGS
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", type=int, default=4, choices=[1, 2, 3, 4, 5])
    ap.add_argument("--prefill-config", type=int, default=5, choices=[0, 3, 5],
                    help="config measured as the line's prefill block (0: none)")
    ap.add_argument("--replicas", action="store_true",
                    help="under torchrun: run independent replicas instead of expert parallelism")
    ap.add_argument("--ep-comm", default="p2p", choices=["p2p", "nccl"],
                    help="expert-parallel exchange: the library's peer-memory kernels or torch all_to_all (NCCL)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--ring", type=int, default=8, help="single-layer configs: distinct layers the steps cycle")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parity", action="store_true")
    ap.add_argument("--parity-tokens", type=int, default=4, help="tokens per rank in the parity check")
    ap.add_argument("--down-q6k", action="store_true",
                    help="configs 1-3: the layers' ffn_down_exps in Q6_K (as Q4_K_M checkpoints store some)")
    args = ap.parse_args()
    _ARGS = args
    from laii_b200.synth import CONFIGS
    cfg = dict(CONFIGS[args.config])
    if args.down_q6k:
        if args.config >= 4:
            raise SystemExit("--down-q6k: single-layer configs 1-3 only")
        cfg["down_q6k"] = True
    if args.impl == "reference":
        run_reference(args, args.config, cfg)
    else:
        run_ours(args, args.config, cfg)


if __name__ == "__main__":
    main()
