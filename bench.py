"""Benchmark of the qwen35moe MoE hot path on B200.

Default workload (`--workload prefill4096`): one MoE layer on 4096 bf16 tokens with uniform
routing (~128 tokens per expert) through the tensor-core router and the tcgen05 grouped GEMMs; tokens/s, with the
gate_up GEMM launch against the measured bf16 tensor peak. At N > 1 GPUs (torchrun) it is expert-parallel: rank r
holds 256/N experts and routes its own 4096 tokens per step (weak scaling), with the dispatch and combine
all-to-alls over NCCL, so the scaling run measures the exchange. At N = 1 the line also carries "decode40", the
configs[1] measurement below, taken on the same GPU in the same run.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload prefill4096|decode40|batch64|prefill32k|typed-decode] [--ggml-type T|all]

--workload decode40: decode of one token through 40 stacked MoE layers of the config-0
shapes (H 2048, 256 experts of FFN 512, top-8, Q4_K gate/up + Q6_K down, shared expert), residual + RMSNorm between
layers, all 20.9 GB of expert weights resident in HBM; one step = one token through the 40 layers; the roofline
line reports the expert-weight HBM bandwidth against the measured copy peak. At N > 1 every rank serves its own
token stream with its own full store (decode does not shard: "replicas only").

--workload batch64: 64 f32 tokens through one MoE layer with Zipf-biased routing (the
sliced router, the dispatch sort and the grouped GEMMs); tokens/s and HBM GB/s over the distinct experts each step
touches.

--workload prefill32k: 32768 bf16 tokens through 40 layers with Zipf routing and a 4 GiB
expert store per GPU (experts over the cap stream from pinned host memory, the next layer prefetched); expert
parallel under torchrun. Run with few steps: `--steps 3 --warmup 3`.

--workload typed-decode (the row of the other expert quant types): one token's 8 routed experts in a ggml type of
willow's Metal path (gguf/metal.py:295), through gemv_batch + SwiGLU + gemv_combine as engines/base.py:492-532 runs
them; one JSON line per type (1 GPU), with the gate_up launch against the measured HBM copy peak.

--impl reference times the CPU restatement of willow's own CPU path (the oracle port) on the host cores, on rank 0;
for prefill4096 and decode40 every step is the whole workload (a 4096-token layer, a 40-layer token), for batch64
the whole 64-token block; it emits the same config as this arm. Defaults for it: 20 steps, 5 warm-up.
"""
import argparse
import json
import os
import statistics
import sys
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

HIDDEN, FFN, EXPERTS, TOP_K = 2048, 512, 256, 8
GATE_UP_Q4_BYTES = 2 * FFN * HIDDEN // 256 * 144                              # 1,179,648
EXPERT_BYTES = GATE_UP_Q4_BYTES + HIDDEN * FFN // 256 * 210                    # 2,039,808
ROUTER_BYTES = EXPERTS * HIDDEN * 4 + HIDDEN * 4                           # router + shared gate, fp32
# DRAM bytes (read + write) per layer of decode_kernel, measured by ncu (dram__bytes_read.sum +
# dram__bytes_write.sum) on a 4-layer launch: 82,377,984 + 2,413,824 bytes; traffic grows with the layers
TRAFFIC_PER_LAYER = (82_377_984 + 2_413_824) / 4
# DRAM bytes (read + write) of one grouped_gemm_kernel<0> launch at 4096 tokens, measured by ncu
# (dram__bytes_read.sum + dram__bytes_write.sum = 454,209,280 + 31,324,928): the gathered activations (151 MB) and the
# Q4_K weights (303 MB) read once, h written
PREFILL_GATE_UP_TRAFFIC = 454_209_280 + 31_324_928
LAYERS = 40
SEED = 0
METRIC = "MoE decode tokens/s (40-layer qwen35moe stack, 1 token per step)"
BATCH_T = 64
METRIC_BATCH = "MoE batched-decode tokens/s (one qwen35moe MoE layer, 64 f32 tokens per step, Zipf routing)"
PREFILL_T = 4096
METRIC_PREFILL = "MoE prefill tokens/s (one qwen35moe MoE layer, 4096 bf16 tokens per step)"
# useful expert-product FLOPs of one prefill layer: every token through 8 routed experts + the shared expert,
# gate_up [2F x H] then down [H x F]
PF32_T = 32768
PF32_CAP = 4 << 30  # expert-store cap per GPU
METRIC_PF32 = ("MoE prefill tokens/s (40-layer qwen35moe stack, 32768 bf16 tokens per step, Zipf routing, "
               "4 GiB expert store per GPU)")
GATE_UP_FLOPS = 2 * PREFILL_T * (TOP_K + 1) * (2 * FFN) * HIDDEN   # 154.6 GFLOP
DOWN_FLOPS = 2 * PREFILL_T * (TOP_K + 1) * HIDDEN * FFN             # 77.3 GFLOP


def peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def workload_config(workload: str, world: int, n_layers: int = LAYERS, type_name: str = "") -> dict:
    """The `config` object of a workload's JSON line: the same dict for this GPU arm and for --impl reference at the
    same N (it names the work, not what a run measured)."""
    base = {"hidden": HIDDEN, "experts": EXPERTS, "ffn": FFN, "top_k": TOP_K}
    if workload == "decode40":
        return {"workload": ("configs[1]: decode 1 token x 40 MoE layers, all experts resident" if n_layers == LAYERS
                             else f"profiling case: decode 1 token x {n_layers} layers (not the benchmark)"),
                **base, "layers": n_layers, "tokens_per_step": 1,
                "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                "l2": "inputs larger than L2: 734 MB of expert weights per step, a new token (new routing) each step"}
    if workload == "batch64":
        return {"workload": "configs[2]: 64 tokens through one MoE layer, Zipf-biased routing", **base,
                "tokens_per_step": BATCH_T, "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                "l2": "16 batches cycled: each step re-routes (distinct experts per step in roofline_step)"}
    if workload == "prefill4096":
        if world == 1:
            return {"workload": "configs[3]: prefill 4096 tokens through one MoE layer, uniform routing", **base,
                    "tokens_per_step": PREFILL_T, "parallelism": "single GPU",
                    "l2": "inputs larger than L2: 524 MB of expert weights and ~500 MB of activations per step"}
        return {"workload": "configs[3]: prefill 4096 tokens per rank through one MoE layer, uniform routing", **base,
                "tokens_per_step": PREFILL_T * world, "parallelism": f"ep{world}",
                "experts_per_rank": EXPERTS // world,
                "l2": "inputs larger than L2: ~500 MB of activations per rank per step"}
    if workload == "prefill32k":
        return {"workload": "configs[4]: prefill 32768 tokens through 40 MoE layers, Zipf routing, 4 GiB cap", **base,
                "layers": n_layers, "tokens_per_step": PF32_T, "tokens_per_rank": PF32_T // world,
                "parallelism": f"ep{world}" if world > 1 else "single GPU", "experts_per_rank": EXPERTS // world,
                "store_cap_bytes": PF32_CAP, "store_slots": int(PF32_CAP // ((EXPERT_BYTES + 255) // 256 * 256)),
                "hot_share": 0.75, "batches_cycled": 2,
                "l2": "inputs larger than L2: 268 MB residual stream per rank and up to 21 GB of experts"}
    if workload == "typed-decode":
        return {"workload": f"typed-decode {type_name}: gemv_batch (gate_up [1024, 2048]) + SwiGLU + gemv_combine "
                            "(down [2048, 512]) for 8 experts per step", "ggml_type": type_name,
                "l2": "inputs larger than L2: each step reads 8 other experts of a >= 2 GB pool"}
    raise ValueError(workload)


def pipelined_e2e(torch, run, x_hosts, K: int, dist=None) -> float:
    """Milliseconds per step of K end-to-end steps whose copies overlap the compute of neighbouring steps, as a
    serving loop double-buffers them: step s's input is copied in from pinned host memory on one copy stream and
    its result read back into pinned host memory on another, while step s - 1 or s + 1 computes on the current
    stream. Every step copies its whole input in and its whole result out inside the timed region; two device input
    buffers and two pinned result buffers, ordered by events (an input buffer is rewritten only after the step that
    read it, a result only after its read-back). run(x_dev, b) enqueues one step on the current stream and returns
    its device result (buffer b of two, or a fresh tensor)."""
    comp = torch.cuda.current_stream()
    h2d, d2h = torch.cuda.Stream(), torch.cuda.Stream()
    x_dev = [torch.empty_like(x_hosts[0], device="cuda") for _ in range(2)]
    # one untimed step per buffer: the pinned result buffers are allocated (a synchronous host allocation) before
    # the timed region
    o_host = []
    for b in range(2):
        x_dev[b].copy_(x_hosts[b % len(x_hosts)])
        out = run(x_dev[b], b)
        o_host.append(torch.empty(out.shape, dtype=out.dtype).pin_memory())
    ev_in = [torch.cuda.Event() for _ in range(2)]    # input b landed
    ev_used = [torch.cuda.Event() for _ in range(2)]  # the step on input b is done
    ev_out = [torch.cuda.Event() for _ in range(2)]   # result b read back
    for b in range(2):
        ev_used[b].record(comp)
        ev_out[b].record(comp)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(comp)
    h2d.wait_stream(comp)
    d2h.wait_stream(comp)
    for s in range(K):
        b = s % 2
        h2d.wait_event(ev_used[b])
        with torch.cuda.stream(h2d):
            x_dev[b].copy_(x_hosts[s % len(x_hosts)], non_blocking=True)
        ev_in[b].record(h2d)
        comp.wait_event(ev_in[b])
        comp.wait_event(ev_out[b])
        out = run(x_dev[b], b)
        ev_used[b].record(comp)
        out.record_stream(d2h)
        d2h.wait_event(ev_used[b])
        with torch.cuda.stream(d2h):
            o_host[b].copy_(out, non_blocking=True)
        ev_out[b].record(d2h)
    comp.wait_stream(h2d)
    comp.wait_stream(d2h)
    e1.record(comp)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / K


class ClockSampler:
    """SM clocks and clock-event (throttle) reasons of the bench's GPU, read through NVML every ~2 ms on a thread
    while the timed region runs, plus once on entry and once on exit, so that even a region of a few milliseconds
    has samples. Reads only; no GPU setting is changed."""
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown"}

    def __init__(self, device: int):
        self.device = device
        self.samples, self.max_mhz, self.reasons = [], None, set()
        self.handle = None
        try:
            import pynvml
            import torch
            pynvml.nvmlInit()
            prop = torch.cuda.get_device_properties(device)
            bus = f"{prop.pci_domain_id:08x}:{prop.pci_bus_id:02x}:{prop.pci_device_id:02x}.0"
            try:
                self.handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            except pynvml.NVMLError:
                self.handle = pynvml.nvmlDeviceGetHandleByIndex(device)
            self.nvml = pynvml
        except Exception:
            self.handle = None

    def _sample(self):
        n = self.nvml
        self.samples.append(float(n.nvmlDeviceGetClockInfo(self.handle, n.NVML_CLOCK_SM)))
        mask = n.nvmlDeviceGetCurrentClocksThrottleReasons(self.handle)
        self.reasons |= {name for bit, name in self.REASONS.items() if mask & bit}

    def _loop(self):
        while not self.stop.wait(0.002):
            try:
                self._sample()
            except Exception:
                return

    def __enter__(self):
        if self.handle is not None:
            import threading
            try:
                self.max_mhz = float(self.nvml.nvmlDeviceGetMaxClockInfo(self.handle, self.nvml.NVML_CLOCK_SM))
                self._sample()
            except Exception:
                self.handle = None
                return self
            self.stop = threading.Event()
            self.thread = threading.Thread(target=self._loop, daemon=True)
            self.thread.start()
        return self

    def __exit__(self, *exc):
        if self.handle is not None:
            self.stop.set()
            self.thread.join()
            try:
                self._sample()
            except Exception:
                pass

    def summary(self):
        sm = self.samples
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(sm), "source": "NVML, ~2 ms"}


def setup_model(device: int, n_layers: int = LAYERS):
    """The model on the GPU: synthetic routed experts generated in HBM, router/shared weights uploaded."""
    import torch
    from willow_v2_b200 import moe, synth
    ctx = moe.Context(device)
    store = moe.ExpertStore(n_layers, EXPERTS, HIDDEN, FFN, ctx=ctx)
    store.fill_synthetic(SEED)
    layers = []
    for l in range(n_layers):
        layers.append(moe.LayerWeights(
            router_w=torch.from_numpy(synth.router_weight(SEED, l)).cuda(),
            shared_gate=torch.from_numpy(synth.shared_gate_weight(SEED, l)).cuda(),
            shared_gate_up=torch.from_numpy(synth.expert_gate_up(SEED, l, EXPERTS).reshape(-1)).cuda(),
            shared_down=torch.from_numpy(synth.expert_down(SEED, l, EXPERTS).reshape(-1)).cuda()))
    torch.cuda.synchronize()
    return ctx, store, layers


def run_decode40(args, rank: int, world: int, dist):
    import torch
    from willow_v2_b200 import moe, synth
    device = torch.cuda.current_device()
    n_layers = args.layers
    ctx, store, layers = setup_model(device, n_layers)
    K, W = args.steps, args.warmup
    # a new token per step (different routing every step); inputs resident before the timed region
    h_all = torch.from_numpy(np.concatenate([synth.hidden(SEED + 1000 * rank, 1, step=s) for s in range(K + W)])).cuda()
    out = torch.empty(HIDDEN, dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream()
    for s in range(W):
        moe.decode_stack(store, layers, h_all[s], 1e-6, out=out)
    torch.cuda.synchronize()
    ctx.check_device()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    launches0 = ctx.launches
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(device) as clocks:
        ev0.record(stream)
        for s in range(K):
            moe.decode_stack(store, layers, h_all[W + s], 1e-6, out=out)
        ev1.record(stream)
        torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    gpu_launches = ctx.launches - launches0
    ms = ev0.elapsed_time(ev1) / K
    ctx.check_device()

    # end to end through the public API: pinned host input -> device, decode, result -> pinned host, every step
    h_host = torch.from_numpy(np.concatenate([synth.hidden(SEED + 7 + 1000 * rank, 1, step=s)
                                              for s in range(K)])).pin_memory()
    o_host = torch.empty(K, HIDDEN, dtype=torch.float32).pin_memory()
    h_dev = torch.empty(HIDDEN, dtype=torch.float32, device="cuda")
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for s in range(K):
        h_dev.copy_(h_host[s], non_blocking=True)
        moe.decode_stack(store, layers, h_dev, 1e-6, out=out)
        o_host[s].copy_(out, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / K

    times = torch.tensor([ms, e2e_ms], dtype=torch.float64, device="cuda")
    if dist:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    ms, e2e_ms = times.tolist()
    hbm, _, peak_kind = peaks()
    expert_bytes = n_layers * (TOP_K + 1) * EXPERT_BYTES
    achieved = expert_bytes / (ms * 1e-3) / 1e9
    result = {
        "metric": METRIC, "value": world * 1e3 / ms, "unit": "tokens/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded GGUF Q4_K/Q6_K blocks with the config-0 distributions; random-init router)",
        "config": workload_config("decode40", world, n_layers),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "traffic": n_layers * TRAFFIC_PER_LAYER, "peak_kind": peak_kind,
                     "algorithmic_bytes_per_launch": expert_bytes,
                     "frac_of_8TBps": achieved / 8000.0,
                     "all_bytes_per_launch": expert_bytes + n_layers * ROUTER_BYTES},
        "e2e": {"value": world * 1e3 / e2e_ms, "unit": "tokens/s", "h2d_bytes_per_step": HIDDEN * 4,
                "d2h_bytes_per_step": HIDDEN * 4},
        "gpu_launches": int(gpu_launches),
        "clocks": clocks.summary(),
    }
    return result, (ctx, store, layers)


def run_batch64(args, rank: int, world: int, dist):
    """64 independent f32 tokens through one MoE layer with the Zipf(s=1.1) routing bias: the split-K
    float32 router, the dispatch sort and the tcgen05 grouped GEMMs (64 tokens is above the default GEMM threshold of
    16). HBM roofline over the distinct experts hit by each step's routing (each expert's bytes counted once, however
    many tokens use it), plus the router."""
    import torch
    from willow_v2_b200 import lib as L
    from willow_v2_b200 import moe, synth
    device = torch.cuda.current_device()
    ctx, store, layers = setup_model(device, 1)
    lw = layers[0]
    lw.router_bias = torch.from_numpy(synth.zipf_bias(SEED)).cuda()
    K, W = args.steps, args.warmup
    T = BATCH_T
    nb = 16  # batches cycled; each step re-routes
    xs = [torch.from_numpy(synth.hidden(SEED + 1000 * rank, T, step=b)).cuda() for b in range(nb)]
    out = torch.empty(T, HIDDEN, dtype=torch.float32, device="cuda")
    sel = torch.empty(T, TOP_K, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream()
    weights = lw.as_struct()

    def step(x, o, s):
        L.check(ctx.handle, L.lib.wmoe_moe_forward_layer(ctx.handle, store.handle, 0, x.data_ptr(), L.F32, T, TOP_K,
                                                         L.ctypes.byref(weights), o.data_ptr(), L.F32,
                                                         None if s is None else s.data_ptr(), None,
                                                         stream.cuda_stream))

    # distinct experts per batch (the algorithmic bytes), from the same routing the timed steps use
    distinct = []
    for b in range(nb):
        step(xs[b], out, sel)
        distinct.append(int(torch.unique(sel).numel()))
    for s in range(W):
        step(xs[s % nb], out, None)
    torch.cuda.synchronize()
    ctx.check_device()
    L.check(ctx.handle, L.lib.wmoe_set_profiling(ctx.handle, K))
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    launches0 = ctx.launches
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(device) as clocks:
        ev0.record(stream)
        for s in range(K):
            step(xs[s % nb], out, None)
        ev1.record(stream)
        torch.cuda.synchronize()
    gpu_launches = ctx.launches - launches0
    ms = ev0.elapsed_time(ev1) / K
    phase = {name: [] for name in L.PHASES}
    for ago in range(K):
        for p, name in enumerate(L.PHASES):
            v = L.ctypes.c_float()
            L.check(ctx.handle, L.lib.wmoe_phase_ms(ctx.handle, ago, p, L.ctypes.byref(v)))
            phase[name].append(v.value)
    L.check(ctx.handle, L.lib.wmoe_set_profiling(ctx.handle, 0))
    phase_ms = {name: statistics.mean(v) for name, v in phase.items()}
    ctx.check_device()
    x_host = [x.cpu().pin_memory() for x in xs]
    o_host = torch.empty(T, HIDDEN, dtype=torch.float32).pin_memory()
    x_dev = torch.empty(T, HIDDEN, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for s in range(K):
        x_dev.copy_(x_host[s % nb], non_blocking=True)
        step(x_dev, out, None)
        o_host.copy_(out, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / K
    times = torch.tensor([ms, e2e_ms, phase_ms["gate_up"]], dtype=torch.float64, device="cuda")
    if dist:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    ms, e2e_ms, gu_ms = times.tolist()
    hbm, _, peak_kind = peaks()
    mean_u = statistics.mean(distinct[s % nb] for s in range(K))
    nbytes = (mean_u + 1) * EXPERT_BYTES + ROUTER_BYTES
    # the gate_up launch: Q4_K blocks of the hit experts + shared, gathered fp16 rows in, fp16 h rows out
    rows = T * (TOP_K + 1)
    gu_bytes = (mean_u + 1) * GATE_UP_Q4_BYTES + rows * HIDDEN * 2 + rows * FFN * 2
    gu_gbs = gu_bytes / (gu_ms * 1e-3) / 1e9
    achieved = nbytes / (ms * 1e-3) / 1e9
    result = {
        "metric": METRIC_BATCH, "value": world * T * 1e3 / ms, "unit": "tokens/s", "n_gpus": world, "steps": K,
        "warmup": W, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic (seeded GGUF Q4_K/Q6_K blocks; f32 N(0,1) tokens; Zipf(1.1) routing bias)",
        "config": workload_config("batch64", world),
        "roofline": {"bound": "hbm", "kernel": "grouped_gemm_kernel<0> (gate_up + SwiGLU)", "achieved": gu_gbs,
                     "peak": hbm, "unit": "GB/s", "frac": gu_gbs / hbm, "traffic": None, "peak_kind": peak_kind,
                     "algorithmic_bytes_per_launch": gu_bytes, "launch_ms": gu_ms},
        "roofline_step": {"achieved": achieved, "frac": achieved / hbm, "algorithmic_bytes": nbytes,
                          "distinct_experts_mean": mean_u,
                          "note": "whole step (all launches); bytes = distinct experts hit + shared + router"},
        "phase_ms": phase_ms,
        "e2e": {"value": world * T * 1e3 / e2e_ms, "unit": "tokens/s", "h2d_bytes_per_step": T * HIDDEN * 4,
                "d2h_bytes_per_step": T * HIDDEN * 4},
        "gpu_launches": int(gpu_launches),
        "clocks": clocks.summary(),
    }
    return result, (ctx, store, layers)


# ---------------------------------------------------------------------------------------------- CPU baseline pool
# The CPU baseline and the reference arm run the oracle port (numpy float32) on every host core: a process pool with
# one BLAS thread per worker, each expert's dequantisation + FFN one task, timed by the wall clock around the pool.
# The pool is spawned (no GPU state is inherited). Dequantisation costs the same whatever the bytes are, so each
# worker generates a few synthetic expert blobs once (untimed) and a task names one by index: the per-task IPC is
# the activation rows only.
N_BLOBS = 16
_POOL = None
_BLOBS = {}


def cpu_baseline_pool():
    """(pool, workers): the spawned process pool of the CPU baseline, started once per process."""
    global _POOL
    try:
        n = len(os.sched_getaffinity(0))  # the cores this process may run on
    except AttributeError:
        n = os.cpu_count() or 1
    n = max(1, min(n, 64))  # each worker holds ~60 MB of expert blobs
    if _POOL is None:
        import concurrent.futures
        import multiprocessing
        keys = ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS")
        saved = {k: os.environ.get(k) for k in keys}
        os.environ.update({k: "1" for k in keys})  # inherited by the workers spawned below, not by this process
        try:
            _POOL = concurrent.futures.ProcessPoolExecutor(n, mp_context=multiprocessing.get_context("spawn"),
                                                           initializer=_worker_init)
            pids = set(_POOL.map(_warm, range(4 * n)))  # every worker started (its blobs made) before any timing
            if len(pids) < n:
                pids |= set(_POOL.map(_warm, range(8 * n)))
        finally:
            for k, v in saved.items():
                if v is None:
                    os.environ.pop(k, None)
                else:
                    os.environ[k] = v
    return _POOL, n


def shutdown_cpu_pool():
    """Stops the CPU-baseline pool before the interpreter exits (its exit hooks otherwise run on torn-down modules)."""
    global _POOL
    if _POOL is not None:
        _POOL.shutdown(wait=True)
        _POOL = None


def _worker_init():
    from oracle import ggml_types as G
    from willow_v2_b200 import synth
    for i in range(N_BLOBS):
        _BLOBS[("Q4_K/Q6_K", i)] = (synth.expert_gate_up(SEED, 0, i), synth.expert_down(SEED, 0, i))
    for t in G.TYPES:  # one expert per type for the typed baseline (tasks of a type all name blob 0)
        _typed_blob(t, 0)


def _typed_blob(type_name: str, i: int):
    key = (type_name, i)
    if key not in _BLOBS:
        from oracle import ggml_types as G
        elements, size = G.BLOCKS[type_name]
        rng = np.random.default_rng(SEED + i)
        gu = rng.integers(0, 256, (2 * FFN * HIDDEN // elements, size), dtype=np.uint8)
        dn = rng.integers(0, 256, (HIDDEN * FFN // elements, size), dtype=np.uint8)
        d_at = TYPED_D_AT.get(type_name, 0)
        for b in (gu, dn):
            for off in ((d_at, 2) if type_name == "Q4_K" else (d_at,)):
                b[:, off:off + 2] = rng.uniform(1e-3, 4e-3, b.shape[0]).astype(np.float16).view(np.uint8).reshape(-1, 2)
        _BLOBS[key] = (gu, dn)
    return _BLOBS[key]


def _ffn_task(task):
    """One expert of the oracle port: dequantise its gate_up / down blocks and run its FFN on `rows` (float32
    [n, H]). Returns the output rows when `keep`, else their sum."""
    kind, i, rows, keep = task
    if kind == "Q4_K/Q6_K":
        import oracle.moe_oracle as ora
        gu, dn = _BLOBS[(kind, i)]
        wg, wd = ora.dequantize(gu, "Q4_K", (2 * FFN, HIDDEN)), ora.dequantize(dn, "Q6_K", (HIDDEN, FFN))
    else:
        from oracle import ggml_types as G
        gu, dn = _typed_blob(kind, i)
        wg, wd = G.dequantize(gu, kind, (2 * FFN, HIDDEN)), G.dequantize(dn, kind, (HIDDEN, FFN))
    a = rows @ wg.T
    g = a[:, :FFN]
    y = (g / (1 + np.exp(-np.clip(g, -80, 80))) * a[:, FFN:]) @ wd.T
    return y if keep else float(y.sum())


_SHM = {}


def _shm_array(name: str, shape):
    """A float32 array over a named shared-memory block (attached once per process)."""
    from multiprocessing import shared_memory
    if name not in _SHM:
        _SHM[name] = shared_memory.SharedMemory(name=name)
    return np.ndarray(shape, dtype=np.float32, buffer=_SHM[name].buf)


def _prefill_task(task):
    """One expert of a whole prefill layer: rows idx of the shared token matrix through its FFN, written to rows
    [off, off + len(idx)) of the shared output matrix."""
    blob, x_name, T, idx, y_name, P, off = task
    x = _shm_array(x_name, (T, HIDDEN))
    y = _shm_array(y_name, (P, HIDDEN))
    y[off:off + len(idx)] = _ffn_task(("Q4_K/Q6_K", blob, x[idx], True))
    return len(idx)


def _warm(_):
    time.sleep(0.05)  # long enough that the 4n warm-up tasks spread over every worker (each past its initializer)
    return os.getpid()


def cpu_baseline_wall(tasks):
    """Runs the tasks on the pool; (wall seconds, results)."""
    pool, _ = cpu_baseline_pool()
    t0 = time.perf_counter()
    out = list(pool.map(_ffn_task, tasks))
    return time.perf_counter() - t0, out


def cpu_baseline_decode_layer(x_norm, router, layer_step: int):
    """One decode layer of the oracle port on the pool: router + top-8 in this process, the 8 routed experts and the
    shared expert in parallel, then the combine in ascending expert id. Returns (seconds it took, output)."""
    import oracle.moe_oracle as ora
    t0 = time.perf_counter()
    w, sel = ora.route(x_norm @ router.T)
    order = np.argsort(sel[0], kind="stable")
    t_route = time.perf_counter() - t0
    tasks = [("Q4_K/Q6_K", (int(sel[0, j]) + layer_step) % N_BLOBS, x_norm, True) for j in order]
    tasks.append(("Q4_K/Q6_K", layer_step % N_BLOBS, x_norm, True))  # the shared expert
    t_pool, ys = cpu_baseline_wall(tasks)
    t1 = time.perf_counter()
    out = np.zeros_like(x_norm)
    for j, y in zip(order, ys[:-1]):
        out += w[0, j] * y
    out += ys[-1]  # the shared expert (its sigmoid gate is a dot product: negligible)
    return t_route + t_pool + (time.perf_counter() - t1), out


def cpu_baseline_batch():
    """The oracle port for configs[2] on every host core: the router on the 64 tokens, then every hit expert (and the
    shared expert) dequantised and run on its tokens, in parallel on the pool."""
    import oracle.moe_oracle as ora
    from willow_v2_b200 import synth
    _, workers = cpu_baseline_pool()
    x = synth.hidden(SEED, BATCH_T, step=777)
    router = synth.router_weight(SEED, 0)
    bias = synth.zipf_bias(SEED)
    t0 = time.perf_counter()
    w, sel = ora.route(x @ router.T + bias)
    t_route = time.perf_counter() - t0
    hit = sorted(set(int(e) for e in sel.reshape(-1)))
    tasks = [("Q4_K/Q6_K", e % N_BLOBS, x[(sel == e).any(axis=1)], False) for e in hit]
    tasks.append(("Q4_K/Q6_K", 0, x, False))  # the shared expert on every token
    t_pool, _ = cpu_baseline_wall(tasks)
    sec = t_route + t_pool
    return {"value": BATCH_T / sec, "unit": "tokens/s", "cores": workers, "kind": "port",
            "sample": f"router on the 64 tokens; the {len(hit)} hit experts + the shared expert dequantised and run "
                      f"on their tokens in parallel on {workers} worker processes (numpy float32)"}


def run_prefill4096_ep(args, rank: int, world: int, dist):
    """configs[3] expert-parallel: rank r holds experts [r * 256 / N, (r + 1) * 256 / N) and routes its own 4096
    tokens per step (weak scaling); dispatch and combine are the library's exchanges (moe_forward_ep_native: count
    all-gather, copy-engine copies into the peers' windows), with its per-phase CUDA events."""
    import torch
    from willow_v2_b200 import moe, synth
    device = torch.cuda.current_device()
    ctx = moe.Context(device)
    per = EXPERTS // world
    store = moe.ExpertStore(1, EXPERTS, HIDDEN, FFN, ctx=ctx, expert_range=(rank * per, (rank + 1) * per))
    store.fill_synthetic(SEED)
    lw = moe.LayerWeights(router_w=torch.from_numpy(synth.router_weight(SEED, 0)).cuda(),
                          shared_gate=torch.from_numpy(synth.shared_gate_weight(SEED, 0)).cuda(),
                          shared_gate_up=torch.from_numpy(synth.expert_gate_up(SEED, 0, EXPERTS).reshape(-1)).cuda(),
                          shared_down=torch.from_numpy(synth.expert_down(SEED, 0, EXPERTS).reshape(-1)).cuda()
                          ).prepare(ctx, decode=False)
    K, W = args.steps, args.warmup
    T = PREFILL_T
    xs = [torch.from_numpy(synth.hidden(SEED + 1000 * rank, T, step=b)).to(torch.bfloat16).cuda() for b in range(4)]
    stream = torch.cuda.current_stream()
    from willow_v2_b200 import lib as L
    if args.ep_exchange == "nccl":
        os.environ["WMOE_EP_NCCL_ROWS"] = "1"
    elif args.ep_exchange == "copy":
        os.environ.pop("WMOE_EP_NCCL_ROWS", None)
    moe.ep_init(ctx)
    if args.ep_chunks is not None:
        L.lib.wmoe_ep_set_chunks(ctx.handle, args.ep_chunks)
    chunks = L.lib.wmoe_ep_set_chunks(ctx.handle, 1)  # read the setting back
    L.lib.wmoe_ep_set_chunks(ctx.handle, chunks)
    rows = "copy engines into IPC windows" if L.lib.wmoe_ep_uses_copy_engines(ctx.handle) == 1 else "NCCL send/recv"
    for s in range(W):
        moe.moe_forward_ep_native(store, 0, xs[s % 4], lw)
    torch.cuda.synchronize()
    ctx.check_device()
    # one step through the torch.distributed orchestration for the transfer sizes (not timed)
    sizes = dict()
    moe.moe_forward_ep(store, 0, xs[0], lw, stats=sizes)
    pairs_in = sizes["pairs_in"]
    bytes_out = (sizes["rows_out"] + sizes["pairs_out"]) * HIDDEN * 2
    dist.barrier()
    torch.cuda.synchronize()
    L.check(ctx.handle, L.lib.wmoe_set_profiling(ctx.handle, K))
    launches0 = ctx.launches
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(device) as clocks:
        ev0.record(stream)
        for s in range(K):
            moe.moe_forward_ep_native(store, 0, xs[s % 4], lw)
        ev1.record(stream)
        torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    gpu_launches = ctx.launches - launches0
    ms = ev0.elapsed_time(ev1) / K
    stage = {name: [] for name in L.EP_PHASES}
    for ago in range(K):
        for p, name in enumerate(L.EP_PHASES):
            v = L.ctypes.c_float()
            L.check(ctx.handle, L.lib.wmoe_phase_ms(ctx.handle, ago, p, L.ctypes.byref(v)))
            stage[name].append(v.value)
    L.check(ctx.handle, L.lib.wmoe_set_profiling(ctx.handle, 0))
    stage_ms = {k: statistics.mean(v) for k, v in stage.items()}
    ctx.check_device()

    # end to end: pinned bf16 host batch -> device, layer, result -> pinned host, every step, the copies of
    # neighbouring steps overlapping the layer (pipelined_e2e)
    x_host = [x.cpu().pin_memory() for x in xs]
    e2e_ms = pipelined_e2e(torch, lambda x_dev, b: moe.moe_forward_ep_native(store, 0, x_dev, lw), x_host, K, dist)
    ctx.ep_finalize()
    dist.barrier()
    experts_ms = stage_ms.get("experts", float("nan"))
    a2a_ms = stage_ms.get("first_rows", 0.0) + stage_ms.get("last_results", 0.0)  # exchange time not overlapped
    times = torch.tensor([ms, e2e_ms, experts_ms, a2a_ms], dtype=torch.float64, device="cuda")
    dist.all_reduce(times, op=dist.ReduceOp.MAX)
    ms, e2e_ms, experts_ms_max, a2a_ms_max = times.tolist()
    _, bf16, peak_kind = peaks()
    flops = (pairs_in + T) * 6_291_456  # this rank's expert products: received pairs + its shared-expert rows
    tflops = flops / (experts_ms * 1e-3) / 1e12
    link = 770.0  # GB/s per direction per GPU, measured peer copy on this pool
    result = {
        "metric": METRIC_PREFILL, "value": world * T * 1e3 / ms, "unit": "tokens/s", "n_gpus": world, "steps": K,
        "warmup": W, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16 in/out, fp16 tensor-core operands, fp32 accumulation",
        "data": "synthetic (seeded GGUF Q4_K/Q6_K blocks with the config-0 distributions; bf16 N(0,1) tokens)",
        "config": workload_config("prefill4096", world),
        "roofline": {"bound": "tensor",
                     "kernel": "expert stages (dispatch + gather + grouped GEMMs, all chunks), rank 0",
                     "achieved": tflops, "peak": bf16, "unit": "TFLOP/s", "frac": tflops / bf16, "traffic": None,
                     "peak_kind": peak_kind, "algorithmic_flops_per_launch": flops, "launch_ms": experts_ms},
        "exchange": {"bytes_out_per_step": bytes_out, "exposed_ms_max": a2a_ms_max,
                     "link_gbs_ref": link, "chunks": chunks,
                     "rows": rows,
                     "note": "exchanges run on a second stream overlapping the expert stages; exposed = waits"},
        "stage_ms_rank0": stage_ms,
        "e2e": {"value": world * T * 1e3 / e2e_ms, "unit": "tokens/s", "h2d_bytes_per_step": T * HIDDEN * 2,
                "d2h_bytes_per_step": T * HIDDEN * 2,
                "copies": "every step's input in and result out inside the timed region, on two copy streams "
                          "overlapping the neighbouring steps' compute (double buffers ordered by events)"},
        "gpu_launches": int(gpu_launches),
        "clocks": clocks.summary(),
    }
    return result, (ctx, store, lw)


def run_prefill32k(args, rank: int, world: int, dist):
    """32768 bf16 tokens (32768 / N per rank) through 40 MoE layers with Zipf(1.1)-biased routing (a
    per-layer permutation), experts partitioned 256/N per GPU, each GPU's expert store capped at 4 GiB: the experts
    over the cap live in pinned host memory and stream in on the store's side stream. While layer l runs, layer
    l + 1's experts are prefetched (a prefill batch reads most of them); after the first warm-up pass, 75% of the
    slots keep the hot set chosen by token counts (store.py:464-484). The whole stack is one wmoe_prefill_stack
    call: residual + RMSNorm in each layer's combine kernel, the next layer's prefetch issued by the library. Strong
    scaling: the 32768 tokens are split over the ranks."""
    import torch
    from willow_v2_b200 import moe, synth
    device = torch.cuda.current_device()
    ctx = moe.Context(device)
    per = EXPERTS // world
    n_layers = args.layers
    store = moe.ExpertStore(n_layers, EXPERTS, HIDDEN, FFN, cap_bytes=PF32_CAP, ctx=ctx,
                            expert_range=(rank * per, (rank + 1) * per))
    store.fill_synthetic(SEED)
    lws = [moe.LayerWeights(router_w=torch.from_numpy(synth.router_weight(SEED, l)).cuda(),
                            shared_gate=torch.from_numpy(synth.shared_gate_weight(SEED, l)).cuda(),
                            shared_gate_up=torch.from_numpy(synth.expert_gate_up(SEED, l, EXPERTS).reshape(-1)).cuda(),
                            shared_down=torch.from_numpy(synth.expert_down(SEED, l, EXPERTS).reshape(-1)).cuda(),
                            router_bias=torch.from_numpy(synth.zipf_bias(SEED + l)).cuda()).prepare(ctx, decode=False)
           for l in range(n_layers)]
    T = PF32_T // world
    # two token batches cycled: each step routes a different batch (the prefetch guess sees only earlier steps)
    h0s = [torch.from_numpy(synth.hidden(SEED, PF32_T, step=99 + b)[rank * T:(rank + 1) * T]).cuda() for b in range(2)]
    h = torch.empty_like(h0s[0])
    stream = torch.cuda.current_stream()
    if world > 1:  # every layer of the stack then runs over the library's communicator (its chunk count)
        moe.ep_init(ctx)

    def stack(h):  # h <- h + moe(rms_norm(h)) for every layer, in place; bf16 block inputs
        return moe.prefill_stack(store, lws, h, x_dtype=torch.bfloat16, out=h)

    K, W = args.steps, args.warmup
    for s in range(W):
        h.copy_(h0s[s % 2])
        stack(h)
        if s == 0:
            store.choose_hot(0.75)  # usage of the first pass
    torch.cuda.synchronize()
    ctx.check_device()
    # pinned host -> device bandwidth of this GPU, for the H2D roofline
    pin = torch.empty(1 << 30, dtype=torch.uint8).pin_memory()
    dev = torch.empty(1 << 30, dtype=torch.uint8, device="cuda")
    dev.copy_(pin, non_blocking=True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    dev.copy_(pin, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    h2d_peak = (1 << 30) / (e0.elapsed_time(e1) * 1e-3) / 1e9
    del pin, dev
    st0 = store.stats()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    launches0 = ctx.launches
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(device) as clocks:
        ev0.record(stream)
        for s in range(K):
            h.copy_(h0s[(W + s) % 2])
            stack(h)
        ev1.record(stream)
        torch.cuda.synchronize()
    gpu_launches = ctx.launches - launches0
    ms = ev0.elapsed_time(ev1) / K
    st1 = store.stats()
    ctx.check_device()
    # end to end through the public calls: the step's tokens from pinned host memory, the result back, every step
    h_host = [x.cpu().pin_memory() for x in h0s]
    o_host = torch.empty_like(h_host[0]).pin_memory()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    for s in range(K):
        h.copy_(h_host[s % 2], non_blocking=True)
        o_host.copy_(stack(h), non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / K
    ctx.check_device()
    if world > 1:
        ctx.ep_finalize()
    bytes_in = (st1["bytes_in"] - st0["bytes_in"]) / K
    calls = (st1["hits"] + st1["misses"]) - (st0["hits"] + st0["misses"])
    hit_rate = (st1["hits"] - st0["hits"]) / calls if calls else 1.0
    times = torch.tensor([ms, e2e_ms], dtype=torch.float64, device="cuda")
    if dist:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    ms, e2e_ms = times.tolist()
    _, bf16, peak_kind = peaks()
    flops = n_layers * PF32_T * (TOP_K + 1) * 6_291_456 // world  # this rank's share of the expert products
    tflops = flops / (ms * 1e-3) / 1e12
    h2d_gbs = bytes_in / (ms * 1e-3) / 1e9
    result = {
        "metric": METRIC_PF32, "value": PF32_T * 1e3 / ms, "unit": "tokens/s", "n_gpus": world, "steps": K,
        "warmup": W, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "bf16 in/out, fp16 tensor-core operands, fp32 accumulation",
        "data": "synthetic (seeded GGUF Q4_K/Q6_K blocks; bf16 N(0,1) tokens; per-layer Zipf(1.1) routing bias)",
        "config": workload_config("prefill32k", world, n_layers),
        "roofline": {"bound": "tensor", "kernel": "whole 40-layer step (expert products / step time), rank 0",
                     "achieved": tflops, "peak": bf16, "unit": "TFLOP/s", "frac": tflops / bf16, "traffic": None,
                     "peak_kind": peak_kind, "algorithmic_flops_per_launch": flops, "launch_ms": ms},
        "h2d": {"bytes_per_step": bytes_in, "achieved_gbs": h2d_gbs, "peak_gbs_measured": h2d_peak,
                "frac": h2d_gbs / h2d_peak if h2d_peak else None, "store_hit_rate": hit_rate,
                "prefetched_per_step": (st1["prefetched"] - st0["prefetched"]) / K,
                "prefetch_used_per_step": (st1["prefetch_used"] - st0["prefetch_used"]) / K,
                "note": "rank 0; expert blobs copied from pinned host memory per step (misses and prefetches)"},
        "e2e": {"value": PF32_T * 1e3 / e2e_ms, "unit": "tokens/s", "h2d_bytes_per_step": T * HIDDEN * 4,
                "d2h_bytes_per_step": T * HIDDEN * 4},
        "gpu_launches": int(gpu_launches),
        "clocks": clocks.summary(),
    }
    return result, (ctx, store, lws)


def cpu_baseline_prefill32k():
    """The oracle port timed as for configs[3] (router + dequantised expert FFNs, 9 experts a token): per-token work
    does not depend on the routing skew, so the 40-layer rate is the one-layer rate / 40."""
    base = cpu_baseline_prefill()
    return {"value": base["value"] / LAYERS, "unit": "tokens/s", "cores": base["cores"], "kind": "port",
            "sample": base["sample"] + "; divided by 40 layers"}


def run_prefill4096(args, rank: int, world: int, dist):
    import torch
    from willow_v2_b200 import lib as L
    from willow_v2_b200 import moe, synth
    if world > 1:
        return run_prefill4096_ep(args, rank, world, dist)
    device = torch.cuda.current_device()
    ctx, store, layers = setup_model(device, 1)
    lw = layers[0].prepare(ctx, decode=False)
    K, W = args.steps, args.warmup
    T = PREFILL_T
    # 4 different batches of 4096 tokens cycled (each step re-routes); inputs resident before the timed region
    xs = [torch.from_numpy(synth.hidden(SEED + 1000 * rank, T, step=b)).to(torch.bfloat16).cuda() for b in range(4)]
    out = torch.empty(T, HIDDEN, dtype=torch.bfloat16, device="cuda")
    stream = torch.cuda.current_stream()

    def step(x, o):
        weights = lw.as_struct()
        L.check(ctx.handle, L.lib.wmoe_moe_forward_layer(ctx.handle, store.handle, 0, x.data_ptr(), L.BF16, T, TOP_K,
                                                         L.ctypes.byref(weights), o.data_ptr(), L.BF16, None, None,
                                                         stream.cuda_stream))

    for s in range(W):
        step(xs[s % 4], out)
    torch.cuda.synchronize()
    ctx.check_device()
    L.check(ctx.handle, L.lib.wmoe_set_profiling(ctx.handle, K))
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    launches0 = ctx.launches
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(device) as clocks:
        ev0.record(stream)
        for s in range(K):
            step(xs[s % 4], out)
        ev1.record(stream)
        torch.cuda.synchronize()
    gpu_launches = ctx.launches - launches0
    ms = ev0.elapsed_time(ev1) / K
    phase = {name: [] for name in L.PHASES}
    for ago in range(K):
        for p, name in enumerate(L.PHASES):
            v = L.ctypes.c_float()
            L.check(ctx.handle, L.lib.wmoe_phase_ms(ctx.handle, ago, p, L.ctypes.byref(v)))
            phase[name].append(v.value)
    L.check(ctx.handle, L.lib.wmoe_set_profiling(ctx.handle, 0))
    phase_ms = {name: statistics.mean(v) for name, v in phase.items()}
    ctx.check_device()

    # end to end through the public API: pinned bf16 host batch -> device, layer, result -> pinned host, every step,
    # the copies of neighbouring steps overlapping the layer (pipelined_e2e)
    x_host = [x.cpu().pin_memory() for x in xs]
    outs = [out, torch.empty_like(out)]

    def run(x_dev, b):
        step(x_dev, outs[b])
        return outs[b]

    e2e_ms = pipelined_e2e(torch, run, x_host, K, dist)
    if dist:
        dist.barrier()

    times = torch.tensor([ms, e2e_ms, phase_ms["gate_up"], phase_ms["down"]], dtype=torch.float64, device="cuda")
    if dist:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    ms, e2e_ms, gu_ms, dn_ms = times.tolist()
    _, bf16, peak_kind = peaks()
    gu_tflops = GATE_UP_FLOPS / (gu_ms * 1e-3) / 1e12
    dn_tflops = DOWN_FLOPS / (dn_ms * 1e-3) / 1e12
    layer_tflops = (GATE_UP_FLOPS + DOWN_FLOPS) / (ms * 1e-3) / 1e12
    result = {
        "metric": METRIC_PREFILL, "value": world * T * 1e3 / ms, "unit": "tokens/s", "n_gpus": world, "steps": K,
        "warmup": W, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16 in/out, fp16 tensor-core operands, fp32 accumulation",
        "data": "synthetic (seeded GGUF Q4_K/Q6_K blocks with the config-0 distributions; bf16 N(0,1) tokens)",
        "config": workload_config("prefill4096", world),
        "roofline": {"bound": "tensor", "kernel": "grouped_gemm_kernel<0> (gate_up + SwiGLU)",
                     "achieved": gu_tflops, "peak": bf16, "unit": "TFLOP/s", "frac": gu_tflops / bf16,
                     "traffic": PREFILL_GATE_UP_TRAFFIC, "peak_kind": peak_kind,
                     "algorithmic_flops_per_launch": GATE_UP_FLOPS, "launch_ms": gu_ms},
        "roofline_down": {"kernel": "grouped_gemm_kernel<1> (down)", "achieved": dn_tflops, "frac": dn_tflops / bf16,
                          "algorithmic_flops_per_launch": DOWN_FLOPS, "launch_ms": dn_ms},
        "layer_tensor_frac": layer_tflops / bf16,
        "phase_ms": phase_ms,
        "e2e": {"value": world * T * 1e3 / e2e_ms, "unit": "tokens/s", "h2d_bytes_per_step": T * HIDDEN * 2,
                "d2h_bytes_per_step": T * HIDDEN * 2,
                "copies": "every step's input in and result out inside the timed region, on two copy streams "
                          "overlapping the neighbouring steps' compute (double buffers ordered by events)"},
        "gpu_launches": int(gpu_launches),
        "clocks": clocks.summary(),
    }
    return result, (ctx, store, layers)


def cpu_baseline_prefill(sample_experts: int = 0, tokens_per_expert: int = 144):
    """willow's CPU path restated (the oracle port) for the prefill layer on every host core: the router on all 4096
    tokens, then a sample of experts (default 4 per worker) dequantised with their FFN on 144 tokens each, in
    parallel on the pool, scaled to the 257 experts (256 routed + shared) of the layer (36,864 token-expert rows)."""
    import oracle.moe_oracle as ora
    from willow_v2_b200 import synth
    _, workers = cpu_baseline_pool()
    n = sample_experts or 4 * workers
    x = synth.hidden(SEED, PREFILL_T, step=321)
    router = synth.router_weight(SEED, 0)
    t0 = time.perf_counter()
    ora.route(x @ router.T)
    t_route = time.perf_counter() - t0
    tasks = [("Q4_K/Q6_K", e % N_BLOBS, x[(e % 28) * tokens_per_expert:(e % 28 + 1) * tokens_per_expert], False)
             for e in range(n)]
    t_pool, _ = cpu_baseline_wall(tasks)
    rows = PREFILL_T * (TOP_K + 1)
    sec = t_route + t_pool / (n * tokens_per_expert) * rows
    return {"value": PREFILL_T / sec, "unit": "tokens/s", "cores": workers, "kind": "port",
            "sample": f"router on all {PREFILL_T} tokens; {n} experts dequantised from GGUF bytes with their FFN on "
                      f"{tokens_per_expert} tokens each, in parallel on {workers} worker processes (numpy float32); "
                      f"scaled to {rows} token-expert rows"}


def cpu_decode_token(h, routers, step: int) -> float:
    """One whole decode token of the oracle port: 40 layers of rms_norm, router + top-8, the 9 experts in parallel on
    the pool, combine and residual, each layer fed by the last. Returns the seconds it took."""
    import oracle.moe_oracle as ora
    t = 0.0
    for l, router in enumerate(routers):
        t0 = time.perf_counter()
        xn = ora.rms_norm(h)
        t += time.perf_counter() - t0
        dt, out = cpu_baseline_decode_layer(xn, router, step * LAYERS + l)
        t0 = time.perf_counter()
        h = h + out
        t += dt + time.perf_counter() - t0
    return t


_PF_SHM = []


def cpu_prefill_layer(x, router) -> float:
    """One whole prefill layer of the oracle port on the pool (4096 tokens): the router and top-8 on every token, each
    of the 256 routed experts on its tokens and the shared expert on all of them (split over the workers), every
    expert dequantised from GGUF bytes (stand-in blobs of the same sizes), outputs in shared memory, then the
    combine in ascending expert id plus the gated shared expert. Returns the seconds it took."""
    import oracle.moe_oracle as ora
    from multiprocessing import shared_memory
    pool, workers = cpu_baseline_pool()
    T = x.shape[0]
    P = T * (TOP_K + 1)
    if not _PF_SHM:
        import atexit
        for nbytes in (T * HIDDEN * 4, P * HIDDEN * 4):
            _PF_SHM.append(shared_memory.SharedMemory(create=True, size=nbytes))
        atexit.register(lambda: [(m.close(), m.unlink()) for m in _PF_SHM])
    xs, ys = _PF_SHM
    np.ndarray((T, HIDDEN), np.float32, buffer=xs.buf)[:] = x
    y = np.ndarray((P, HIDDEN), np.float32, buffer=ys.buf)
    t0 = time.perf_counter()
    logits = x @ router.T
    w, sel = ora.route(logits[:, :EXPERTS])
    flat = sel.reshape(-1)
    order = np.argsort(flat, kind="stable")  # pairs grouped by expert, tokens ascending within an expert
    counts = np.bincount(flat, minlength=EXPERTS)
    starts = np.concatenate([[0], np.cumsum(counts)])
    tasks = [(e % N_BLOBS, xs.name, T, (order[starts[e]:starts[e + 1]] // TOP_K).astype(np.int32), ys.name, P,
              int(starts[e])) for e in range(EXPERTS) if counts[e]]
    chunk = -(-T // workers)
    tasks += [(0, xs.name, T, np.arange(c, min(T, c + chunk), dtype=np.int32), ys.name, P, T * TOP_K + c)
              for c in range(0, T, chunk)]
    list(pool.map(_prefill_task, tasks))
    pos = np.empty(T * TOP_K, np.int64)
    pos[order] = np.arange(T * TOP_K)
    pos = pos.reshape(T, TOP_K)
    asc = np.argsort(sel, axis=1, kind="stable")
    out = np.zeros((T, HIDDEN), np.float32)
    rows = np.arange(T)
    for j in range(TOP_K):
        k = asc[:, j]
        out += w[rows, k, None] * y[pos[rows, k]]
    out += ora.sigmoid(logits[:, EXPERTS:EXPERTS + 1]) * y[T * TOP_K:]
    return time.perf_counter() - t0


def cpu_baseline(sample_layers: int = 4):
    """willow's CPU path restated (the oracle port) on every host core: per layer the router + top-8, the 9 experts'
    dequantisation from GGUF bytes and FFN in parallel on the pool, the combine; tokens/s scaled to the 40-layer
    token from the sampled layers."""
    import oracle.moe_oracle as ora
    from willow_v2_b200 import synth
    _, workers = cpu_baseline_pool()
    h = synth.hidden(SEED, 1, step=123)
    total = 0.0
    for l in range(sample_layers):
        total += cpu_baseline_decode_layer(ora.rms_norm(h), synth.router_weight(SEED, l), l)[0]
    per_layer = total / sample_layers
    return {"value": 1.0 / (per_layer * LAYERS), "unit": "tokens/s", "cores": workers, "kind": "port",
            "sample": f"{sample_layers} of the 40 layers of one decode token (router + top-8; 9 experts dequantised "
                      f"and run in parallel on {workers} worker processes; combine; float32 numpy), scaled to 40 "
                      f"layers"}


def run_reference(args, rank, world):
    """The reference arm: the CPU restatement of willow's CPU path on the host cores, rank 0 only."""
    if rank != 0:
        return None
    if args.workload == "prefill32k":
        K, W = args.steps, args.warmup
        n = cpu_baseline_pool()[1]  # one expert per worker each step
        vals = [cpu_baseline_prefill(sample_experts=n)["value"] / LAYERS for _ in range(W + K)][W:]
        value = statistics.mean(vals)
        base = cpu_baseline_prefill(sample_experts=n)
        return {"metric": METRIC_PF32, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": K,
                "warmup": W, "ms_per_step": PF32_T / value * 1e3, "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
                "config": workload_config("prefill32k", world),
                "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": base["cores"], "kind": "port",
                                 "sample": "each step: " + base["sample"] + "; divided by 40 layers"},
                "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    if args.workload == "batch64":
        K, W = args.steps, args.warmup
        vals = [cpu_baseline_batch()["value"] for _ in range(W + K)][W:]
        value = statistics.mean(vals)
        base = cpu_baseline_batch()
        return {"metric": METRIC_BATCH, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": K,
                "warmup": W, "ms_per_step": BATCH_T / value * 1e3, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
                "config": workload_config("batch64", world),
                "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": base["cores"], "kind": "port",
                                 "sample": "each step: " + base["sample"]},
                "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    if args.workload == "prefill4096":
        res = reference_prefill4096(args.steps, args.warmup, world)
        if world == 1 and not args.no_decode40:
            res["decode40"] = reference_decode40(min(args.steps, 8), 1, world)
        return res
    return reference_decode40(args.steps, args.warmup, world)


def reference_decode40(K: int, W: int, world: int) -> dict:
    """The reference arm for configs[1]: every step is one whole 40-layer token of the oracle port (cpu_decode_token),
    so ms_per_step x steps is the time measured."""
    from willow_v2_b200 import synth
    _, workers = cpu_baseline_pool()
    routers = [synth.router_weight(SEED, l) for l in range(LAYERS)]
    times = [cpu_decode_token(synth.hidden(SEED, 1, step=10_000 + s), routers, s) for s in range(W + K)][W:]
    sec = statistics.mean(times)
    value = 1.0 / sec
    return {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": sec * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic", "impl": "reference", "config": workload_config("decode40", world),
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": workers, "kind": "port",
                             "sample": f"each step one whole token: 40 layers of rms_norm, router + top-8, the 9 "
                                       f"experts dequantised from GGUF bytes (stand-in blobs of the same sizes) and "
                                       f"run in parallel on {workers} worker processes, combine, residual (numpy "
                                       f"float32)"},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def reference_prefill4096(K: int, W: int, world: int) -> dict:
    """The reference arm for configs[3]: every step is one whole 4096-token layer of the oracle port
    (cpu_prefill_layer); 4 batches cycled like the GPU arm."""
    from willow_v2_b200 import synth
    _, workers = cpu_baseline_pool()
    router = np.vstack([synth.router_weight(SEED, 0), synth.shared_gate_weight(SEED, 0).reshape(1, -1)])
    xs = [synth.hidden(SEED, PREFILL_T, step=b) for b in range(4)]
    times = [cpu_prefill_layer(xs[s % 4], router) for s in range(W + K)][W:]
    sec = statistics.mean(times)
    value = PREFILL_T / sec
    return {"metric": METRIC_PREFILL, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": sec * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic", "impl": "reference", "config": workload_config("prefill4096", world),
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": workers, "kind": "port",
                             "sample": f"each step one whole layer of {PREFILL_T} tokens: router + top-8 on every "
                                       f"token, the 256 routed experts on their tokens and the shared expert on all, "
                                       f"each dequantised from GGUF bytes (stand-in blobs of the same sizes), in "
                                       f"parallel on {workers} worker processes (numpy float32), combine"},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


TYPED_D_AT = {"Q6_K": 208}  # byte offset of the fp16 scale in a block (0 for the other types)
# DRAM bytes (read + write) of one gemv_batch launch over 8 Q8_0 gate_up matrices, measured by ncu
# (dram__bytes_read.sum + dram__bytes_write.sum = 17,845,760 + 0): the algorithmic 17,825,792 plus the activations
# and addresses. The other types were not captured.
TYPED_TRAFFIC = {"Q8_0": 17_845_760}


def run_typed_decode(args, type_name: str):
    """willow's batched decode of one token's routed experts in another ggml type (engines/base.py:492-532 with
    gguf/metal.py's kernels): gemv_batch over 8 experts' gate_up [1024, 2048], SwiGLU, gemv_combine over their down
    [2048, 512] with bf16 routing weights. Each step's 8 experts are drawn from a pool of at least 2 GB of experts
    (L2 holds under 7% of it). Steps are captured in CUDA graphs of G steps (each on other experts) and replayed,
    so the device time is not the host's launch rate; two more graphs hold only the gemv_batch or only the combine
    launches, for their per-launch times."""
    import torch
    from willow_v2_b200 import ggml, moe
    from willow_v2_b200 import lib as L
    ctx = moe.default_context()
    K, W = args.steps, args.warmup
    elements, size = ggml.BLOCKS[type_name]
    gu_b = 2 * FFN * ggml.row_bytes(type_name, HIDDEN)
    dn_b = HIDDEN * ggml.row_bytes(type_name, FFN)
    eb = gu_b + dn_b
    pool = max(EXPERTS, -(-(2 << 30) // eb))
    g = torch.Generator(device="cuda").manual_seed(SEED)
    slab = torch.randint(0, 256, (pool * eb,), dtype=torch.uint8, device="cuda", generator=g)
    blocks = slab.view(-1, size)
    d_at = TYPED_D_AT.get(type_name, 0)
    nb = blocks.shape[0]
    for off in ((d_at, 2) if type_name == "Q4_K" else (d_at,)):
        d = torch.empty(nb, dtype=torch.float16, device="cuda").uniform_(1e-3, 4e-3, generator=g)
        blocks[:, off:off + 2] = d.view(torch.uint8).view(nb, 2)
    del d
    G = 50  # steps per graph
    rng = np.random.default_rng(SEED)
    sels = [rng.choice(pool, TOP_K, replace=False) for _ in range(G)]
    base = slab.data_ptr()
    gu_ptrs = [torch.tensor([base + int(e) * eb for e in s], dtype=torch.int64, device="cuda") for s in sels]
    dn_ptrs = [torch.tensor([base + int(e) * eb + gu_b for e in s], dtype=torch.int64, device="cuda") for s in sels]
    pos = torch.arange(TOP_K, dtype=torch.int64, device="cuda")
    x = torch.randn(HIDDEN, generator=g, device="cuda").to(torch.bfloat16)
    route = torch.rand(TOP_K, generator=g, device="cuda")
    route = (route / route.sum()).to(torch.bfloat16)
    gate_up = torch.empty(TOP_K, 2 * FFN, dtype=torch.bfloat16, device="cuda")
    h = torch.empty(TOP_K, FFN, dtype=torch.bfloat16, device="cuda")
    y = torch.empty(HIDDEN, dtype=torch.bfloat16, device="cuda")
    tid = L.GGML_TYPES[type_name]

    def up(i):
        st = torch.cuda.current_stream().cuda_stream
        L.check(ctx.handle, L.lib.wmoe_gemv_batch(ctx.handle, tid, gu_ptrs[i].data_ptr(), pos.data_ptr(), TOP_K, TOP_K,
                                                  2 * FFN, HIDDEN, x.data_ptr(), L.BF16, gate_up.data_ptr(), L.BF16,
                                                  st))

    def act():  # willow's expert_gate (engines/base.py:99-102) on the library's kernel
        L.check(ctx.handle, L.lib.wmoe_expert_gate(ctx.handle, gate_up.data_ptr(), TOP_K, FFN, h.data_ptr(),
                                                   torch.cuda.current_stream().cuda_stream))

    def down(i):
        st = torch.cuda.current_stream().cuda_stream
        L.check(ctx.handle, L.lib.wmoe_gemv_combine(ctx.handle, tid, dn_ptrs[i].data_ptr(), pos.data_ptr(), TOP_K,
                                                    TOP_K, HIDDEN, FFN, h.data_ptr(), route.data_ptr(), L.BF16,
                                                    y.data_ptr(), st))

    for s in range(W):
        up(s % G), act(), down(s % G)
    torch.cuda.synchronize()
    ctx.check_device()
    graphs = {}
    for name, body in (("step", lambda i: (up(i), act(), down(i))), ("up", up), ("down", down)):
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in range(G):
                body(i)
        graphs[name] = graph
    reps = max(-(-K // G), 400)  # at least 20,000 steps (~0.7 s): the clock sampler sees the timed region
    stream = torch.cuda.current_stream()

    def timed(name):
        graphs[name].replay()  # untimed replay: warm instruction caches and the graph itself
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            graphs[name].replay()
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / (reps * G)

    launches0 = ctx.launches
    with ClockSampler(torch.cuda.current_device()) as clocks:
        step_ms = timed("step")
    gpu_launches = 3 * reps * G  # the graph's replays launch the captured kernels; ctx counts captures, not replays
    gu_ms, dn_ms = timed("up"), timed("down")
    ctx.check_device()
    del launches0
    # e2e through the public Python API, no graph: x from pinned host memory in, the token's experts in one
    # ggml.batched_decode_experts call (engines/base.py:492-532), y back out
    x_host = x.cpu().pin_memory()
    y_host = torch.empty(HIDDEN, dtype=torch.bfloat16).pin_memory()
    x_dev = torch.empty_like(x)
    offs = [[int(e) * eb for e in s] for s in sels]
    dn_offs = [[o + gu_b for o in s] for s in offs]
    slots = list(range(TOP_K))
    for s in range(W):
        ggml.batched_decode_experts(slab, type_name, type_name, FFN, x_dev, offs[s % G], dn_offs[s % G], route,
                                    slots, ctx=ctx)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(stream)
    y_dev = torch.empty(1, HIDDEN, dtype=torch.bfloat16, device="cuda")
    for s in range(K):
        x_dev.copy_(x_host, non_blocking=True)
        ggml.batched_decode_experts(slab, type_name, type_name, FFN, x_dev, offs[s % G], dn_offs[s % G], route,
                                    slots, ctx=ctx, out=y_dev)
        y_host.copy_(y_dev.reshape(-1), non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / K
    hbm, _, peak_kind = peaks()
    gu_gbs = TOP_K * gu_b / (gu_ms * 1e-3) / 1e9
    dn_gbs = TOP_K * dn_b / (dn_ms * 1e-3) / 1e9
    step_gbs = TOP_K * eb / (step_ms * 1e-3) / 1e9
    return {
        "metric": f"typed batched-decode tokens/s (8 routed experts of one MoE layer, {type_name} weights)",
        "value": 1e3 / step_ms, "unit": "tokens/s", "n_gpus": 1, "steps": reps * G, "warmup": W,
        "ms_per_step": step_ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16 (f32 sums)",
        "data": f"synthetic: random {type_name} blocks with fp16 scales U[1e-3, 4e-3]; bf16 N(0,1) token",
        "config": workload_config("typed-decode", 1, type_name=type_name),
        "pool": {"expert_bytes": eb, "pool_experts": pool, "pool_bytes": pool * eb,
                 "timing": f"CUDA graphs of {G} steps replayed {reps} times; events around the replays"},
        "roofline": {"bound": "hbm", "kernel": "ggml_gemv_kernel (gemv_batch of the 8 gate_up matrices)",
                     "achieved": gu_gbs, "peak": hbm, "unit": "GB/s", "frac": gu_gbs / hbm,
                     "traffic": TYPED_TRAFFIC.get(type_name), "peak_kind": peak_kind,
                     "algorithmic_bytes_per_launch": TOP_K * gu_b, "launch_ms": gu_ms},
        "combine": {"kernel": "ggml_combine_kernel (8 down matrices + bf16 weighted sum)", "launch_ms": dn_ms,
                    "achieved_gbs": dn_gbs, "frac": dn_gbs / hbm},
        "roofline_step": {"achieved": step_gbs, "frac": step_gbs / hbm, "algorithmic_bytes": TOP_K * eb},
        "e2e": {"value": 1e3 / e2e_ms, "unit": "tokens/s", "h2d_bytes_per_step": HIDDEN * 2,
                "d2h_bytes_per_step": HIDDEN * 2, "path": "willow_v2_b200.ggml.batched_decode_experts (one library call)"},
        "gpu_launches": int(gpu_launches),
        "clocks": clocks.summary(),
    }


def cpu_baseline_typed(type_name: str):
    """The oracle port of the same step on every host core: one token's 8 experts (dequantise gate_up and down,
    SwiGLU, down product) in parallel on the pool, for about 2 s of tokens."""
    _, workers = cpu_baseline_pool()
    x = np.random.default_rng(SEED).standard_normal((1, HIDDEN)).astype(np.float32)
    tasks = [(type_name, 0, x, False) for _ in range(TOP_K)]
    times = []
    while not times or sum(times) < 2.0:
        times.append(cpu_baseline_wall(tasks)[0])
    dt = statistics.mean(times)
    return {"value": 1.0 / dt, "unit": "tokens/s", "cores": workers, "kind": "port",
            "sample": f"{len(times)} tokens x 8 experts ({type_name}) in parallel on {workers} worker processes, same "
                      f"shapes, ~2 s"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None, help="default 2000 (reference arm: 20)")
    ap.add_argument("--warmup", type=int, default=None, help="default 50 (reference arm: 5)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="prefill4096",
                    choices=["decode40", "batch64", "prefill4096", "prefill32k", "typed-decode"])
    ap.add_argument("--ggml-type", default="all", help="typed-decode: one ggml type, or all (one JSON line each)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--layers", type=int, default=LAYERS, help="stack depth (40 = the benchmark; fewer = profiling)")
    ap.add_argument("--no-decode40", action="store_true",
                    help="prefill4096 at N=1: skip the decode40 measurement attached to the line")
    ap.add_argument("--ep-chunks", type=int, default=None,
                    help="prefill4096 at N>1: token chunks per rank (default: the library's choice for N)")
    ap.add_argument("--ep-exchange", choices=["auto", "copy", "nccl"], default="auto",
                    help="prefill4096 at N>1: the rows' exchange (default: the library's choice for N)")
    args = ap.parse_args()
    if args.steps is None:
        args.steps = 20 if args.impl == "reference" else 2000
    if args.warmup is None:
        args.warmup = 5 if args.impl == "reference" else 50
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference" and args.workload == "typed-decode":
        if rank == 0:
            from willow_v2_b200.ggml import TYPES
            for t in (TYPES if args.ggml_type == "all" else [args.ggml_type]):
                base = cpu_baseline_typed(t)
                v = base["value"]
                print(json.dumps({
                    "metric": f"typed batched-decode tokens/s (8 routed experts of one MoE layer, {t} weights)",
                    "value": v, "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                    "ms_per_step": 1e3 / v, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                    "dtype": "f32", "data": "synthetic", "impl": "reference",
                    "config": workload_config("typed-decode", 1, type_name=t),
                    "cpu_baseline": base,
                    "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
                    flush=True)
        shutdown_cpu_pool()
        return
    if args.impl == "reference":
        res = run_reference(args, rank, world)
        if res is not None:
            print(json.dumps(res), flush=True)
        shutdown_cpu_pool()
        return
    import torch
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as d
        d.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                             device_id=torch.device("cuda", local))
        dist = d
    if args.workload == "typed-decode":
        from willow_v2_b200 import ggml
        for t in (ggml.TYPES if args.ggml_type == "all" else [args.ggml_type]):
            result = run_typed_decode(args, t)
            if not args.no_cpu_baseline:
                result["cpu_baseline"] = cpu_baseline_typed(t)
            print(json.dumps(result), flush=True)
        shutdown_cpu_pool()
        return
    if args.workload == "prefill4096":
        result, _keep = run_prefill4096(args, rank, world, dist)
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            result["cpu_baseline"] = cpu_baseline_prefill()
        if world == 1 and not args.no_decode40:
            # configs[1] on the same GPU, its own line attached: the 40-layer single-token decode (HBM roofline)
            del _keep
            torch.cuda.empty_cache()
            d40, _keep = run_decode40(args, rank, world, dist)
            result["decode40"] = {k: d40[k] for k in ("metric", "value", "unit", "ms_per_step", "steps", "warmup",
                                                     "config", "roofline", "e2e", "gpu_launches", "clocks")}
    elif args.workload == "prefill32k":
        result, _keep = run_prefill32k(args, rank, world, dist)
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            result["cpu_baseline"] = cpu_baseline_prefill32k()
    elif args.workload == "batch64":
        result, _keep = run_batch64(args, rank, world, dist)
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            result["cpu_baseline"] = cpu_baseline_batch()
    else:
        result, _keep = run_decode40(args, rank, world, dist)
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            result["cpu_baseline"] = cpu_baseline()
    if rank == 0:
        print(json.dumps(result), flush=True)
    shutdown_cpu_pool()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
