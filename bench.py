"""MoE-layer throughput benchmark (tokens/s) of the B200 framework, or of the reference's
CPU path with ``--impl reference``.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 ... bench.py --gpus N

Workload (one step): one forward of a Mixtral-8x7B-shape MoE layer, T=4096 tokens, d=4096,
E=8 experts, top-2 softmax routing renormalised over fp32 router logits, SwiGLU experts with
inner dim 14336, bf16, seeded synthetic N(0,1) activations and N(0,0.02) weights.  The
layer runs through the drop-in API: ``DistMoEBlock.forward`` with one ``DistExpertsBlock``
holding the 8 experts on the same GPU, connected through the NVLink/CUDA-IPC transfer engine.

* ``value``: tokens/s of forwards whose input is already in HBM (device-timed with CUDA
  events, barrier + synchronize on both sides; max over ranks).
* ``e2e``: the same API with the input in pinned host memory: the H2D copy of the tokens and
  the D2H read of the layer output are inside the timed region.
* ``roofline``: the grouped expert MLP (the tcgen05 GEMM pair) timed with CUDA events on its
  own stream during the timed steps, against the measured bf16 peak.
* ``cpu_baseline``: the oracle port of the reference's torch path (routing +
  ``local_experts``), timed on this host's cores on a bounded token sample.

With N GPUs (``--parallel experts``, the default for N > 1) the experts are sharded: GPU g
holds experts [g*8/N, (g+1)*8/N), every rank hosts its own 4096 tokens, and every host
sends each token to the GPUs of its two experts and combines the results (one
``DistMoEBlock`` per rank whose expert blocks span all N GPUs; activations cross NVLink
through the CUDA-IPC transfer engine).  Per-GPU work stays fixed as N grows (weak scaling).
``--parallel replicas`` runs an independent single-GPU layer per rank instead.  The expert
weights (2.8 GB in all) exceed L2, so every step streams them from HBM.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

# Up to 32 hardware work queues per GPU (CUDA's default is 8): an expert-parallel process
# drives a few tens of streams (buffer pools, helper streams), and streams that share a queue
# serialise.  Must be set before CUDA starts.
os.environ.setdefault("CUDA_DEVICE_MAX_CONNECTIONS", "32")

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import torch  # noqa: E402

METRIC = "moe_layer_tokens_per_s"
# Layer traffic of the grouped MLP (both GEMMs of one launch) for the Mixtral workload, from
# `ncu --metrics dram__bytes_read.sum,dram__bytes_write.sum` on the layer (one pass; see
# profiles/launches_mixtral_moe_layer.md).  None for workloads without a capture.
MIXTRAL_MLP_TRAFFIC_BYTES = (1971 + 228 + 1409 + 58) * 10**6  # GEMM1 read+write, GEMM2 read+write


class Workload:
    """One benchmark configuration: layer shape, routing, initialisation and how tokens and
    experts spread over the GPUs."""

    def __init__(self, name, *, tokens, d, E, k, I, seed, w_std, router_mode="softmax", n_group=1,
                 topk_group=1, scale=1.0, score_bias_std=0.0, shared_inner=0, strong=False, io_max=8192,
                 traffic=None):
        self.name, self.tokens, self.d, self.E, self.k, self.I = name, tokens, d, E, k, I
        self.seed, self.w_std, self.router_mode = seed, w_std, router_mode
        self.n_group, self.topk_group, self.scale = n_group, topk_group, scale
        self.score_bias_std, self.shared_inner, self.strong = score_bias_std, shared_inner, strong
        self.io_max, self.traffic = io_max, traffic

    def tokens_per_rank(self, world: int) -> int:
        return self.tokens // world if self.strong else self.tokens

    def io(self, world: int, parallel: str) -> tuple:
        """(io_buffer_size, number_of_io_buffers) for one host of `world` ranks."""
        if parallel != "experts":
            return self.io_max, max(2, -(-self.tokens * self.k // self.io_max))
        per_block = self.tokens_per_rank(world) * self.k // world
        size = min(self.io_max, max(256, -(-(per_block * 3 // 2) // 256) * 256))
        return size, 2 * world

    def mlp_flops(self, T: int) -> float:
        return 6.0 * T * self.k * self.d * self.I + 6.0 * T * self.d * self.shared_inner

    def config(self, world: int, parallel: str) -> dict:
        io_size, io_buffers = self.io(world, parallel)
        T = self.tokens_per_rank(world)
        if parallel == "experts":
            par = f"ep{world}: {self.E // world} experts per GPU, one host per GPU with {T} tokens"
        elif parallel == "replicas":
            par = f"replicas x{world}"
        else:
            par = "single gpu"
        router = (f"sigmoid + selection bias N(0,{self.score_bias_std}), {self.n_group} groups / top-{self.topk_group}, "
                  f"top-{self.k} renormalised x{self.scale}, fp32 logits" if self.router_mode == "sigmoid_group"
                  else f"softmax top-{self.k} renormalised, fp32 logits")
        c = {"workload": self.name, "tokens_per_gpu": T, "tokens_per_step": T * world, "hidden": self.d,
             "experts": self.E, "top_k": self.k, "inner": self.I, "router": router, "activation": "silu (SwiGLU)",
             "expert_blocks": world if parallel == "experts" else 1, "io_buffer_size": io_size,
             "io_buffers": io_buffers, "transfer_engine": "NVLinkIPC",
             "l2": "no flush: the expert weights exceed the 126 MB L2 every step",
             "parallelism": par, "seed": self.seed}
        if self.shared_inner:
            c["shared_expert_inner"] = self.shared_inner
        return c


WORKLOADS = {
    # Mixtral-8x7B-shape layer on each GPU (weak scaling over GPUs).
    "mixtral": Workload("mixtral-8x7b-moe-layer", tokens=4096, d=4096, E=8, k=2, I=14336, seed=1, w_std=0.02,
                        io_max=8192, traffic=MIXTRAL_MLP_TRAFFIC_BYTES),
    # Qwen3-30B-A3B-shape decode step: few tokens (--tokens 16, 64 or 256) in all, 128 experts
    # (16 per GPU over 8 GPUs); time per step is the figure of merit.
    "qwen3-decode": Workload("qwen3-30b-a3b-decode-moe-layer", tokens=64, d=2048, E=128, k=8, I=768, seed=3,
                             w_std=0.02, strong=True, io_max=2048),
    # DeepSeek-V3-shape layer, 8192 tokens per step in all (strong scaling: T/N per GPU).
    "deepseek": Workload("deepseek-v3-moe-layer", tokens=8192, d=7168, E=256, k=8, I=2048, seed=2, w_std=0.006,
                         router_mode="sigmoid_group", n_group=8, topk_group=4, scale=2.5, score_bias_std=0.01,
                         shared_inner=2048, strong=True, io_max=65535),
}


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["bf16_tflops"]), float(p["bf16_tflops_sustained"]), float(p["hbm_gbs"]), "measured"
    except Exception:
        return 1590.0, 1400.0, 6650.0, "fallback"


class ClockSampler:
    """SM clock, power and throttle reasons of one GPU, sampled every 20 ms during the timed
    region (NVML; nvidia-smi as a fallback)."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20, "sw_power_cap": 0x4}

    def __init__(self, gpu_index: int, period_s: float = 0.02):
        self.gpu = gpu_index
        self.period = period_s
        self.samples = []
        self.max_mhz = None
        self._stop = None
        self._thread = None

    def __enter__(self):
        import threading
        try:
            import pynvml
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.gpu)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
        except Exception:
            return self
        self._stop = threading.Event()

        def run():
            while not self._stop.is_set():
                try:
                    self.samples.append((pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM),
                                         pynvml.nvmlDeviceGetPowerUsage(h) / 1000.0,
                                         pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)))
                except Exception:
                    pass
                self._stop.wait(self.period)

        self._thread = threading.Thread(target=run, daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *a):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=2)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["no samples"]}
        sm = sorted(x[0] for x in self.samples)
        reasons = sorted({name for _, _, r in self.samples for name, bit in self.REASONS.items() if r & bit})
        return {"sm_mhz": sm[len(sm) // 2], "sm_min_mhz": sm[0], "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(self.samples), "power_w_max": max(x[1] for x in self.samples)}


def _dist():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    if ws > 1:
        import torch.distributed as dist
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300))
        return dist, dist.get_rank(), ws, int(os.environ.get("LOCAL_RANK", "0"))
    return None, 0, 1, 0


def _barrier(dist, dev):
    torch.cuda.synchronize(dev)
    if dist is not None:
        dist.barrier()
        torch.cuda.synchronize(dev)


def _max_over_ranks(dist, v: float, dev) -> float:
    if dist is None:
        return v
    t = torch.tensor([v], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ----------------------------------------------------------------------------- CPU (oracle port)
class _Cycled:
    """E experts' weights backed by fewer distinct copies (expert e -> copy e mod n)."""

    def __init__(self, stack: torch.Tensor, E: int):
        self.stack, self.shape = stack, (E,) + tuple(stack.shape[1:])

    def __getitem__(self, e):
        return self.stack[int(e) % self.stack.shape[0]]


class CpuReference:
    """The oracle port of the reference's torch path on this host's cores: fp32-logit routing
    (the workload's router), then ``local_experts`` (per hit expert: gather, gate/up/down in
    bf16, weighted index_add; plus the shared expert) on a token sample of the layer with
    full-size weights."""

    def __init__(self, w: Workload, step_budget_s: float = 1.5, max_tokens: int = 1024):
        from oracle import moe_oracle as O

        self.O, self.w = O, w
        self.threads = torch.get_num_threads()
        g = torch.Generator().manual_seed(w.seed)
        # One random matrix per projection, copied into separate memory for up to 32 experts
        # (expert e uses copy e mod 32): the timing depends on the shapes and on the weights
        # streaming from DRAM, not on their values.
        bf = torch.bfloat16
        base_g = (torch.randn(w.I, w.d, generator=g) * w.w_std).to(bf)
        base_u = (torch.randn(w.I, w.d, generator=g) * w.w_std).to(bf)
        base_d = (torch.randn(w.d, w.I, generator=g) * w.w_std).to(bf)
        copies = min(w.E, 32)
        self.wg = _Cycled(torch.stack([base_g] * copies), w.E)
        self.wu = _Cycled(torch.stack([base_u] * copies), w.E)
        self.wd = _Cycled(torch.stack([base_d] * copies), w.E)
        self.wr = (torch.randn(w.E, w.d, generator=g) * w.w_std).to(bf)
        self.bias = torch.randn(w.E, generator=g) * w.score_bias_std if w.score_bias_std else None
        self.shared = None
        if w.shared_inner:
            self.shared = tuple((torch.randn(*sh, generator=g) * w.w_std).to(bf)
                                for sh in ((w.shared_inner, w.d), (w.shared_inner, w.d), (w.d, w.shared_inner)))
        self.g = g
        n = 64
        dt = self.step(n)
        while dt < step_budget_s / 2 and n < max_tokens:
            n *= 2
            dt = self.step(n)
        self.n = n

    def step(self, n: int = 0) -> float:
        n = n or self.n
        O, w = self.O, self.w
        x = torch.randn(n, w.d, generator=self.g).to(torch.bfloat16)
        mode = O.ROUTER_SIGMOID_GROUP if w.router_mode == "sigmoid_group" else O.ROUTER_SOFTMAX
        t0 = time.perf_counter()
        logits = O.router_logits(x, self.wr, fp32_logits=True)
        O.local_experts(x, logits, self.wg, self.wu, self.wd, w.k, act=O.ACT_SILU, renormalize=True, mode=mode,
                        score_bias=self.bias, scale=w.scale, n_group=w.n_group, topk_group=w.topk_group,
                        shared=self.shared)
        return time.perf_counter() - t0

    def sample(self, reps: int) -> str:
        return f"{self.n} tokens of the {self.w.name} shape per step (full-size bf16 weights, torch CPU), {reps} steps"

    def tokens_per_s(self, reps: int = 3) -> float:
        return self.n / statistics.median(self.step() for _ in range(reps))


def run_reference(args, rank):
    """The oracle port of the reference's CPU torch path, on this host's cores (rank 0 only)."""
    if rank != 0:
        return
    w = WORKLOADS[args.workload]
    parallel = args.parallel if args.gpus > 1 else "single"
    ref = CpuReference(w)
    for _ in range(args.warmup):
        ref.step()
    times = [ref.step() for _ in range(args.steps)]
    tok_s = ref.n * len(times) / sum(times)
    line = {"metric": METRIC, "value": tok_s, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": w.tokens_per_rank(args.gpus) * args.gpus / tok_s * 1e3,
            "higher_is_better": True, "scaling": "strong" if w.strong else "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": w.config(args.gpus, parallel),
            "impl": "reference",
            "cpu_baseline": {"value": tok_s, "unit": "tokens/s", "cores": ref.threads, "kind": "port",
                             "sample": ref.sample(args.steps)},
            "e2e": {"value": tok_s, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- GPU (ours)
def _randn_bf16(shape, std, gen, dev, chunk_elems=1 << 28):
    """Seeded N(0, std) bf16 tensor made on the GPU a slice at a time (no fp32 copy of the
    whole stack)."""
    out = torch.empty(shape, dtype=torch.bfloat16, device=dev)
    row = 1
    for n in shape[1:]:
        row *= n
    chunk_rows = max(1, chunk_elems // row)
    for i in range(0, shape[0], chunk_rows):
        j = min(shape[0], i + chunk_rows)
        out[i:j] = (torch.randn((j - i,) + tuple(shape[1:]), generator=gen, device=dev) * std).to(torch.bfloat16)
    return out


def run_ours(args, dist, rank, world, local_rank):
    from distributedmoe_b200 import _native as N
    from distributedmoe_b200.MoE.local_cluster import LocalCluster
    from distributedmoe_b200.MoE.sharded_cluster import ShardedCluster

    w = WORKLOADS[args.workload]
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    parallel = args.parallel if world > 1 else "single"
    if parallel == "experts" and w.E % world:
        raise SystemExit(f"--parallel experts needs a GPU count that divides {w.E}")
    E_here = w.E // world if parallel == "experts" else w.E
    io_size, io_buffers = w.io(world, parallel)
    T = w.tokens_per_rank(world) if parallel == "experts" else w.tokens
    D, dt = w.d, torch.bfloat16
    gen = torch.Generator(device=dev).manual_seed(w.seed + rank)
    gate = _randn_bf16((E_here, w.I, D), w.w_std, gen, dev)
    up = _randn_bf16((E_here, w.I, D), w.w_std, gen, dev)
    down = _randn_bf16((E_here, D, w.I), w.w_std, gen, dev)
    w_r = _randn_bf16((w.E, D), w.w_std, gen, dev)
    bias = torch.randn(w.E, generator=gen, device=dev) * w.score_bias_std if w.score_bias_std else None
    shared = None
    if w.shared_inner:
        shared = (_randn_bf16((w.shared_inner, D), w.w_std, gen, dev), _randn_bf16((w.shared_inner, D), w.w_std, gen, dev),
                  _randn_bf16((D, w.shared_inner), w.w_std, gen, dev))
    x = _randn_bf16((T, D), 1.0, gen, dev)
    x_host = x.cpu().pin_memory()
    y_host = torch.empty(T, D, dtype=dt).pin_memory()

    opts = dict(io_buffer_size=io_size, number_of_io_buffers=io_buffers, activation="silu", renormalize=True,
                router_fp32_logits=True, router_mode=w.router_mode, routed_scaling_factor=w.scale, n_group=w.n_group,
                topk_group=w.topk_group)
    if parallel == "experts":
        cluster = ShardedCluster(w.E, w.k, D, dt, dev, (gate, up, down), **opts)
    else:
        cluster = LocalCluster(w.E, [list(range(w.E))], w.k, D, dt, dev, [dev], stacked=[(gate, up, down)], **opts)
    moe = cluster.moe
    with torch.no_grad():
        moe.gate.weight.copy_(w_r)
    if bias is not None:
        moe.score_bias = bias
    if shared is not None:
        moe.set_shared_expert(*shared)
    stream = torch.cuda.current_stream(dev)
    try:
        for _ in range(args.warmup):
            moe(x)
        _barrier(dist, dev)
        N.check_device_status(dev)

        # ---------------------------------------------------------- value: device-resident input
        launches0 = N.launch_count()
        N.enable_kernel_timing(True)
        with ClockSampler(dev.index) as clk:
            _barrier(dist, dev)
            t0 = torch.cuda.Event(enable_timing=True)
            t1 = torch.cuda.Event(enable_timing=True)
            t0.record(stream)
            for _ in range(args.steps):
                moe(x)
            t1.record(stream)
            _barrier(dist, dev)
        krecs = N.kernel_records()
        ktimes = {name: [ms for ms, _ in recs] for name, recs in krecs.items()}
        N.enable_kernel_timing(False)
        launches = N.launch_count() - launches0
        ms = _max_over_ranks(dist, t0.elapsed_time(t1) / args.steps, dev)
        N.check_device_status(dev)

        # ---------------------------------------------------------- e2e: pinned host in/out
        for _ in range(2):
            y = moe(x_host.to(dev, non_blocking=True))
            y_host.copy_(y, non_blocking=True)
        _barrier(dist, dev)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            xd = x_host.to(dev, non_blocking=True)
            y = moe(xd)
            y_host.copy_(y, non_blocking=True)
        e1.record(stream)
        _barrier(dist, dev)
        e2e_ms = _max_over_ranks(dist, e0.elapsed_time(e1) / args.steps, dev)
    finally:
        cluster.close()

    if rank != 0:
        return
    burst, sustained, hbm, src = _peaks()
    # Grouped MLP launches on this GPU: FLOPs of the rows each launch computed (6 d I per
    # row) over the summed CUDA-event durations.  With one launch per step that is the
    # layer's FLOPs over the mean launch time.
    mlp = krecs.get("grouped_gated_mlp", [])
    per_launch = w.mlp_flops(T) / max(1, len(mlp) // max(1, args.steps))
    flops_each = [f if f is not None else per_launch for _, f in mlp]
    mlp_ms = statistics.mean(m for m, _ in mlp) if mlp else None
    flops = statistics.mean(flops_each) if mlp else None
    achieved = sum(flops_each) / (sum(m for m, _ in mlp) * 1e-3) / 1e12 if mlp else None
    comb = ktimes.get("combine", [])
    comb_ms = statistics.median(comb) if comb else None
    comb_bytes = T * w.k * D * 2 + T * D * 2 + T * w.k * 4
    cpu_tok_s, cores, sample = None, None, None
    if not args.no_cpu:
        ref = CpuReference(w)
        cpu_tok_s, cores, sample = ref.tokens_per_s(3), ref.threads, ref.sample(3)
    total_tokens = T * world
    line = {
        "metric": METRIC, "value": total_tokens / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong" if (w.strong and parallel == "experts") else "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": w.config(world, parallel),
        "impl": "ours",
        "e2e": {"value": total_tokens / (e2e_ms * 1e-3), "unit": "tokens/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": total_tokens * D * 2, "d2h_bytes_per_step": total_tokens * D * 2},
        "gpu_launches": launches,
        "roofline": {"bound": "tensor", "kernel": "grouped_gated_mlp (tcgen05 gate/up+SwiGLU, down)",
                     "achieved": achieved, "peak": sustained, "unit": "TFLOP/s",
                     "frac": (achieved / sustained) if achieved else None, "peak_kind": f"{src} sustained bf16",
                     "frac_of_burst_peak": (achieved / burst) if achieved else None,
                     "flops_per_launch": flops, "ms_per_launch": mlp_ms, "launches_per_step": len(mlp) / args.steps,
                     "traffic": w.traffic if parallel != "experts" else None},
        "hbm_ops": {"combine_ms": comb_ms, "combine_gbs": comb_bytes / (comb_ms * 1e-3) / 1e9 if comb_ms else None,
                    "hbm_peak_gbs": hbm,
                    "op_ms": {k: statistics.median(v) for k, v in ktimes.items() if v}},
        "cpu_baseline": {"value": cpu_tok_s, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample},
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)


def run_gemm_only(args):
    """Kernel-only mode for profiling the grouped expert MLP: X [rows, d] split evenly over
    `gemm_experts` experts of the workload's expert shape, SwiGLU, bf16.  Prints one JSON line
    with the CUDA-event time per launch pair (not a bench line)."""
    from distributedmoe_b200 import _native as N

    w = WORKLOADS[args.workload]
    dev = torch.device("cuda", 0)
    Eg, rows, D = args.gemm_experts, args.gemm_rows, w.d
    gen = torch.Generator(device=dev).manual_seed(w.seed)
    X = _randn_bf16((rows, D), 1.0, gen, dev)
    wg = _randn_bf16((Eg, w.I, D), w.w_std, gen, dev)
    wu = _randn_bf16((Eg, w.I, D), w.w_std, gen, dev)
    wd = _randn_bf16((Eg, D, w.I), w.w_std, gen, dev)
    Y = torch.empty(rows, D, dtype=torch.bfloat16, device=dev)
    ends = [rows * (e + 1) // Eg for e in range(Eg)]
    for _ in range(args.warmup):
        N.grouped_gated_mlp(X, wg, wu, wd, list(range(Eg)), ends, N.ACT_SILU, Y)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.steps):
        N.grouped_gated_mlp(X, wg, wu, wd, list(range(Eg)), ends, N.ACT_SILU, Y)
    b.record()
    torch.cuda.synchronize()
    N.check_device_status(dev)
    ms = a.elapsed_time(b) / args.steps
    print(json.dumps({"mode": "gemm", "workload": w.name, "rows": rows, "experts": Eg, "ms_per_launch_pair": ms,
                      "tflops": 6.0 * rows * D * w.I / (ms * 1e-3) / 1e12}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="mixtral", choices=sorted(WORKLOADS))
    ap.add_argument("--tokens", type=int, default=None,
                    help="tokens per step: per GPU for weak-scaling workloads, in all for the others")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--parallel", default="experts", choices=["experts", "replicas"],
                    help="with N > 1 GPUs: shard the experts over the GPUs, or run one layer per GPU")
    ap.add_argument("--mode", default="layer", choices=["layer", "gemm"],
                    help="gemm: time only the grouped expert MLP (for kernel profiling)")
    ap.add_argument("--gemm-rows", type=int, default=4096)
    ap.add_argument("--gemm-experts", type=int, default=2)
    args = ap.parse_args()
    if args.tokens is not None:
        if args.tokens < 1:
            raise SystemExit("--tokens must be positive")
        WORKLOADS[args.workload].tokens = args.tokens
    if args.mode == "gemm":
        run_gemm_only(args)
        return
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        run_reference(args, int(os.environ.get("RANK", "0")))
        return
    dist, rank, world, local_rank = _dist()
    try:
        run_ours(args, dist, rank, world, local_rank)
    finally:
        if dist is not None:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
