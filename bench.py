"""MoE-layer throughput benchmark (tokens/s) of the B200 framework, or of the reference's
CPU path with ``--impl reference``.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload mixtral|deepseek|qwen3-decode|skewed-ft] [--data-plane direct|tasks]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 ... bench.py --gpus N

Workload (one step): one forward of a Mixtral-8x7B-shape MoE layer, T=4096 tokens, d=4096,
E=8 experts, top-2 softmax routing renormalised over fp32 router logits, SwiGLU experts with
inner dim 14336, bf16, seeded synthetic N(0,1) activations and N(0,0.02) weights.  The
layer runs through the drop-in API: ``DistMoEBlock.forward`` with one ``DistExpertsBlock``
holding the 8 experts on the same GPU.  ``--data-plane direct`` (default) uses the
NVLinkDirect backend, whose forward is device-driven (router, routing plan, count exchange,
gather into the receive window, one grouped MLP, combine; no host synchronisation);
``--data-plane tasks`` uses the reference's task protocol over the NVLinkIPC backend.

* ``value``: tokens/s of forwards whose input is already in HBM (device-timed with CUDA
  events, barrier + synchronize on both sides; max over ranks).
* ``e2e``: the same API with the input in pinned host memory: the H2D copy of the tokens and
  the D2H read of the layer output are inside the timed region.
* ``roofline``: the grouped expert MLP (the tcgen05 GEMM pair) timed with CUDA events on the
  stream it is launched on during the timed steps, against the measured bf16 burst peak (a
  region of tens of milliseconds, not a seconds-long run under the power cap); the
  bandwidth-bound kernels (router, gather, combine) against the measured HBM copy peak.
* ``cpu_baseline``: the oracle port of the reference's torch path (routing +
  ``local_experts``), timed on this host's cores.

With N GPUs (``--parallel experts``, the default for N > 1) the experts are sharded: GPU g
holds experts [g*E/N, (g+1)*E/N), every rank hosts its own tokens and sends each token to
the GPUs of its experts (one ``DistMoEBlock`` per rank whose expert blocks span all N GPUs).
Mixtral keeps 4096 tokens per GPU (weak scaling); DeepSeek and Qwen3 decode keep the total
fixed (strong scaling).  ``--parallel replicas`` runs an independent layer per rank.  The
expert weights exceed the 126 MB L2, so every step streams them from HBM.

``--workload skewed-ft``: the Mixtral shape with every expert in two blocks, a Zipf(1.2)
router bias, the even split over alive replicas, one block disabled half-way through the
timed steps and enabled again at three quarters; it reports tokens/s per phase and checks a
token sample of every step against the oracle.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
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
# DRAM bytes of the grouped MLP (both GEMMs of one launch) for the Mixtral workload, from
# `ncu --metrics dram__bytes_read.sum,dram__bytes_write.sum` over the layer's launches (one
# pass): GEMM1 read + write, GEMM2 read + write.  None for workloads without a capture.
MIXTRAL_MLP_TRAFFIC_BYTES = (2018 + 228 + 1417 + 62) * 10**6


class Workload:
    """One benchmark configuration: layer shape, routing, initialisation and how tokens and
    experts spread over the GPUs."""

    def __init__(self, name, *, tokens, d, E, k, I, seed, w_std, router_mode="softmax", n_group=1,
                 topk_group=1, scale=1.0, score_bias_std=0.0, shared_inner=0, strong=False, io_max=8192,
                 traffic=None, replicas=1, zipf_s=0.0, fail_block=None):
        self.name, self.tokens, self.d, self.E, self.k, self.I = name, tokens, d, E, k, I
        self.seed, self.w_std, self.router_mode = seed, w_std, router_mode
        self.n_group, self.topk_group, self.scale = n_group, topk_group, scale
        self.score_bias_std, self.shared_inner, self.strong = score_bias_std, shared_inner, strong
        self.io_max, self.traffic = io_max, traffic
        self.replicas, self.zipf_s, self.fail_block = replicas, zipf_s, fail_block

    def tokens_per_rank(self, world: int) -> int:
        return self.tokens // world if self.strong else self.tokens

    def blocks(self, world: int):
        """(expert_blocks, block_ranks).  One block per GPU holding a contiguous E/world
        share; with two replicas every block also holds the next block's share (on one GPU:
        E blocks of two consecutive experts)."""
        E = self.E
        if self.replicas == 1:
            return [list(range(g * E // world, (g + 1) * E // world)) for g in range(world)], list(range(world))
        if world == 1:
            return [[b, (b + 1) % E] for b in range(E)], [0] * E
        share = [list(range(g * E // world, (g + 1) * E // world)) for g in range(world)]
        return [share[g] + share[(g + 1) % world] for g in range(world)], list(range(world))

    def io(self, world: int, parallel: str) -> tuple:
        """(io_buffer_size, number_of_io_buffers) for one host of `world` ranks (task plane)."""
        if parallel != "experts":
            return self.io_max, max(2, -(-self.tokens * self.k // self.io_max))
        per_block = self.tokens_per_rank(world) * self.k // world
        size = min(self.io_max, max(256, -(-(per_block * 3 // 2) // 256) * 256))
        return size, 2 * world

    def mlp_flops(self, rows: int) -> float:
        """Routed grouped-MLP FLOPs of `rows` expert rows (6 d I each)."""
        return 6.0 * rows * self.d * self.I

    def config(self, world: int, parallel: str, data_plane: str) -> dict:
        T = self.tokens_per_rank(world)
        blocks, _ = self.blocks(world if parallel == "experts" else 1)
        if parallel == "experts":
            par = f"ep{world}: {len(blocks[0])} expert instances per GPU, one host per GPU with {T} tokens"
        elif parallel == "replicas":
            par = f"replicas x{world}"
        else:
            par = "single gpu"
        router = (f"sigmoid + selection bias N(0,{self.score_bias_std}), {self.n_group} groups / top-{self.topk_group}, "
                  f"top-{self.k} renormalised x{self.scale}, fp32 logits" if self.router_mode == "sigmoid_group"
                  else f"softmax top-{self.k} renormalised, fp32 logits")
        if self.zipf_s:
            router += f", Zipf(s={self.zipf_s}) logit bias"
        c = {"workload": self.name, "tokens_per_gpu": T, "tokens_per_step": T * world, "hidden": self.d,
             "experts": self.E, "top_k": self.k, "inner": self.I, "router": router, "activation": "silu (SwiGLU)",
             "expert_blocks": len(blocks), "replicas": self.replicas,
             "transfer_engine": "NVLinkDirect" if data_plane == "direct" else "NVLinkIPC",
             "data_plane": "device-driven exchange" if data_plane == "direct" else "task protocol",
             "l2": "no flush: the expert weights exceed the 126 MB L2 every step",
             "parallelism": par, "seed": self.seed}
        if data_plane == "tasks":
            c["io_buffer_size"], c["io_buffers"] = self.io(world, parallel)
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
    # Skewed-load fault-tolerance run: Mixtral shape, 16384 tokens per step in all, every
    # expert in two blocks, Zipf(1.2) router bias, one block lost half-way.
    "skewed-ft": Workload("skewed-fault-tolerance-mixtral-moe-layer", tokens=16384, d=4096, E=8, k=2, I=14336,
                          seed=4, w_std=0.02, strong=True, io_max=32768, replicas=2, zipf_s=1.2, fail_block=3),
}


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["bf16_tflops"]), float(p["bf16_tflops_sustained"]), float(p["hbm_gbs"]), "measured"
    except Exception:
        return 1590.0, 1400.0, 6650.0, "fallback"


class ClockSampler:
    """SM clock, power and throttle reasons of one GPU, sampled through NVML every 20 ms during
    the timed region.  Without NVML nothing is sampled and the summary says so."""

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
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [],
                    "not_sampled": "NVML unavailable or returned no samples"}
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
    bf16, weighted index_add; plus the shared expert).  It runs the workload's full token
    count when one step fits the time budget, else the largest power-of-two sample that does
    (the sample is stated in the line)."""

    def __init__(self, w: Workload, tokens: int, step_budget_s: float = 8.0):
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
        self.logit_bias = _zipf_bias(w) if w.zipf_s else None
        self.shared = None
        if w.shared_inner:
            self.shared = tuple((torch.randn(*sh, generator=g) * w.w_std).to(bf)
                                for sh in ((w.shared_inner, w.d), (w.shared_inner, w.d), (w.d, w.shared_inner)))
        self.g = g
        self.full = tokens
        n = min(64, tokens)
        dt = self.step(n)
        while n < tokens and dt * min(2 * n, tokens) / n < step_budget_s:
            n = min(2 * n, tokens)
            dt = self.step(n)
        self.n = n

    def step(self, n: int = 0) -> float:
        n = n or self.n
        O, w = self.O, self.w
        x = torch.randn(n, w.d, generator=self.g).to(torch.bfloat16)
        mode = O.ROUTER_SIGMOID_GROUP if w.router_mode == "sigmoid_group" else O.ROUTER_SOFTMAX
        t0 = time.perf_counter()
        logits = O.router_logits(x, self.wr, fp32_logits=True, logit_bias=self.logit_bias)
        O.local_experts(x, logits, self.wg, self.wu, self.wd, w.k, act=O.ACT_SILU, renormalize=True, mode=mode,
                        score_bias=self.bias, scale=w.scale, n_group=w.n_group, topk_group=w.topk_group,
                        shared=self.shared)
        return time.perf_counter() - t0

    def sample(self, reps: int) -> str:
        what = "the full" if self.n == self.full else f"a {self.n}-token sample of the {self.full}-token"
        return (f"{what} {self.w.name} step (full-size bf16 weights, torch CPU, {self.threads} threads), "
                f"{reps} steps, tokens/s = tokens / seconds")

    def tokens_per_s(self, reps: int = 3) -> float:
        return self.n / statistics.median(self.step() for _ in range(reps))


def run_reference(args, rank):
    """The oracle port of the reference's CPU torch path, on this host's cores (rank 0 only)."""
    if rank != 0:
        return
    w = WORKLOADS[args.workload]
    parallel = args.parallel if args.gpus > 1 else "single"
    total = w.tokens_per_rank(args.gpus) * args.gpus
    # Each step runs the full token count when the whole run fits about a minute, else the
    # largest power-of-two sample that does.
    ref = CpuReference(w, total, step_budget_s=min(8.0, 60.0 / (args.steps + args.warmup)))
    for _ in range(args.warmup):
        ref.step()
    steps = args.steps
    times = [ref.step() for _ in range(steps)]
    tok_s = ref.n * len(times) / sum(times)
    line = {"metric": METRIC, "value": tok_s, "unit": "tokens/s", "n_gpus": args.gpus, "steps": steps,
            "warmup": args.warmup, "ms_per_step": total / tok_s * 1e3,
            "higher_is_better": True, "scaling": "strong" if w.strong else "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": w.config(args.gpus, parallel, args.data_plane), "impl": "reference",
            "cpu_baseline": {"value": tok_s, "unit": "tokens/s", "cores": ref.threads, "kind": "port",
                             "sample": ref.sample(steps)},
            "e2e": {"value": tok_s, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- the layer
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


def expert_weights(w: Workload, experts, dev):
    """(gate [n, I, d], up [n, I, d], down [n, d, I]) of the listed experts, in list order.
    Expert e's weights come from its own seed, so every rank (and the oracle) can make any
    expert's weights."""
    n = len(experts)
    gate = torch.empty(n, w.I, w.d, dtype=torch.bfloat16, device=dev)
    up = torch.empty_like(gate)
    down = torch.empty(n, w.d, w.I, dtype=torch.bfloat16, device=dev)
    for i, e in enumerate(experts):
        gen = torch.Generator(device=dev).manual_seed(w.seed * 1_000_003 + 7919 * int(e) + 1)
        gate[i] = _randn_bf16((1, w.I, w.d), w.w_std, gen, dev)[0]
        up[i] = _randn_bf16((1, w.I, w.d), w.w_std, gen, dev)[0]
        down[i] = _randn_bf16((1, w.d, w.I), w.w_std, gen, dev)[0]
    return gate, up, down


def _zipf_bias(w: Workload, dev=None) -> torch.Tensor:
    """Zipf(s) log-bias per expert: -s * log(rank), ranks a seeded permutation of 1..E."""
    ranks = torch.randperm(w.E, generator=torch.Generator().manual_seed(w.seed)) + 1
    b = torch.tensor([-w.zipf_s * math.log(float(r)) for r in ranks], dtype=torch.float32)
    return b if dev is None else b.to(dev)


class Layer:
    """The benchmark layer exactly as this file measures it: weights, router, the cluster
    (LocalCluster on one GPU, ShardedCluster over ranks) and this rank's input tokens."""

    def __init__(self, w: Workload, dev: torch.device, world: int = 1, rank: int = 0, parallel: str = "single",
                 data_plane: str = "direct", x_seed_offset: int = 0, cuda_graphs: bool = False,
                 expert_precision: str = "model"):
        from distributedmoe_b200.MoE.local_cluster import LocalCluster
        from distributedmoe_b200.MoE.sharded_cluster import ShardedCluster
        from distributedmoe_b200.TensorTransferEngine import TensorTransferEngineBackend as B

        self.w, self.dev, self.world, self.rank = w, dev, world, rank
        ep = parallel == "experts" and world > 1
        backend = B.NVLinkDirect if data_plane == "direct" else B.NVLinkIPC
        self.T = w.tokens_per_rank(world) if ep else w.tokens
        blocks, block_ranks = w.blocks(world if ep else 1)
        self.blocks, self.block_ranks = blocks, block_ranks
        gen = torch.Generator(device=dev).manual_seed(w.seed)
        D = w.d
        self.w_r = _randn_bf16((w.E, D), w.w_std, gen, dev)
        self.score_bias = torch.randn(w.E, generator=gen, device=dev) * w.score_bias_std if w.score_bias_std else None
        self.shared = None
        if w.shared_inner:
            self.shared = (_randn_bf16((w.shared_inner, D), w.w_std, gen, dev),
                           _randn_bf16((w.shared_inner, D), w.w_std, gen, dev),
                           _randn_bf16((D, w.shared_inner), w.w_std, gen, dev))
        xgen = torch.Generator(device=dev).manual_seed(w.seed + 7 * rank + 1 + x_seed_offset)
        self.x = _randn_bf16((self.T, D), 1.0, xgen, dev)
        opts = dict(activation="silu", renormalize=True, router_fp32_logits=True, router_mode=w.router_mode,
                    routed_scaling_factor=w.scale, n_group=w.n_group, topk_group=w.topk_group,
                    expert_block_policy="least_loaded" if w.replicas > 1 else "fifo")
        if ep:
            mine = blocks[rank]
            self.stack = expert_weights(w, mine, dev)
            if data_plane == "direct":
                opts["cuda_graphs"] = cuda_graphs
                opts["expert_precision"] = expert_precision
            self.cluster = ShardedCluster(w.E, w.k, D, torch.bfloat16, dev, self.stack, backend=backend,
                                          max_tokens=self.T, blocks=blocks, **opts,
                                          **({} if data_plane == "direct" else dict(zip(
                                              ("io_buffer_size", "number_of_io_buffers"), w.io(world, parallel)))))
        else:
            distinct = sorted({e for b in blocks for e in b})
            full = expert_weights(w, distinct, dev)
            pos = {e: i for i, e in enumerate(distinct)}
            stacks = []
            for b in blocks:
                idx = torch.tensor([pos[e] for e in b], device=dev)
                stacks.append(tuple(t if len(blocks) == 1 else t.index_select(0, idx).contiguous() for t in full))
            self.stack = full
            io_size, io_buffers = w.io(1, "single")
            if data_plane == "direct":
                opts["cuda_graphs"] = cuda_graphs
                opts["expert_precision"] = expert_precision
            self.cluster = LocalCluster(w.E, blocks, w.k, D, torch.bfloat16, dev, [dev] * len(blocks),
                                        stacked=stacks, io_buffer_size=io_size, number_of_io_buffers=io_buffers,
                                        backend=backend, max_tokens=self.T, **opts)
        self.moe = self.cluster.moe
        with torch.no_grad():
            self.moe.gate.weight.copy_(self.w_r)
        self.logit_bias = None
        if w.zipf_s:
            lin = torch.nn.Linear(D, w.E, bias=True, dtype=torch.bfloat16, device=dev)
            with torch.no_grad():
                lin.weight.copy_(self.w_r)
                lin.bias.copy_(_zipf_bias(w, dev).to(torch.bfloat16))
            self.moe.gate = lin
            self.logit_bias = lin.bias.detach().float()
        if self.score_bias is not None:
            self.moe.score_bias = self.score_bias
        if self.shared is not None:
            self.moe.set_shared_expert(*self.shared)

    def close(self):
        self.cluster.close()


def oracle_fp32(layer: Layer, x: torch.Tensor, experts_weights=None) -> torch.Tensor:
    """The oracle's layer output for tokens x in fp32 on x's device (routing from the
    router kernel's fp32 logits, which the routing tests pin to the oracle's)."""
    from distributedmoe_b200 import _native as N
    from oracle import moe_oracle as O

    w = layer.w
    _, _, logits = N.router(x, layer.w_r, w.k, logit_bias=layer.logit_bias, want_logits=True)
    g, u, dn = experts_weights if experts_weights is not None else layer.stack
    mode = O.ROUTER_SIGMOID_GROUP if w.router_mode == "sigmoid_group" else O.ROUTER_SOFTMAX
    return O.local_experts(x, logits, g, u, dn, w.k, act=O.ACT_SILU, renormalize=True, mode=mode,
                           score_bias=layer.score_bias, scale=w.scale, n_group=w.n_group, topk_group=w.topk_group,
                           shared=layer.shared, compute_dtype=torch.float32)


# ----------------------------------------------------------------------------- GPU (ours)
def _op_stats(krecs, name, steps):
    recs = krecs.get(name, [])
    if not recs:
        return None
    ms = [m for m, _ in recs]
    return {"launches_per_step": len(recs) / steps, "ms_per_launch": statistics.mean(ms), "ms_total": sum(ms)}


def _e2e_pipelined(moe, x_host, dev, stream, steps, dist) -> float:
    """ms per step of `steps` forwards fed from pinned host memory and read back to pinned
    host memory, with the copies on their own streams (double-buffered on both sides)."""
    copy_in = torch.cuda.Stream(device=dev)
    copy_out = torch.cuda.Stream(device=dev)
    xd = [torch.empty(x_host.shape, dtype=x_host.dtype, device=dev) for _ in range(2)]
    y_host = [torch.empty(x_host.shape, dtype=x_host.dtype).pin_memory() for _ in range(2)]
    in_done = [torch.cuda.Event() for _ in range(2)]
    used = [torch.cuda.Event() for _ in range(2)]  # the layer finished reading xd[i]
    out_done = [torch.cuda.Event() for _ in range(2)]

    def run(n, t0=None):
        for i in range(2):
            used[i].record(stream)
            out_done[i].record(copy_out)
        if t0 is not None:
            t0.record(stream)
        copy_in.wait_stream(stream)
        copy_out.wait_stream(stream)
        for s in range(n):
            b = s % 2
            copy_in.wait_event(used[b])
            with torch.cuda.stream(copy_in):
                xd[b].copy_(x_host, non_blocking=True)
                in_done[b].record(copy_in)
            stream.wait_event(in_done[b])
            y = moe(xd[b])
            used[b].record(stream)
            copy_out.wait_event(used[b])
            copy_out.wait_event(out_done[b])  # y_host[b] is free again
            with torch.cuda.stream(copy_out):
                y_host[b].copy_(y, non_blocking=True)
                out_done[b].record(copy_out)
            y.record_stream(copy_out)
        stream.wait_stream(copy_out)

    run(2)
    # Three timed repetitions, the median reported: the host links of these GPUs are shared
    # with other jobs on the machine, and one repetition can catch another job's transfers.
    reps = []
    for _ in range(3):
        _barrier(dist, dev)
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        run(steps, t0)
        t1.record(stream)
        _barrier(dist, dev)
        reps.append(_max_over_ranks(dist, t0.elapsed_time(t1) / steps, dev))
    return sorted(reps)[1]


def run_ours(args, dist, rank, world, local_rank):
    from distributedmoe_b200 import _native as N

    w = WORKLOADS[args.workload]
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    parallel = args.parallel if world > 1 else "single"
    if parallel == "experts" and w.E % world:
        raise SystemExit(f"--parallel experts needs a GPU count that divides {w.E}")
    graphs = args.cuda_graphs == "on" or (args.cuda_graphs == "auto" and w.name.endswith("decode-moe-layer"))
    graphs = graphs and args.data_plane == "direct"
    fp8 = args.expert_precision == "fp8"
    if fp8 and args.data_plane != "direct":
        raise SystemExit("--expert-precision fp8 runs on the direct data plane")
    layer = Layer(w, dev, world, rank, parallel, args.data_plane, cuda_graphs=graphs,
                  expert_precision="fp8" if fp8 else "model")
    moe, x, T, D = layer.moe, layer.x, layer.T, w.d
    x_host = x.cpu().pin_memory()
    y_host = torch.empty(T, D, dtype=torch.bfloat16).pin_memory()
    stream = torch.cuda.current_stream(dev)
    ft = w.fail_block is not None
    lost = w.fail_block % len(layer.blocks) if ft else None
    try:
        for _ in range(args.warmup):
            moe(x)
        _barrier(dist, dev)
        N.check_device_status(dev)

        # ---------------------------------------------------------- value: device-resident input
        launches0 = N.launch_count()
        N.enable_kernel_timing(True)
        step_ev = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)] if ft else None
        samples = []
        with ClockSampler(dev.index) as clk:
            _barrier(dist, dev)
            t0 = torch.cuda.Event(enable_timing=True)
            t1 = torch.cuda.Event(enable_timing=True)
            t0.record(stream)
            for s in range(args.steps):
                if ft:
                    step_ev[s].record(stream)
                    if s == args.steps // 2:
                        moe.disable_experts_block(lost)
                    if s == (3 * args.steps) // 4:
                        moe.enable_experts_block(lost)
                    y = moe(x)
                    samples.append(y[::256].clone())
                else:
                    moe(x)
            t1.record(stream)
            if ft:
                step_ev[args.steps].record(stream)
            _barrier(dist, dev)
        krecs = N.kernel_records()
        N.enable_kernel_timing(False)
        launches = N.launch_count() - launches0
        ms = _max_over_ranks(dist, t0.elapsed_time(t1) / args.steps, dev)
        N.check_device_status(dev)

        # ---------------------------------------------------------- e2e: pinned host in/out
        # Serial: every step copies its tokens in, runs the layer and copies the result out
        # on one stream.
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
        e2e_serial_ms = _max_over_ranks(dist, e0.elapsed_time(e1) / args.steps, dev)
        # Pipelined (a serving loop): the same copies on two copy streams, so step i+1's H2D
        # and step i-1's D2H overlap step i's layer (PCIe runs both directions at once).
        # Every copy of every step is inside the timed region.
        e2e_ms = _e2e_pipelined(moe, x_host, dev, stream, args.steps, dist)
        N.check_device_status(dev)

        ft_report = None
        if ft:
            per_step = [step_ev[s].elapsed_time(step_ev[s + 1]) for s in range(args.steps)]
            h, q = args.steps // 2, (3 * args.steps) // 4
            phase = lambda a, b: (T * world * (b - a) / (sum(per_step[a:b]) * 1e-3)) if b > a else None
            everything = expert_weights(w, list(range(w.E)), dev) if parallel == "experts" else None
            ref = oracle_fp32(layer, x[::256].contiguous(), everything)
            errs = [((y.float() - ref).norm() / ref.norm()).item() for y in samples]
            worst = _max_over_ranks(dist, max(errs), dev)
            ft_report = {"tokens_per_s_before": phase(0, h), "tokens_per_s_block_lost": phase(h, q),
                         "tokens_per_s_restored": phase(q, args.steps), "lost_block": lost,
                         "lost_at_step": h, "restored_at_step": q,
                         "parity": {"steps_checked": args.steps, "tokens_per_step_checked": samples[0].shape[0],
                                    "max_rel_l2": worst, "bar": 1e-2, "ok": worst < 1e-2}}
    finally:
        layer.close()

    if rank != 0:
        return
    burst, sustained, hbm, src = _peaks()
    steps = args.steps
    # Routed grouped MLP: FLOPs of the rows it computed over its CUDA-event time.  On one GPU
    # every routed row is computed here (T * k rows, 6 d I FLOPs each).
    mlp = _op_stats(krecs, "grouped_gated_mlp", steps)
    roof = None
    if mlp is not None:
        host_table_flops = [f for _, f in krecs["grouped_gated_mlp"] if f is not None]
        if host_table_flops:
            flops_step = sum(host_table_flops) / steps
        else:
            flops_step = w.mlp_flops(T * w.k) if world == 1 or parallel != "experts" else None
        achieved = flops_step / (mlp["ms_total"] / steps * 1e-3) / 1e12 if flops_step else None
        roof = {"bound": "tensor", "kernel": "grouped_gated_mlp (tcgen05 gate/up+SwiGLU, down)",
                "achieved": achieved, "peak": burst, "unit": "TFLOP/s",
                "frac": achieved / burst if achieved else None,
                "peak_kind": f"{src} burst bf16 (timed region of {steps} steps, {ms * steps:.0f} ms)",
                "frac_of_sustained_peak": achieved / sustained if achieved else None,
                "sustained_peak": sustained,
                "flops_per_launch": flops_step / mlp["launches_per_step"] if flops_step else None,
                "ms_per_launch": mlp["ms_per_launch"], "launches_per_step": mlp["launches_per_step"],
                "traffic": w.traffic if (parallel != "experts" and world == 1) else None}
        # Bandwidth-bound kernels: algorithmic bytes per launch over their CUDA-event time.
        n_act = T * w.k
        movers = {
            "router": (T * D * 2 + w.E * D * 2 + n_act * 12, "x read + router weights + indices/weights out"),
            "ep_dispatch": (2 * n_act * ((D + 16) if fp8 else D * 2) + n_act * 8,
                            "routed rows read + written, indices" + (" (8-bit records, d + 16 bytes)" if fp8 else "")),
            "quantize_rows_e4m3": (T * D * 2 + T * (D + 16), "tokens read (bf16), records written"),
            "ep_combine": (n_act * D * 2 + T * D * 2 + n_act * 12, "routed rows read, tokens written, indices"),
            "permute_rows": (None, "task-plane gathers"),
            "combine": (n_act * D * 2 + T * D * 2 + n_act * 8, "permuted rows read, tokens written"),
        }
        hbm_ops = {}
        for name, (nbytes, what) in movers.items():
            st = _op_stats(krecs, name, steps)
            if st is None or nbytes is None:
                continue
            per = nbytes / st["launches_per_step"]
            gbs = per / (st["ms_per_launch"] * 1e-3) / 1e9
            hbm_ops[name] = {"us_per_launch": st["ms_per_launch"] * 1e3, "bytes_per_launch": per, "bytes": what,
                             "gbs": gbs, "frac": gbs / hbm}
        roof["hbm"] = {"peak_gbs": hbm, "peak_kind": f"{src} copy", "ops": hbm_ops}
        if fp8:
            roof["note"] = ("gate/up GEMM on e4m3 tensor cores (nominally twice the bf16 rate), down GEMM bf16; "
                            "the peak is the measured bf16 one")
    op_us = {name: _op_stats(krecs, name, steps)["ms_per_launch"] * 1e3 for name in krecs if krecs[name]}
    cpu_tok_s, cores, sample = None, None, None
    if not args.no_cpu:
        ref = CpuReference(w, T * world)
        cpu_tok_s, cores, sample = ref.tokens_per_s(3), ref.threads, ref.sample(3)
    total_tokens = T * world
    line = {
        "metric": METRIC, "value": total_tokens / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world,
        "steps": steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong" if (w.strong and parallel == "experts") else "weak",
        "vs_baseline": None, "dtype": "e4m3 gate/up, bf16 down and combine" if fp8 else "bf16", "data": "synthetic",
        "config": dict(w.config(world, parallel, args.data_plane), cuda_graphs=graphs,
                       **({"expert_precision": "fp8"} if fp8 else {})), "impl": "ours",
        "e2e": {"value": total_tokens / (e2e_ms * 1e-3), "unit": "tokens/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": total_tokens * D * 2, "d2h_bytes_per_step": total_tokens * D * 2,
                "copies": "pinned host in/out every step; H2D of step i+1 and D2H of step i-1 on two copy "
                          "streams overlapping step i; median of three timed repetitions",
                "serial": {"value": total_tokens / (e2e_serial_ms * 1e-3), "ms_per_step": e2e_serial_ms,
                           "copies": "H2D, layer, D2H back to back on one stream"}},
        "gpu_launches": launches,
        "roofline": roof,
        "op_us": op_us,
        "cpu_baseline": {"value": cpu_tok_s, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample},
        "clocks": clk.summary(),
    }
    if ft_report is not None:
        line["fault_tolerance"] = ft_report
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
    if args.gemm_ragged:
        # Ragged experts as top-k routing makes them: binomial-like sizes around rows / Eg.
        gs = torch.Generator().manual_seed(w.seed + 5)
        share = torch.full((Eg,), rows / Eg) + torch.randn(Eg, generator=gs) * (rows / Eg) ** 0.5
        share = share.clamp_min(0)
        cuts = (share.cumsum(0) * rows / share.sum()).round().long().tolist()
        ends = [min(rows, max(0, c)) for c in cuts]
        ends[-1] = rows
    fp8 = args.expert_precision == "fp8"
    if fp8:  # operands quantised once, outside the timed region: the GEMM pair alone is timed
        xq, xs = N.quantize_rows_e4m3(X)
        ex = N.Fp8Experts(wg, wu, wd)

    def launch():
        if fp8:
            N.grouped_gated_mlp_fp8(xq, xs, ex, list(range(Eg)), ends, N.ACT_SILU, Y)
        else:
            N.grouped_gated_mlp(X, wg, wu, wd, list(range(Eg)), ends, N.ACT_SILU, Y)

    for _ in range(args.warmup):
        launch()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.steps):
        launch()
    b.record()
    torch.cuda.synchronize()
    N.check_device_status(dev)
    ms = a.elapsed_time(b) / args.steps
    print(json.dumps({"mode": "gemm", "workload": w.name, "rows": rows, "experts": Eg, "ms_per_launch_pair": ms,
                      "segment_rows": [b - a for a, b in zip([0] + ends[:-1], ends)] if args.gemm_ragged else None,
                      "precision": "e4m3 gate/up, bf16 down" if fp8 else "bf16",
                      "tflops": 6.0 * rows * D * w.I / (ms * 1e-3) / 1e12}), flush=True)


def run_movers(args):
    """Kernel-only mode for profiling the bandwidth-bound kernels of one forward on one GPU,
    without expert weights: router, routing plan, exchange placement, gather into the
    receive window, combine, at the workload's token count.  Prints one JSON line with the
    CUDA-event time and algorithmic GB/s per kernel (not a bench line)."""
    from distributedmoe_b200 import _native as N
    from distributedmoe_b200.MoE.instances import InstanceTable

    w = WORKLOADS[args.workload]
    dev = torch.device("cuda", 0)
    T, D, E, k = w.tokens, w.d, w.E, w.k
    gen = torch.Generator(device=dev).manual_seed(w.seed)
    x = _randn_bf16((T, D), 1.0, gen, dev)
    w_r = _randn_bf16((E, D), w.w_std, gen, dev)
    score_bias = torch.randn(E, generator=gen, device=dev) * w.score_bias_std if w.score_bias_std else None
    n = T * k
    recv = torch.empty(n, D, dtype=torch.bfloat16, device=dev)
    back = torch.full((n,), -1, dtype=torch.int32, device=dev)
    rows = _randn_bf16((n, D), 1.0, gen, dev)
    flags = torch.zeros(N.ep_flags_bytes() // 8, dtype=torch.int64, device=dev)
    win = N.ep_window(1, 0, [flags.data_ptr()], [0], [recv.data_ptr()], [back.data_ptr()], [rows.data_ptr()])
    inst = InstanceTable.from_blocks([list(range(E))], [0], 1, E)
    alive_n, alive_inst = inst.alive_arrays([True])
    i32 = dict(dtype=torch.int32, device=dev)
    R = N.EP_MAX_REPLICAS
    table = (torch.tensor(alive_n, **i32), torch.tensor(alive_inst, **i32), torch.tensor(inst.inst_rank, **i32),
             torch.tensor(inst.inst_slot, **i32), torch.tensor(inst.inst_first, **i32))
    place = (torch.zeros(E, **i32), torch.zeros(E * R, **i32), torch.zeros(E * (R + 1), **i32),
             torch.zeros(E, **i32))
    segs = (torch.zeros(E, **i32), torch.zeros(E, **i32))
    ret, done = torch.empty(n, **i32), torch.zeros(1, **i32)
    out = torch.empty(T, D, dtype=torch.bfloat16, device=dev)
    mode = N.ROUTER_SIGMOID_GROUP if w.router_mode == "sigmoid_group" else N.ROUTER_SOFTMAX

    def one():
        idx, wts, _ = N.router(x, w_r, k, mode=mode, renormalize=True, scale=w.scale, score_bias=score_bias,
                               n_group=w.n_group, topk_group=w.topk_group, w_dtype=torch.float32)
        plan = N.route_plan(idx, None, E, want_slot=True, want_weight=False)
        N.ep_plan(win, plan["counts"], E, E, N.EP_POLICY_ROTATE, table, n, 10**9, place + segs)
        N.ep_dispatch(win, x, T, k, E, plan["offsets"], plan["perm_token"], plan["perm_slot"], place, table[2], n, ret,
                      done)
        N.ep_combine(win, plan["inverse"], ret, wts, T, k, out)

    for _ in range(args.warmup):
        one()
    torch.cuda.synchronize()
    N.enable_kernel_timing(True)
    for _ in range(args.steps):
        one()
    recs = N.kernel_records()
    N.enable_kernel_timing(False)
    N.check_device_status(dev)
    _, _, hbm, src = _peaks()
    nbytes = {"router": T * D * 2 + E * D * 2 + n * 12, "ep_dispatch": 2 * n * D * 2 + n * 12,
              "ep_combine": n * D * 2 + T * D * 2 + n * 12}
    res = {}
    for name, r in recs.items():
        us = statistics.median(m for m, _ in r) * 1e3
        res[name] = {"us": us}
        if name in nbytes:
            res[name]["gbs"] = nbytes[name] / (us * 1e-6) / 1e9
            res[name]["frac_of_hbm"] = res[name]["gbs"] / hbm
    print(json.dumps({"mode": "movers", "workload": w.name, "tokens": T, "hbm_peak_gbs": hbm, "peak_kind": src,
                      "ops": res}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="mixtral", choices=sorted(WORKLOADS))
    ap.add_argument("--data-plane", default="direct", choices=["direct", "tasks"],
                    help="direct: device-driven NVLinkDirect exchange; tasks: the reference's task protocol")
    ap.add_argument("--tokens", type=int, default=None,
                    help="tokens per step: per GPU for weak-scaling workloads, in all for the others")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--cuda-graphs", default="auto", choices=["auto", "on", "off"],
                    help="replay each forward from a captured CUDA graph (auto: for the decode workload)")
    ap.add_argument("--parallel", default="experts", choices=["experts", "replicas"],
                    help="with N > 1 GPUs: shard the experts over the GPUs, or run one layer per GPU")
    ap.add_argument("--mode", default="layer", choices=["layer", "gemm", "movers"],
                    help="gemm: time only the grouped expert MLP; movers: only the router, plan, gather and "
                         "combine (for kernel profiling)")
    ap.add_argument("--expert-precision", default="bf16", choices=["bf16", "fp8"],
                    help="fp8: routed experts on 8-bit records and e4m3 gate/up GEMMs (not the headline "
                         "precision: the headline line is bf16)")
    ap.add_argument("--gemm-rows", type=int, default=4096)
    ap.add_argument("--gemm-experts", type=int, default=2)
    ap.add_argument("--gemm-ragged", action="store_true",
                    help="--mode gemm: uneven expert segments (about rows/experts +- its square root)")
    args = ap.parse_args()
    if args.tokens is not None:
        if args.tokens < 1:
            raise SystemExit("--tokens must be positive")
        WORKLOADS[args.workload].tokens = args.tokens
    if args.mode == "gemm":
        run_gemm_only(args)
        return
    if args.mode == "movers":
        run_movers(args)
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
