#!/usr/bin/env python
"""Benchmark of the B200 2-bit MoE layer (qmoe-rs hot path).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline workload (configs[3] of the benchmark definition): one
DeepSeek-V3-shaped MoE layer -- hidden 7168, 256 routed experts, sigmoid
scoring with 8 groups of which the best 4 are kept, top-8 experts with
renormalised weights scaled by 2.5, one shared expert, expert intermediate
2048, SwiGLU -- over 4096 bf16 tokens per GPU.  On N GPUs the layer is
expert-parallel (256 / N experts per GPU, the gate and the shared expert on
every GPU, each GPU routing its own 4096 tokens and exchanging rows with the
others over NVLink): weak scaling, per-GPU work fixed.  Expert weights are
seeded N(0, 0.02) packed to qmoe-rs's 2-bit format, the gate f32 N(0, 0.02),
activations bf16 N(0, 1).

A step is one forward of the layer over one batch.  The timed region replays
K steps (CUDA graphs of the forward) back to back between CUDA events, with a
barrier and a device synchronize on both sides, and takes the max over ranks.
Every step streams the layer's weights from HBM: 2.85 GB on one GPU, and at
least 0.4 GB per GPU at N = 8, all far above the 126 MB L2.

On one GPU the line also carries the decode-sized lines the metric's second
half asks for (HBM rooflines): the same V3 layer over 32 bf16 tokens, and
configs[1] (the DeepSeek-V2-Lite layer over 32 f32 tokens), plus configs[2]
(V2-Lite prefill, 2048 bf16 tokens) and the device packer.

Prints one JSON line (rank 0).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for p in (ROOT, os.path.join(ROOT, "qmoe-rs_b200", "python")):
    if p not in sys.path:
        sys.path.insert(0, p)

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "MoE-layer tokens/sec at 1/2/4/8 B200; decode HBM GB/s as % of peak"
UNIT = "tokens/s"
L2_BYTES = 126 * 2**20

V3 = dict(key="v3",
          name="configs[3]: DeepSeek-V3 MoE layer (hidden 7168, 256 experts, sigmoid 8 groups / "
               "top-4 groups / top-8, 1 shared expert, intermediate 2048), 4096 bf16 tokens per GPU, "
               "expert-parallel over the GPUs",
          E=256, k=8, H=7168, I=2048, Is=2048, T=4096, act="bf16", scoring=1, n_group=8,
          topk_group=4, norm_topk=True, routed_scale=2.5)
V2 = dict(key="v2lite",
          name="configs[1]: DeepSeek-V2-Lite MoE layer (hidden 2048, 64 experts, softmax top-6, "
               "2 shared experts, intermediate 1408), decode, 32 f32 tokens per GPU",
          E=64, k=6, H=2048, I=1408, Is=2816, T=32, act="f32", scoring=0, n_group=1,
          topk_group=1, norm_topk=True, routed_scale=1.0)
WORKLOADS = {"v3": V3, "v2lite": V2}

# kernels launched per forward (counted from the launch sequence in csrc/api.cu)
LAUNCHES = {
    # decode (<= 64 tokens, all experts local): front cluster (logits,
    # selection, permute); gate/up GEMV (x limbs first); down GEMV (h limbs
    # first, weighted combine last)
    "decode_front": 3,
    # decode batches the front cluster does not take (T * E > 4096): router
    # partials, their ordered sums, selection with the permute in its last
    # CTA, gate/up GEMV, down GEMV
    "decode_router": 5,
    # prefill: router partials or logits, selection, permute, bf16 gather,
    # gate/up GEMM, down GEMM, combine
    "prefill": 7,
    # expert-parallel rank, decode: front cluster (route + send list),
    # dispatch, permute (waits for the peers' rows), gate/up GEMV, down GEMV
    # (returns the partial sums to their ranks), finish
    "ep_decode": 6,
    # expert-parallel rank, prefill: router logits, selection, plan,
    # dispatch, permute (waits), gather, gate/up GEMM, down GEMM, combine,
    # return, finish
    "ep_prefill": 11,
}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="v3",
                    help="headline workload: v3 = configs[3] (default), v2lite = configs[1]")
    ap.add_argument("--ep-exchange", choices=["p2p", "nccl"], default="p2p",
                    help="N > 1: peer-memory kernels or NCCL all-to-alls for the EP exchanges")
    ap.add_argument("--seed", type=int, default=1234)
    ap.add_argument("--no-cpu-baseline", action="store_true",
                    help="skip the CPU-baseline leg (for profiler runs)")
    ap.add_argument("--no-sublines", action="store_true",
                    help="N = 1: only the headline workload")
    ap.add_argument("--ncu-case", choices=["decode", "prefill", "pack", "v3-prefill", "v3-decode",
                                           "v3-route", "v3"],
                    default=None,
                    help="only run 3 eager forwards of a short fixed case for an ncu capture, "
                         "print nothing")
    return ap.parse_args()


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def tensor_peaks():
    """(sustained, burst, kind) bf16 TFLOP/s.  The expert GEMMs are timed
    inside runs of back-to-back layer steps under the power cap, so their
    roofline denominator is the sustained cuBLAS figure; the burst figure is
    reported beside it."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        if "bf16_tflops_sustained" in d:
            return float(d["bf16_tflops_sustained"]), float(d["bf16_tflops"]), "measured sustained"
        return float(d["bf16_tflops"]), float(d["bf16_tflops"]), "measured burst"
    return 1400.0, 1590.0, "fallback sustained"


def read_profile_traffic(name: str, key: str = "traffic_bytes_per_launch"):
    """DRAM bytes per launch of a kernel from its committed ncu summary (a
    line '<key>: N'), or None."""
    path = os.path.join(ROOT, "profiles", name)
    if not os.path.exists(path):
        return None
    for line in open(path):
        if line.startswith(key + ":"):
            try:
                return float(line.split(":", 1)[1].strip())
            except ValueError:
                return None
    return None


# ---------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------

class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while running."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
        0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
    }

    def __init__(self, device_index: int, period_s: float = 0.005):
        self.period = period_s
        self.samples = []
        self.reasons = set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nv = None

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                for bit, name in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                break
            time.sleep(self.period)

    def __enter__(self):
        if self._nv is not None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._t is not None:
            self._t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [],
                    "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons - {"gpu_idle"}),
                "samples": len(self.samples)}


# ---------------------------------------------------------------------------
# workloads
# ---------------------------------------------------------------------------

def act_dtype(W, T=None):
    return torch.bfloat16 if W["act"] == "bf16" else torch.float32


def act_bytes(W):
    return 2 if W["act"] == "bf16" else 4


def rel_err(a, b) -> float:
    """max |a - b| / max |b| (the max-abs relative error of the parity bar)."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = max(float(np.max(np.abs(b))) if b.size else 0.0, 1e-30)
    return float(np.max(np.abs(a - b))) / den if a.size else 0.0


def make_cfg(W):
    from qmoe_b200 import MoEConfig
    return MoEConfig(W["E"], W["k"], W["H"], W["I"], shared_intermediate_dim=W["Is"],
                     scoring=W["scoring"], n_group=W["n_group"], topk_group=W["topk_group"],
                     norm_topk_prob=W["norm_topk"], routed_scaling_factor=W["routed_scale"])


def oracle_cfg(W):
    from oracle import oracle as qo
    return qo.MoEConfig(W["E"], W["k"], W["H"], W["I"], W["Is"], scoring=W["scoring"],
                        n_group=W["n_group"], topk_group=W["topk_group"],
                        norm_topk_prob=W["norm_topk"], routed_scaling_factor=W["routed_scale"])


def synth_weights(W, seed: int, device: str, experts=None, packer=None):
    """Seeded layer; each expert has its own generator (seed, expert id), so
    ranks that build disjoint expert ranges agree on every expert, and all
    ranks build the same gate and shared expert.  `packer` maps an f32
    [out, in] weight to (packed, scales); default: the package quantizer
    (the device packer for CUDA tensors)."""
    from qmoe_b200 import quantize as qz
    pack = packer or qz.quantize_weight

    def gen(s):
        return torch.Generator(device=device).manual_seed(s)

    def mat(g, o, i):
        return pack(torch.randn(o, i, generator=g, device=device) * 0.02)

    out = []
    for e in (range(W["E"]) if experts is None else experts):
        g = gen(seed * 1009 + 1 + e)
        out.append([mat(g, W["I"], W["H"]), mat(g, W["I"], W["H"]), mat(g, W["H"], W["I"])])
    g = gen(seed * 1009)
    shared = [mat(g, W["Is"], W["H"]), mat(g, W["Is"], W["H"]), mat(g, W["H"], W["Is"])]
    gate_w = torch.randn(W["E"], W["H"], generator=g, device=device) * 0.02
    return out, shared, gate_w


def torch_packer(w):
    """quantize.py's arithmetic in plain torch ops (for the reference arm's
    inputs, so that arm runs nothing of this package's CUDA library)."""
    from qmoe_b200 import quantize as qz
    s = qz.row_scales(w)
    return qz.pack_codes(qz.ternary_codes(w, s)), s


def synth_x(W, T, seed, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    return torch.randn(T, W["H"], generator=g, device=dev).to(act_dtype(W))


def zipf_targets(E: int, s: float = 1.1, hottest: float = 0.08):
    """Assignment shares following Zipf(s) by popularity rank, shifted
    (p_r ~ (r + q)^-s, the Zipf-Mandelbrot form) so the hottest expert takes
    `hottest` of all assignments -- a token can pick an expert only once, so
    a top-8 router caps any expert at 1/8 of the assignments, below the
    unshifted Zipf(1.1) head over 256 experts."""
    r = np.arange(1, E + 1, dtype=np.float64)
    lo, hi = 0.0, 1e4
    for _ in range(200):
        q = 0.5 * (lo + hi)
        p = (r + q) ** -s
        p /= p.sum()
        lo, hi = (q, hi) if p[0] > hottest else (lo, q)
    return p


def route_torch(W, logits, bias):
    """Selection of the layer's router (sigmoid, group-limited top-k) in
    torch ops, for calibrating the bias only (the product routes on the
    device, bit-exact with the oracle)."""
    E, K, G, TG = W["E"], W["k"], W["n_group"], W["topk_group"]
    choice = torch.sigmoid(logits) + bias
    gs = choice.view(-1, G, E // G).topk(2, dim=-1).values.sum(-1)
    keep = torch.zeros_like(gs, dtype=torch.bool).scatter_(1, gs.topk(TG, dim=-1).indices, True)
    masked = choice.masked_fill(~keep.repeat_interleave(E // G, dim=1), float("-inf"))
    return masked.topk(K, dim=-1).indices


def zipf_bias(W, gate_w, seed: int, tokens: int = 4096, iters: int = 400):
    """a seeded per-expert selection bias under which expert
    popularity follows the shifted Zipf(1.1) of zipf_targets over a seeded
    permutation of the experts (hottest ~8% of assignments).  Fitted on
    `tokens` seeded N(0, 1) tokens: start from a bias proportional to the log
    target, then damped multiplicative corrections of the measured shares.
    Under group-limited routing the head follows the target closely while
    the coldest experts starve.  Returns (bias [E] f32 on the gate's device,
    target shares in expert order)."""
    E = W["E"]
    dev = gate_w.device
    g = torch.Generator(device="cpu").manual_seed(seed)
    perm = torch.randperm(E, generator=g)
    target = torch.empty(E, dtype=torch.float64)
    target[perm] = torch.from_numpy(zipf_targets(E))
    target = target.to(dev)
    xg = torch.Generator(device=dev).manual_seed(seed + 1)
    x = torch.randn(tokens, W["H"], generator=xg, device=dev)
    logits = x @ gate_w.t()
    lp = torch.log(target).float()
    bias = 0.05 * (lp - lp.mean())
    for _ in range(iters):
        idx = route_torch(W, logits, bias)
        share = torch.bincount(idx.reshape(-1), minlength=E).double() / idx.numel()
        bias += (0.08 * torch.log((target + 1e-5) / (share + 1e-5))).float().clamp(-0.05, 0.05)
        bias -= bias.mean()
    return bias.float().contiguous(), target.cpu().numpy()


def per_expert_bytes(W):
    return 3 * W["H"] * W["I"] // 4 + 4 * (2 * W["I"] + W["H"])


def shared_bytes(W):
    return 3 * W["H"] * W["Is"] // 4 + 4 * (2 * W["Is"] + W["H"])


def layer_bytes(W, T, touched):
    """Algorithmic HBM bytes of one forward: packed rows and scales of every
    expert the batch touches, the shared expert's, the gate, x in, out."""
    return float(touched * per_expert_bytes(W) + shared_bytes(W) + 4 * W["E"] * W["H"]
                 + 2 * act_bytes(W) * T * W["H"])


def gate_up_bytes(W, T, touched):
    """The gate/up GEMV: packed gate+up rows and scales of the touched
    experts and the shared expert, the activations read, the f32 SwiGLU rows
    written."""
    pe = 2 * (W["I"] * W["H"] // 4) + 2 * 4 * W["I"]
    sh = 2 * (W["Is"] * W["H"] // 4) + 2 * 4 * W["Is"]
    return float(touched * pe + sh + act_bytes(W) * T * W["H"]
                 + 4 * (T * W["k"] * W["I"] + T * W["Is"]))


def down_bytes(W, T, touched):
    """The down GEMV (limbs of h first, weighted combine last): packed down
    rows and scales, the f32 SwiGLU rows read, the output written."""
    pe = W["H"] * W["I"] // 4 + 4 * W["H"]
    sh = W["H"] * W["Is"] // 4 + 4 * W["H"]
    return float(touched * pe + sh + 4 * (T * W["k"] * W["I"] + T * W["Is"])
                 + act_bytes(W) * T * W["H"])


def layer_flops(W, T):
    H, I, Is, K, E = W["H"], W["I"], W["Is"], W["k"], W["E"]
    gu = 2.0 * T * K * 2 * H * I + 2.0 * T * 2 * H * Is
    dn = 2.0 * T * K * H * I + 2.0 * T * H * Is
    return gu, dn, gu + dn + 2.0 * T * E * H


def headline_config(W, ws, args):
    """The `config` object of the JSON line (identical in both arms)."""
    return {"workload": W["name"], "T_per_gpu": W["T"], "E": W["E"], "top_k": W["k"],
            "hidden": W["H"], "intermediate": W["I"], "shared_intermediate": W["Is"],
            "scoring": "sigmoid" if W["scoring"] == 1 else "softmax",
            "n_group": W["n_group"], "topk_group": W["topk_group"],
            "norm_topk_prob": W["norm_topk"], "routed_scaling_factor": W["routed_scale"],
            "activations": W["act"], "parallelism": f"ep{ws}" if ws > 1 else "single",
            "experts_per_gpu": W["E"] // ws,
            "l2": "inputs larger than L2: every step streams the layer's packed weights "
                  "(> 126 MB per GPU) from HBM"}


# ---------------------------------------------------------------------------
# CPU baseline (oracle restatement of qmoe-rs's SIMD path)
# ---------------------------------------------------------------------------

def to_host_experts(experts, shared):
    ne = [[(p.cpu().numpy().reshape(-1), s.cpu().numpy()) for p, s in ex] for ex in experts]
    ns = [(p.cpu().numpy().reshape(-1), s.cpu().numpy()) for p, s in shared]
    return ne, ns


def time_cpu_oracle(W, ne, ns, gw, nthreads: int, tokens: int, min_seconds: float, seed: int):
    from oracle import oracle as qo
    cfg = oracle_cfg(W)
    x = np.random.default_rng(seed).standard_normal((tokens, W["H"])).astype(np.float32)
    if W["act"] == "bf16":     # the bf16 activations the GPU arm reads, upcast exactly
        x = torch.from_numpy(x).bfloat16().float().numpy()
    n = 0
    t0 = time.perf_counter()
    while True:
        qo.layer_forward(cfg, gw, ne, x, shared=ns, nthreads=nthreads)
        n += 1
        el = time.perf_counter() - t0
        if el >= min_seconds:
            break
    return n * tokens / el, n, el


# ---------------------------------------------------------------------------
# reference arm
# ---------------------------------------------------------------------------

def run_reference(args):
    """qmoe-rs's CPU path on this host: the oracle restatement (qmoe-rs is
    Rust and cannot be built here), all host threads, token-parallel, on a
    bounded sample of the headline workload's tokens per step."""
    ws, rank, _ = dist_env()
    if rank != 0:
        return
    W = WORKLOADS[args.workload]
    nthreads = os.cpu_count() or 1
    # inputs (not timed): the seeded layer packed by quantize.py's arithmetic
    # in plain torch (on a CUDA device when there is one, for speed)
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    experts, shared, gate_w = synth_weights(W, args.seed, dev, packer=torch_packer)
    ne, ns = to_host_experts(experts, shared)
    gw = gate_w.cpu().numpy()
    del experts, shared, gate_w
    if dev == "cuda":
        torch.cuda.empty_cache()
    from oracle import oracle as qo
    cfg = oracle_cfg(W)
    tokens = min(W["T"], max(nthreads, 8))
    x = np.random.default_rng(args.seed).standard_normal((tokens, W["H"])).astype(np.float32)
    if W["act"] == "bf16":
        x = torch.from_numpy(x).bfloat16().float().numpy()
    t0 = time.perf_counter()
    qo.layer_forward(cfg, gw, ne, x, shared=ns, nthreads=nthreads)
    per_step = time.perf_counter() - t0
    budget = 120.0
    steps, warm = args.steps, args.warmup
    if (steps + warm) * per_step > budget:
        warm = min(warm, 2)
        steps = max(3, int(budget / per_step) - warm)
    for _ in range(warm):
        qo.layer_forward(cfg, gw, ne, x, shared=ns, nthreads=nthreads)
    t0 = time.perf_counter()
    for _ in range(steps):
        qo.layer_forward(cfg, gw, ne, x, shared=ns, nthreads=nthreads)
    el = time.perf_counter() - t0
    value = steps * tokens / el
    sample = (f"{tokens} of the {W['T']} tokens per step ({nthreads} threads, token-parallel), "
              f"{steps} steps timed")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "steps_run": steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * el / steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": W["act"], "data": "synthetic",
        "config": headline_config(W, max(ws, args.gpus), args),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": nthreads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "note": "qmoe-rs (Rust nightly + candle) cannot be built here; timed its C "
                "restatement oracle/qmoe_oracle.c with the same per-token/per-expert loop "
                "and f32x4 lane structure (bf16 activations upcast exactly to f32, the "
                "reference's only input type)",
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# timing helpers (one GPU)
# ---------------------------------------------------------------------------

def graph_stage_times(layers, xs, stream, n_prof: int = 100):
    """Average per-stage device time (ms) of the forward from the layer's
    stage events.  Each profiled forward is queued behind a device-side
    sleep, so the whole forward is enqueued before the GPU reaches it and no
    host launch gap enters the numbers."""
    for L in layers:
        L.set_profiling(True)
    stage_ms = {}
    with torch.cuda.stream(stream):
        for i in range(n_prof):
            r = i % len(layers)
            torch.cuda._sleep(2_000_000)       # ~1 ms of device time
            layers[r].forward(xs[r])
            for k, v in layers[r].stage_times().items():
                stage_ms.setdefault(k, []).append(v)
    for L in layers:
        L.set_profiling(False)
    return {k: float(np.mean(v)) for k, v in stage_ms.items()}


def time_graphs(layers, xs, steps: int, warmup: int, clocks_dev=None):
    """Forwards of the replicas back to back in one CUDA graph (as
    consecutive MoE layers of a model would run), replayed; returns (ms per
    forward, clock summary or None, stream)."""
    reps = len(layers)
    T = xs[0].shape[0]
    for L in layers:
        L.reserve(T)
    stream = torch.cuda.Stream()
    graphs = []
    with torch.cuda.stream(stream):
        for L, x in zip(layers, xs):
            L.forward(x)
        torch.cuda.current_stream().synchronize()
        for L, x in zip(layers, xs):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                L.forward(x)
            graphs.append(g)
        chain = torch.cuda.CUDAGraph()
        with torch.cuda.graph(chain, stream=stream):
            for L, x in zip(layers, xs):
                L.forward(x)
    torch.cuda.synchronize()
    for i in range(max(3, warmup)):
        graphs[i % reps].replay()
    chain.replay()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    clk = ClockSampler(clocks_dev) if clocks_dev is not None else None
    if clk:
        clk.__enter__()
    e0.record()
    for _ in range(steps // reps):
        chain.replay()
    for i in range(steps % reps):
        graphs[i].replay()
    e1.record()
    torch.cuda.synchronize()
    if clk:
        clk.__exit__()
    ms = e0.elapsed_time(e1) / steps
    del graphs, chain
    return ms, (clk.summary() if clk else None), stream


def e2e_host(layer, x_dev, n: int):
    """Forward through the public API with page-locked host buffers: the
    host->device copy of x and the device->host result inside every call."""
    x_host = x_dev.cpu().pin_memory()
    out_host = torch.empty_like(x_host).pin_memory()
    for _ in range(3):
        layer.forward(x_host, out=out_host)
    torch.cuda.synchronize()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(n):
        layer.forward(x_host, out=out_host)
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / n


def touched_experts(layer, x):
    _, idx, _ = layer.forward(x, return_routing=True)
    return int(len(np.unique(idx.cpu().numpy())))


# ---------------------------------------------------------------------------
# sub-lines (one GPU)
# ---------------------------------------------------------------------------

def run_decode_line(W, layers, xs, steps: int):
    """A decode-sized batch on the one-GPU layer: HBM rooflines of the two
    expert GEMVs and of the whole forward."""
    T = xs[0].shape[0]
    touched = touched_experts(layers[0], xs[0])
    ms, _, stream = time_graphs(layers, xs, steps, 5)
    stages = graph_stage_times(layers, xs, stream, n_prof=40)
    hbm, _, peak_kind = load_peaks()
    gu_b, dn_b, ly_b = gate_up_bytes(W, T, touched), down_bytes(W, T, touched), layer_bytes(W, T, touched)
    gu_ms, dn_ms = stages.get("gate_up", float("nan")), stages.get("down", float("nan"))
    launches = LAUNCHES["decode_front"] if T * W["E"] <= 4096 and T <= 64 else LAUNCHES["decode_router"]
    traffic = read_profile_traffic("qgemv_decode_v3_t32.txt" if W is V3 else "qgemv_gate_up_decode_v2lite_t32.txt")
    return {
        "value": T / (ms / 1e3), "unit": UNIT, "ms_per_step": ms, "T": T, "dtype": W["act"],
        "touched_experts": touched,
        "roofline": {"bound": "hbm", "kernel": "decode GEMV gate/up + SwiGLU (x limbs first)",
                     "achieved": gu_b / (gu_ms / 1e3) / 1e9, "peak": hbm, "unit": "GB/s",
                     "frac": gu_b / (gu_ms / 1e3) / 1e9 / hbm, "peak_kind": peak_kind,
                     "traffic": traffic, "algorithmic_bytes": gu_b, "kernel_ms": gu_ms},
        "roofline_down": {"bound": "hbm", "kernel": "decode GEMV down (h limbs first, combine last)",
                          "achieved": dn_b / (dn_ms / 1e3) / 1e9, "peak": hbm, "unit": "GB/s",
                          "frac": dn_b / (dn_ms / 1e3) / 1e9 / hbm, "algorithmic_bytes": dn_b,
                          "kernel_ms": dn_ms},
        "layer": {"algorithmic_bytes": ly_b, "achieved_gbs": ly_b / (ms / 1e3) / 1e9,
                  "frac": ly_b / (ms / 1e3) / 1e9 / hbm},
        "stage_ms": stages, "gpu_launches_per_step": launches,
    }


def run_prefill_line(W, layers, xs, steps: int):
    """A prefill-sized bf16 batch: tensor rooflines of the two expert GEMMs
    and the whole forward."""
    T = xs[0].shape[0]
    ms, _, stream = time_graphs(layers, xs, steps, 3)
    stages = graph_stage_times(layers, xs, stream, n_prof=10)
    gu_f, dn_f, fl = layer_flops(W, T)
    bf16, burst, peak_kind = tensor_peaks()
    gu_tf = gu_f / (stages["gate_up"] / 1e3) / 1e12
    return {
        "value": T / (ms / 1e3), "unit": UNIT, "ms_per_step": ms, "T": T, "dtype": "bf16",
        "tflops": fl / (ms / 1e3) / 1e12, "frac_layer": fl / (ms / 1e3) / 1e12 / bf16,
        "algorithmic_flops": fl,
        "roofline": {"bound": "tensor", "kernel": "qgemm_prefill gate/up + SwiGLU",
                     "achieved": gu_tf, "peak": bf16, "unit": "TFLOP/s",
                     "frac": gu_tf / bf16, "peak_kind": peak_kind, "frac_of_burst": gu_tf / burst,
                     "kernel_ms": stages["gate_up"],
                     "down_tflops": dn_f / (stages["down"] / 1e3) / 1e12,
                     "down_frac": dn_f / (stages["down"] / 1e3) / 1e12 / bf16},
        "stage_ms": stages, "gpu_launches_per_step": LAUNCHES["prefill"],
    }


PACK_ROWS = 64 * 1408      # the V2-Lite layer's 64 stacked gate matrices: [64 x 1408, 2048] f32


def run_pack(seed: int, dev: str, steps: int = 10):
    """The device packer (quantize.py's format producer, csrc/pack.cu) over
    the V2-Lite layer's stacked gate weights, [64 x 1408, 2048] f32 = 738 MB
    (> L2), scales computed.  Algorithmic bytes: the f32 read, the packed
    bytes and the scales written."""
    from qmoe_b200 import quantize as qz
    H = V2["H"]
    g = torch.Generator(device=dev).manual_seed(seed + 313)
    wt = torch.randn(PACK_ROWS, H, generator=g, device=dev) * 0.02
    for _ in range(3):
        qz.device_quantize(wt)
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    a.record()
    for _ in range(steps):
        qz.device_quantize(wt)
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / steps
    nbytes = 4 * PACK_ROWS * H + PACK_ROWS * H // 4 + 4 * PACK_ROWS
    hbm, _, peak_kind = load_peaks()
    gbs = nbytes / (ms / 1e3) / 1e9
    del wt
    torch.cuda.empty_cache()
    return {"workload": "V2-Lite gate weights of 64 experts, [90112, 2048] f32 -> 2-bit + row scales",
            "ms": ms, "algorithmic_bytes": nbytes, "achieved_gbs": gbs, "peak_gbs": hbm,
            "frac": gbs / hbm, "peak_kind": peak_kind,
            "weights_per_s": PACK_ROWS * H / (ms / 1e3)}


def build_layers(W, seed, dev, ctx, reps):
    from qmoe_b200 import QMoELayer
    layers = []
    keep = None
    for r in range(reps):
        experts, shared, gate_w = synth_weights(W, seed + 1000 * r, dev)
        layers.append(QMoELayer(make_cfg(W), gate_w, experts, shared=shared, ctx=ctx))
        if r == 0:
            keep = (experts, shared, gate_w)
        del experts, shared, gate_w
    return layers, keep


def replicas_for(W, per_gpu_bytes):
    """Replicas needed so that consecutive forwards never find their weights in L2."""
    return max(1, -(-4 * L2_BYTES // per_gpu_bytes)) if per_gpu_bytes < 4 * L2_BYTES else 1


# ---------------------------------------------------------------------------
# our arm, one GPU
# ---------------------------------------------------------------------------

def run_single(args, W, dev, local):
    from qmoe_b200 import default_context
    ctx = default_context(local)
    T = W["T"]
    all_bytes = W["E"] * per_expert_bytes(W) + shared_bytes(W)
    reps = replicas_for(W, all_bytes)
    layers, keep = build_layers(W, args.seed, dev, ctx, reps)
    xs = [synth_x(W, T, args.seed + 7 * r, dev) for r in range(reps)]
    torch.cuda.synchronize()
    prefill = W["act"] == "bf16" and T * W["k"] // W["E"] >= 16
    touched = touched_experts(layers[0], xs[0])

    ms, clocks, stream = time_graphs(layers, xs, args.steps, args.warmup, clocks_dev=local)
    value = T / (ms / 1e3)
    stages = graph_stage_times(layers, xs, stream, n_prof=10 if prefill else 100)
    e2e_ms = e2e_host(layers[0], xs[0], max(10, min(args.steps, 100 if prefill else 500)))
    hbm, _, peak_kind = load_peaks()
    bf16, burst, tpeak_kind = tensor_peaks()
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": W["act"], "data": "synthetic",
        "config": headline_config(W, 1, args),
    }
    if prefill:
        gu_f, dn_f, fl = layer_flops(W, T)
        gu_tf = gu_f / (stages["gate_up"] / 1e3) / 1e12
        dn_tf = dn_f / (stages["down"] / 1e3) / 1e12
        line["roofline"] = {
            "bound": "tensor", "kernel": "qgemm_prefill gate/up + SwiGLU (tcgen05, 2-bit dequant "
                                         "in the pipeline)",
            "achieved": gu_tf, "peak": bf16, "unit": "TFLOP/s", "frac": gu_tf / bf16,
            "peak_kind": tpeak_kind, "peak_burst": burst, "frac_of_burst": gu_tf / burst,
            "traffic": read_profile_traffic("qgemm_prefill_gate_up_v3.txt", "traffic_bytes_per_launch_full_v3"),
            "traffic_note": "ncu DRAM bytes of a 32-expert, 512-token V3-shaped launch, scaled by the "
                            "items of the full launch (8704 / 1088)",
            "algorithmic_flops": gu_f, "kernel_ms": stages["gate_up"],
            "down_tflops": dn_tf, "down_frac": dn_tf / bf16, "down_frac_of_burst": dn_tf / burst}
        line["layer"] = {"algorithmic_flops": fl, "tflops": fl / (ms / 1e3) / 1e12,
                         "frac": fl / (ms / 1e3) / 1e12 / bf16, "stage_ms": stages,
                         "touched_experts": touched}
        launches = LAUNCHES["prefill"]
    else:
        gu_b = gate_up_bytes(W, T, touched)
        ach = gu_b / (stages["gate_up"] / 1e3) / 1e9
        line["roofline"] = {
            "bound": "hbm", "kernel": "decode GEMV gate/up + SwiGLU (x limbs first)",
            "achieved": ach, "peak": hbm, "unit": "GB/s", "frac": ach / hbm, "peak_kind": peak_kind,
            "traffic": read_profile_traffic("qgemv_gate_up_decode_v2lite_t32.txt"),
            "algorithmic_bytes": gu_b, "kernel_ms": stages["gate_up"]}
        lb = layer_bytes(W, T, touched)
        line["layer"] = {"algorithmic_bytes": lb, "achieved_gbs": lb / (ms / 1e3) / 1e9,
                         "frac": lb / (ms / 1e3) / 1e9 / hbm, "stage_ms": stages,
                         "touched_experts": touched}
        launches = LAUNCHES["decode_front"]
    ab = act_bytes(W) * T * W["H"]
    line["e2e"] = {"value": T / (e2e_ms / 1e3), "unit": UNIT, "h2d_bytes_per_step": ab,
                   "d2h_bytes_per_step": ab, "ms_per_step": e2e_ms,
                   "path": "QMoELayer.forward -> qmoe_layer_forward with page-locked host x and out"}
    line["gpu_launches"] = launches * args.steps
    line["clocks"] = clocks

    sub = {}
    if not args.no_sublines:
        if W is V3:
            # the V3 layer in decode: 32 bf16 tokens through the GEMV path
            xd = [synth_x(W, 32, args.seed + 11, dev)]
            sub["decode_v3"] = dict(workload="configs[3] layer, decode, 32 bf16 tokens",
                                    **run_decode_line(W, layers[:1], xd, 200))
        del layers, xs
        torch.cuda.empty_cache()
        v2_layers, _ = build_layers(V2, args.seed, dev, ctx, 4)
        xs2 = [synth_x(V2, 32, args.seed + 7 * r, dev) for r in range(4)]
        sub["decode_v2lite"] = dict(workload=V2["name"], **run_decode_line(V2, v2_layers, xs2, 1000))
        xp = [synth_x(dict(V2, act="bf16"), 2048, args.seed + 99 + r, dev) for r in range(4)]
        sub["prefill_v2lite"] = dict(workload="configs[2]: the V2-Lite layer, prefill, 2048 bf16 "
                                              "tokens", **run_prefill_line(V2, v2_layers, xp, 20))
        del v2_layers, xs2, xp
        torch.cuda.empty_cache()
        sub["pack"] = run_pack(args.seed, dev)
    line.update(sub)

    if not args.no_cpu_baseline:
        experts, shared, gate_w = keep
        ne, ns = to_host_experts(experts, shared)
        gw = gate_w.cpu().numpy()
        ntok = 8 if W is V3 else W["T"]
        v, n, el = time_cpu_oracle(W, ne, ns, gw, 1, ntok, 10.0, args.seed)
        line["cpu_baseline"] = {
            "value": v, "unit": UNIT, "cores": 1, "kind": "port",
            "sample": f"{n} x {ntok} tokens of the {W['T']}-token batch on 1 thread, {el:.1f} s "
                      "(C restatement of qmoe-rs's f32x4 SIMD path)"}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# our arm, N GPUs (expert parallel)
# ---------------------------------------------------------------------------

def ep_measure(args, W, T, ws, rank, local, dev, dist, bias=None, steps=None):
    """One expert-parallel workload on N GPUs: each rank holds E/N experts, a
    gate and shared-expert replica and its own T tokens; dispatch and return
    by stores into the peers' memory (--ep-exchange p2p) or NCCL all-to-all.
    Returns (ms per step (max over ranks), parity, stage times of rank 0,
    load and exchange figures, e2e ms, clocks) -- the same on every rank."""
    from qmoe_b200 import ExpertParallelMoE, QMoELayer, default_context
    steps = steps or args.steps
    cfg = make_cfg(W)
    epr = W["E"] // ws
    mine = range(rank * epr, (rank + 1) * epr)
    per_rank_bytes = epr * per_expert_bytes(W) + shared_bytes(W)
    reps = replicas_for(W, per_rank_bytes)
    ctx = default_context(local)
    dt = act_dtype(W)
    layers = []
    for r in range(reps):
        experts, shared, gate_w = synth_weights(W, args.seed + 1000 * r, dev, experts=mine)
        layers.append(ExpertParallelMoE(cfg, gate_w, experts, rank, ws, shared=shared, ctx=ctx,
                                        capacity=T, exchange=args.ep_exchange, dtype=dt, bias=bias))
        del experts, shared, gate_w
    xs = [synth_x(W, T, args.seed + 31 * rank + 7 * r, dev) for r in range(reps)]
    torch.cuda.synchronize()
    dist.barrier()

    # parity: the first eager forward of replica 0 against the whole layer on
    # this GPU (same seeded weights, this rank's tokens)
    out_ep, idx_ep, _ = layers[0].forward(xs[0], return_routing=True)
    experts, shared, gate_w = synth_weights(W, args.seed, dev)
    full = QMoELayer(cfg, gate_w, experts, shared=shared, ctx=ctx, bias=bias)
    del experts, shared
    out_1, idx_1, _ = full.forward(xs[0], return_routing=True)
    torch.cuda.synchronize()
    err = rel_err(out_ep.float().cpu().numpy(), out_1.float().cpu().numpy())
    same_idx = bool(torch.equal(idx_ep, idx_1))
    # routed assignments of this rank's tokens per owning rank
    owner = torch.bincount((idx_1.reshape(-1).long() // epr), minlength=ws).double()
    per_expert = torch.bincount(idx_1.reshape(-1).long(), minlength=W["E"]).double()
    full.close()
    del full, out_1, idx_1, gate_w
    torch.cuda.empty_cache()
    tol = 2e-2 if W["act"] == "bf16" else 1e-4
    pr = torch.tensor([err, 0.0 if same_idx else 1.0], device=dev, dtype=torch.float64)
    dist.all_reduce(pr, op=dist.ReduceOp.MAX)
    parity = {"ok": bool(pr[0].item() <= tol and pr[1].item() == 0.0), "max_rel_err": float(pr[0].item()),
              "tolerance": tol, "routing_bit_exact": bool(pr[1].item() == 0.0),
              "against": "the whole layer on one GPU, each rank's own tokens (first eager forward)"}
    # the exchange's waits are bounded (about a second): start the next
    # forwards together, not after each rank's own set-up time
    torch.cuda.synchronize()
    dist.barrier()

    for i in range(max(3, args.warmup)):
        layers[i % reps].forward(xs[i % reps])
    torch.cuda.synchronize()
    dist.barrier()
    # the replicas' forwards back to back in one CUDA graph (exchanges
    # included: the peer-memory kernels, or NCCL captured with the kernels)
    stream = torch.cuda.Stream()
    graphs = []
    with torch.cuda.stream(stream):
        for r in range(reps):
            layers[r].forward(xs[r])
        torch.cuda.current_stream().synchronize()
        for r in range(reps):
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=stream):
                layers[r].forward(xs[r])
            graphs.append(gr)
        chain = torch.cuda.CUDAGraph()
        with torch.cuda.graph(chain, stream=stream):
            for r in range(reps):
                layers[r].forward(xs[r])
    torch.cuda.synchronize()
    dist.barrier()
    for i in range(max(3, args.warmup)):
        graphs[i % reps].replay()
    chain.replay()
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    align = torch.zeros(1, device=dev)
    with ClockSampler(local) as clk:
        # the start event follows a collective on the device, so every rank's
        # clock starts when the last rank arrives (host launch skew between
        # the ranks is not counted as exchange waiting)
        dist.all_reduce(align)
        e0.record()
        for _ in range(steps // reps):
            chain.replay()
        for i in range(steps % reps):
            graphs[i].replay()
        e1.record()
        torch.cuda.synchronize()
    dist.barrier()
    ctx.synchronize()        # raises if any exchange wait of the timed forwards gave up
    t = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item()) / steps
    for gr in graphs:
        del gr
    graphs.clear()
    del chain
    torch.cuda.synchronize()
    dist.barrier()

    # per-stage device times of this rank's forward (all ranks in step)
    layers[0].layer.set_profiling(True)
    st = {}
    with torch.cuda.stream(stream):
        for i in range(10):
            dist.barrier()
            layers[0].forward(xs[0])
            for k, v in layers[0].layer.stage_times().items():
                st.setdefault(k, []).append(v)
    layers[0].layer.set_profiling(False)
    st = {k: float(np.mean(v)) for k, v in st.items()}
    names = {"router": "route_plan_dispatch", "permute": "wait_dispatch_permute", "quant_up": "gather_or_limbs"}
    stages = {names.get(k, k): v for k, v in st.items()}
    torch.cuda.synchronize()
    dist.barrier()

    # rows this rank sent to the others (dispatch) and got back (return)
    counts = layers[0]._bufs["plan"]["counts"].cpu().long()
    sent_rows = int(counts.sum().item() - counts[rank].item())
    row_bytes = act_bytes(W) * W["H"]

    # end to end: pinned host tokens in, host result out, every step
    x_host = xs[0].cpu().pin_memory()
    out_host = torch.empty_like(x_host).pin_memory()
    n_e2e = max(10, min(steps, 50 if W["act"] == "bf16" else 200))
    for i in range(3):
        out_host.copy_(layers[0].forward(x_host.to(dev, non_blocking=True)), non_blocking=True)
    torch.cuda.synchronize()
    dist.barrier()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    dist.all_reduce(align)
    a.record()
    for i in range(n_e2e):
        out_host.copy_(layers[0].forward(x_host.to(dev, non_blocking=True)), non_blocking=True)
    b.record()
    torch.cuda.synchronize()
    t = torch.tensor([a.elapsed_time(b) / n_e2e], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_ms = float(t.item())

    # load: routed assignments landing on each rank (all ranks' tokens)
    owner = owner.to(dev)
    dist.all_reduce(owner)
    per_rank = [float(v) for v in owner.cpu().tolist()]
    per_expert = per_expert.to(dev)
    dist.all_reduce(per_expert)
    hottest = float(per_expert.max().item() / max(1.0, per_expert.sum().item()))
    sr = torch.tensor([float(sent_rows)], device=dev, dtype=torch.float64)
    allsr = [torch.zeros_like(sr) for _ in range(ws)]
    dist.all_gather(allsr, sr)
    sent = [float(v.item()) for v in allsr]
    load = {"routed_assignments_per_rank": per_rank,
            "imbalance_max_over_mean": max(per_rank) / max(1e-9, float(np.mean(per_rank))),
            "hottest_expert_share": hottest,
            "dispatch_rows_sent_per_rank": sent,
            "exchange_bytes_per_rank_max": 2 * row_bytes * max(sent),
            "exchange_bytes_note": "rows sent to other GPUs x row bytes, dispatch plus the same rows' "
                                   "partial sums returned (activation dtype); unused padded rows cross nothing"}
    torch.cuda.synchronize()
    dist.barrier()
    for L in layers:          # every rank is done with the others' buffers
        L.close()
    del layers, xs
    torch.cuda.empty_cache()
    dist.barrier()
    return ms_max, parity, stages, load, e2e_ms, clk.summary(), reps


def run_ep(args, W, ws, rank, local, dev, dist):
    """N > 1: the headline workload expert-parallel over the N GPUs (weak
    scaling: tokens per GPU fixed), then configs[4] (the V3 layer under a
    Zipf(1.1) expert popularity, 16384 tokens over the N GPUs)."""
    T = W["T"]
    ms, parity, stages, load, e2e_ms, clocks, reps = ep_measure(args, W, T, ws, rank, local, dev, dist)
    value = ws * T / (ms / 1e3)
    zipf = None
    if W is V3 and not args.no_sublines:
        Tz = 16384 // ws
        _, _, gate_w = synth_weights(dict(W, E=W["E"]), args.seed, dev, experts=[])
        bias, target = zipf_bias(W, gate_w, args.seed + 4)
        dist.broadcast(bias, 0)
        del gate_w
        zs = max(10, min(args.steps, 100))
        zms, zpar, zst, zload, ze2e, _, _ = ep_measure(args, W, Tz, ws, rank, local, dev, dist, bias=bias,
                                                        steps=zs)
        zipf = {"workload": "configs[4]: the configs[3] layer, 16384 bf16 tokens over the GPUs, per-expert "
                            "selection bias giving a shifted Zipf(1.1) popularity (hottest ~8% of "
                            "assignments) over a seeded expert permutation",
                "value": 16384 / (zms / 1e3), "unit": UNIT, "ms_per_step": zms, "T_per_gpu": Tz,
                "steps": zs, "parity": zpar, "stage_ms_rank0": zst, "load": zload,
                "target_hottest_share": float(np.max(target)),
                "e2e_ms_per_step": ze2e}
    dec = None
    if W is V3 and not args.no_sublines:
        # configs[1] in decode, expert parallel: 32 f32 tokens per GPU
        ds = max(50, min(10 * args.steps, 500))
        dms, dpar, dst, dload, de2e, _, _ = ep_measure(args, V2, 32, ws, rank, local, dev, dist, steps=ds)
        dec = {"workload": "configs[1] layer (V2-Lite), decode, 32 f32 tokens per GPU, expert parallel "
                           "(weak scaling)",
               "value": ws * 32 / (dms / 1e3), "unit": UNIT, "ms_per_step": dms, "steps": ds,
               "parity": dpar, "stage_ms_rank0": dst, "load": dload, "e2e_ms_per_step": de2e}
    if rank == 0:
        prefill = W["act"] == "bf16" and T * W["k"] // W["E"] >= 16
        gu_f, dn_f, fl = layer_flops(W, T)
        bf16, burst, peak_kind = tensor_peaks()
        roof = None
        if prefill and stages.get("gate_up"):
            gu_tf = gu_f / (stages["gate_up"] / 1e3) / 1e12
            roof = {"bound": "tensor", "kernel": "qgemm_prefill gate/up + SwiGLU (rank 0)",
                    "achieved": gu_tf, "peak": bf16, "unit": "TFLOP/s", "frac": gu_tf / bf16,
                    "peak_kind": peak_kind, "frac_of_burst": gu_tf / burst, "traffic": None, "kernel_ms": stages["gate_up"],
                    "note": "flops of one GPU's worth of tokens (the weak-scaling share of the "
                            "routed work and this rank's shared-expert rows)"}
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": W["act"], "data": "synthetic",
            "config": headline_config(W, ws, args),
            "exchange": ("peer-memory stores into the other GPUs' IPC-mapped buffers (NVLink), "
                         "arrival flags" if args.ep_exchange == "p2p" else "NCCL all_to_all_single")
                        + ", fixed-capacity rows",
            "replicas": reps,
            "roofline": roof,
            "parity": parity,
            "stage_ms_rank0": stages,
            "load": load,
            "e2e": {"value": ws * T / (e2e_ms / 1e3), "unit": UNIT,
                    "h2d_bytes_per_step": act_bytes(W) * T * W["H"] * ws,
                    "d2h_bytes_per_step": act_bytes(W) * T * W["H"] * ws, "ms_per_step": e2e_ms},
            "gpu_launches": (LAUNCHES["ep_prefill"] if prefill else LAUNCHES["ep_decode"]) * args.steps,
            "clocks": clocks,
        }
        if zipf is not None:
            line["zipf"] = zipf
        if dec is not None:
            line["decode_v2lite_ep"] = dec
        print(json.dumps(line), flush=True)
    dist.barrier()
    dist.destroy_process_group()


def run_ours(args):
    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = f"cuda:{local}"
    W = WORKLOADS[args.workload]
    if ws > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device(dev))
        return run_ep(args, W, ws, rank, local, dev, dist)
    return run_single(args, W, dev, local)


def run_ncu_case(args):
    """A short fixed workload for ncu captures (one layer, 3 forwards)."""
    from qmoe_b200 import QMoELayer, default_context
    torch.cuda.set_device(0)
    if args.ncu_case == "pack":
        # 16 experts' stacked gate weights: 184 MB (> L2), three packs and
        # no other launch of the packer before them
        from qmoe_b200 import quantize as qz
        g = torch.Generator(device="cuda").manual_seed(args.seed + 313)
        wt = torch.randn(16 * 1408, V2["H"], generator=g, device="cuda") * 0.02
        for _ in range(3):
            qz.device_quantize(wt)
        torch.cuda.synchronize()
        return
    if args.ncu_case.startswith("v3"):
        # v3-prefill: 32 experts of the V3 shape (353 MB of packed weights)
        # and 512 bf16 tokens, i.e. ~128 tokens per expert as in configs[3];
        # v3-decode: the whole V3 layer (2.85 GB) over 32 bf16 tokens
        # v3: the whole configs[3] forward (4096 tokens), for the launch list
        W = dict(V3, E=32, n_group=8, topk_group=4) if args.ncu_case == "v3-prefill" else V3
        T = {"v3-prefill": 512, "v3": 4096}.get(args.ncu_case, 32)
    else:
        W, T = V2, (32 if args.ncu_case == "decode" else 2048)
        if args.ncu_case == "prefill":
            W = dict(V2, act="bf16")
    if args.ncu_case == "v3-route":
        T = 4096                 # the router alone over the configs[3] batch
    experts, shared, gate_w = synth_weights(W, args.seed, "cuda")
    layer = QMoELayer(make_cfg(W), gate_w, experts, shared=shared, ctx=default_context(0))
    del experts, shared
    x = synth_x(W, T, args.seed + 7, "cuda")
    for _ in range(3):
        if args.ncu_case == "v3-route":
            layer.route(x)
        else:
            layer.forward(x)
    torch.cuda.synchronize()


def main():
    args = parse()
    if args.ncu_case:
        run_ncu_case(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
