"""Benchmark: fused geo-biased station attention, forward + backward, on 1..8 B200 (one process per GPU).

Workload (the scaling configuration): 256 issue dates sharded over the ranks, 16 heads, 512 stations,
head dim 128, bf16; per-head alpha/beta/gamma; geo prior from synthetic station coordinates
(lat ~ U(35,49), lon ~ U(-124,-104), elevation ~ U(500,3500) m). One step = forward + backward of the attention
on this rank's issue dates followed by an NCCL all-reduce of the bias-parameter gradients (N > 1).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload c5|c4|configs]

Prints ONE JSON line on rank 0. ``value`` is whole-job algorithmic TFLOP/s, 12*B*H*N^2*D per fwd+bwd (recompute not
counted), over the max-over-ranks device time of K steps (replays of the step captured as one CUDA graph, so host-side
launch work does not pace the GPU at small shards). ``e2e`` is the same metric through the public API with
the step's inputs copied from pinned host memory and the bias gradients read back, every step. ``roofline``
describes the dominant kernel timed live with CUDA events on its launching stream. ``--impl reference`` times the
reference's operator on the host CPU cores (the oracle's restatement of the eager PyTorch op, all threads) on a
bounded sample of the same workload.
"""
import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

import numpy as np
import torch

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "geo-attn fwd+bwd TFLOPS & % tensor peak at 1/2/4/8 B200 vs eager; ms/step"
UNIT = "TFLOP/s"
B_TOTAL, H, N, D = 256, 16, 512, 128
E2E_SLICES = 8   # issue-date slices of the end-to-end step (host copies of one overlap compute of the previous)


def flops(b):
    return 12.0 * b * H * N * N * D


T_START = time.time()


def phase(msg):
    """One progress line per phase on stderr (rank-tagged), so a run that stops can be located from its log."""
    print("[bench rank %s %.1fs] %s" % (os.environ.get("RANK", "0"), time.time() - T_START, msg), file=sys.stderr,
          flush=True)


def config(world):
    return {"workload": "geo-attn fwd+bwd, %d issue dates sharded over %d GPU(s), H=%d heads, N=%d stations, "
                        "D=%d, bf16, per-head alpha/beta/gamma, prior from station coordinates" % (B_TOTAL, world, H, N, D),
            "global_batch": B_TOTAL, "per_gpu_batch": B_TOTAL // world, "heads": H, "stations": N, "head_dim": D,
            "parallelism": "dp%d over issue dates; NCCL all-reduce of d(alpha,beta,gamma)" % world,
            "l2": "inputs larger than L2: q,k,v,dO = %.0f MB per rank vs 126 MB L2" % (4 * B_TOTAL // world * H * N * D * 2 / 1e6)}


def stations(seed=0):
    rng = np.random.default_rng(seed)
    lat = rng.uniform(35.0, 49.0, N)
    lon = rng.uniform(-124.0, -104.0, N)
    elev_ft = rng.uniform(500.0, 3500.0, N) / 0.3048
    return lat, lon, elev_ft


def inputs(b, seed, device):
    g = torch.Generator().manual_seed(seed)
    s = D ** -0.25
    q, k, v = (torch.randn(b, H, N, D, generator=g) * s for _ in range(3))
    do = torch.randn(b, H, N, D, generator=g)
    gp = torch.Generator().manual_seed(7)
    a = torch.rand(H, generator=gp) * 0.9 + 0.1
    bb = torch.randn(H, generator=gp) * 0.5
    c = torch.randn(H, generator=gp) * 0.5
    t = [x.to(torch.bfloat16) for x in (q, k, v, do)]
    return t, [x.to(device) for x in (a, bb, c)]


def peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            m = json.load(f)
        return m.get("bf16_tflops_sustained", 1381.7), "measured (MEASURED_PEAKS.json bf16_tflops_sustained)"
    return 1400.0, "fallback (sustained bf16 1.4 PFLOP/s)"


def traffic_per_launch(kernel):
    """DRAM bytes per launch of `kernel` for this workload from the committed ncu summary, else None."""
    p = os.path.join(REPO, "profiles", "traffic_c5_bf16_d128.txt")
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.startswith(kernel + " "):
            try:
                return float(line.split()[1])
            except (IndexError, ValueError):
                return None
    return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 50 ms around the timed region (under the same load)."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus):
        self.gpus = set(gpus)
        self.proc = None
        self.path = os.path.join("/tmp", "geoattn_clocks_%d.csv" % os.getpid())

    def start(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "--query-gpu=" + self.Q, "--format=csv,noheader,nounits",
                                          "-lms", "50"], stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        self.proc.wait()
        self.f.close()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9 or not f[0].isdigit() or int(f[0]) not in self.gpus:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(n)
        os.unlink(self.path)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons), "samples": len(sm)}


def cpu_reference(seconds, threads):
    """The reference operator on the host CPU (the oracle's restatement of the eager PyTorch op, fp32), fwd+bwd on
    one issue date (H heads x N stations x D) repeated for about `seconds`; returns TFLOP/s and the sample."""
    from oracle import geo_attention as oga
    from oracle import geometry as ogeo
    torch.set_num_threads(threads)
    lat, lon, el = stations(0)
    dist, ang = (torch.from_numpy(x).float() for x in ogeo.distance_and_angularity(lat, lon, el))
    (q, k, v, do), (a, b, c) = inputs(1, 1000, "cpu")
    q, k, v, do = (t.float() for t in (q, k, v, do))
    oga.grads(q, k, v, dist, ang, a, b, c, do, dtype=torch.float32)  # warm-up
    reps, t0 = 0, time.perf_counter()
    while True:
        oga.grads(q, k, v, dist, ang, a, b, c, do, dtype=torch.float32)
        reps += 1
        el_s = time.perf_counter() - t0
        if el_s >= seconds or reps >= 5000:
            break
    return flops(1) * reps / el_s / 1e12, reps, el_s


def peak_extra_memory(fn, dev):
    """Peak device memory one fwd+bwd allocates beyond what is live before it (inputs, dO, parameters), as the
    reference reports for its operators: MiB, from the caching allocator's peak counter."""
    torch.cuda.synchronize(dev)
    base = torch.cuda.memory_allocated(dev)
    torch.cuda.reset_peak_memory_stats(dev)
    fn()
    torch.cuda.synchronize(dev)
    peak = torch.cuda.max_memory_allocated(dev)
    return {"peak_extra_mib": (peak - base) / 2 ** 20,
            "what": "peak allocated during one fwd+bwd minus the memory live before it (q, k, v, dO, parameters, "
                    "prior); outputs, gradients, row statistics and the backward workspace (with the bf16 dS scratch) "
                    "included"}


def gpu_eager_ms(q, k, v, do, dist, ang, a, b, c, steps):
    """Eager PyTorch on the same GPU and inputs (bf16 storage; the reference's op written with torch ops)."""
    def op(q, k, v):
        s = torch.matmul(q, k.transpose(-2, -1)) / math.sqrt(D)
        p1 = torch.softmax(s, dim=-1)
        z = a.view(1, -1, 1, 1) * p1 + b.view(1, -1, 1, 1) * (1 / (1 + dist)) + c.view(1, -1, 1, 1) * (1 / (1 + ang))
        return torch.matmul(torch.softmax(z, dim=-1).to(v.dtype), v)
    x = [t.detach().requires_grad_(True) for t in (q, k, v)]
    try:
        for _ in range(2):
            op(*x).backward(do)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            for t in x:
                t.grad = None
            op(*x).backward(do)
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps
    except torch.OutOfMemoryError:
        return None
    finally:
        del x
        torch.cuda.empty_cache()


REF_SAMPLE_DATES = 32   # issue dates per step of the reference arm: a bounded sample (1/8) of the 256-date workload


def cpu_step_sample(n_dates, threads):
    """One step of the reference arm: fwd+bwd of the eager operator (the oracle's restatement of the reference's eager
    PyTorch op, fp32, on the host CPU) over `n_dates` issue dates of the workload, one issue date per call as the
    reference's training loop batches them. Returns the wall time in ms."""
    from oracle import geo_attention as oga
    from oracle import geometry as ogeo
    torch.set_num_threads(threads)
    lat, lon, el = stations(0)
    dist, ang = (torch.from_numpy(x).float() for x in ogeo.distance_and_angularity(lat, lon, el))
    (q, k, v, do), (a, b, c) = inputs(1, 1000, "cpu")
    q, k, v, do = (t.float() for t in (q, k, v, do))
    t0 = time.perf_counter()
    for _ in range(n_dates):
        oga.grads(q, k, v, dist, ang, a, b, c, do, dtype=torch.float32)
    return (time.perf_counter() - t0) * 1e3


def cpu_c2_extrapolated(threads, reps=5):
    """The TF32 configuration's shape (H=8, N=512, D=64, fp32) on the host CPU at B = 1..4 issue dates (median ms of
    `reps` fwd+bwd each), and the least-squares line through them evaluated at its B = 32."""
    from oracle import geo_attention as oga
    from oracle import geometry as ogeo
    torch.set_num_threads(threads)
    h1, n1, d1 = 8, 512, 64
    rng = np.random.default_rng(0)
    lat, lon = rng.uniform(35.0, 49.0, n1), rng.uniform(-124.0, -104.0, n1)
    el = rng.uniform(500.0, 3500.0, n1) / 0.3048
    dist, ang = (torch.from_numpy(x).float() for x in ogeo.distance_and_angularity(lat, lon, el))
    g = torch.Generator().manual_seed(0)
    a = torch.rand(h1, generator=g) * 0.9 + 0.1
    b, c = torch.randn(h1, generator=g) * 0.5, torch.randn(h1, generator=g) * 0.5
    ms = {}
    for bb in (1, 2, 3, 4):
        q, k, v, do = (torch.randn(bb, h1, n1, d1, generator=g) * (d1 ** -0.25 if i < 3 else 1.0) for i in range(4))
        oga.grads(q, k, v, dist, ang, a, b, c, do, dtype=torch.float32)
        ts = []
        for _ in range(reps):
            t0 = time.perf_counter()
            oga.grads(q, k, v, dist, ang, a, b, c, do, dtype=torch.float32)
            ts.append((time.perf_counter() - t0) * 1e3)
        ms[bb] = statistics.median(ts)
    xs, ys = np.array(list(ms)), np.array(list(ms.values()))
    slope, icpt = np.polyfit(xs, ys, 1)
    return {"ms_fwd_bwd_by_issue_dates": ms, "ms_fwd_bwd_extrapolated_b32": float(slope * 32 + icpt),
            "cores": threads, "shape_hnd": [h1, n1, d1], "dtype": "fp32",
            "what": "eager FP32 fwd+bwd on the host CPU at B = 1..4, least-squares line evaluated at B = 32"}


def cpu_c1(threads, reps=10):
    """The CPU configuration: eager FP32 fwd+bwd at B=1 issue date, H=8, N=512, D=64 (q, k, v ~ N(0,1) D^-1/4 from
    seed 0; coordinates lat ~ U(35,49), lon ~ U(-124,-104), elevation ~ U(500,3500) m; a_h ~ U(0.1,1),
    b_h, g_h ~ N(0, 0.5)); median ms of `reps` calls after one warm-up."""
    from oracle import geo_attention as oga
    from oracle import geometry as ogeo
    torch.set_num_threads(threads)
    b1, h1, n1, d1 = 1, 8, 512, 64
    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn(b1, h1, n1, d1, generator=g) * d1 ** -0.25 for _ in range(3))
    rng = np.random.default_rng(0)
    lat, lon = rng.uniform(35.0, 49.0, n1), rng.uniform(-124.0, -104.0, n1)
    el = rng.uniform(500.0, 3500.0, n1) / 0.3048
    dist, ang = (torch.from_numpy(x).float() for x in ogeo.distance_and_angularity(lat, lon, el))
    a = torch.rand(h1, generator=g) * 0.9 + 0.1
    b, c = torch.randn(h1, generator=g) * 0.5, torch.randn(h1, generator=g) * 0.5
    do = torch.randn(b1, h1, n1, d1, generator=g)
    oga.grads(q, k, v, dist, ang, a, b, c, do, dtype=torch.float32)
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        oga.grads(q, k, v, dist, ang, a, b, c, do, dtype=torch.float32)
        ts.append((time.perf_counter() - t0) * 1e3)
    fl = 12.0 * b1 * h1 * n1 * n1 * d1
    ms = statistics.median(ts)
    return {"ms_fwd_bwd": ms, "gflop": fl / 1e9, "tflops": fl / (ms * 1e-3) / 1e12, "cores": threads, "reps": reps,
            "shape_bhnd": [b1, h1, n1, d1], "dtype": "fp32",
            "what": "eager FP32 fwd+bwd of the reference operator on the host CPU (oracle's torch restatement)"}


def run_reference(args):
    """The reference arm: the reference's eager operator on the host CPU cores, all threads. Each of the K timed steps
    is a bounded sample of the workload -- REF_SAMPLE_DATES issue dates fwd+bwd, timed for real -- so ms_per_step is
    the measured time of that sample step and value the measured rate."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    for _ in range(args.warmup):
        cpu_step_sample(1, threads)
    ts = [cpu_step_sample(REF_SAMPLE_DATES, threads) for _ in range(args.steps)]
    ms = statistics.mean(ts)
    value = flops(REF_SAMPLE_DATES) / (ms * 1e-3) / 1e12
    sample = ("each step: fwd+bwd of %d of the %d issue dates (H=%d, N=%d, D=%d), fp32 eager on the CPU, one date per "
              "call; %d steps, %.1f s timed" % (REF_SAMPLE_DATES, B_TOTAL, H, N, D, args.steps, sum(ts) / 1e3))
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "step_is": "a bounded sample: %d issue dates of the %d-date workload" % (REF_SAMPLE_DATES, B_TOTAL),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
            "config": config(world),
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "c1_cpu": cpu_c1(threads), "c2_cpu": cpu_c2_extrapolated(threads)}
    print(json.dumps(line), flush=True)
    return 0


def run_c4(args):
    """Full training step of a random-init geo-attention encoder (12 pre-LN layers, d_model 2048, 16 x 128 heads,
    FFN 8192) on 24 weekly timesteps x 512 stations of one issue date, bf16 autocast, MSE loss, fused AdamW; every
    layer's spatial attention is the geo-attention kernel. Prints one JSON line (ms per training step)."""
    import torch.nn as nn
    import foreswe_gpu_optimization_b200 as g

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    torch.manual_seed(0)
    layers, dm, heads, dh, dff, weeks, feats = 12, 2048, 16, 128, 8192, 24, 15
    geom = g.StationGeometry(*stations(0), device=dev)
    dmat, amat = geom.distance_and_angularity()
    eager = [False]

    class Layer(nn.Module):
        def __init__(self):
            super().__init__()
            self.n1, self.n2 = nn.LayerNorm(dm), nn.LayerNorm(dm)
            self.W_q, self.W_k, self.W_v, self.W_o = (nn.Linear(dm, dm) for _ in range(4))
            self.fc1, self.fc2 = nn.Linear(dm, dff), nn.Linear(dff, dm)
            self.alpha = nn.Parameter(torch.rand(heads) * 0.9 + 0.1)
            self.beta = nn.Parameter(torch.randn(heads) * 0.5)
            self.gamma = nn.Parameter(torch.randn(heads) * 0.5)

        def forward(self, x):                      # x [weeks, stations, d_model]
            h = self.n1(x)
            q, k, v = (w(h).view(weeks, N, heads, dh).transpose(1, 2) for w in (self.W_q, self.W_k, self.W_v))
            if eager[0]:                           # the production method (custom_encoder_model.py:25-39)
                s_ = torch.softmax(torch.matmul(q, k.transpose(-2, -1)) / math.sqrt(dh), dim=-1)
                z = (self.alpha.view(-1, 1, 1) * s_ + self.beta.view(-1, 1, 1) / (1 + dmat)
                     + self.gamma.view(-1, 1, 1) / (1 + amat))
                a = torch.matmul(torch.softmax(z, dim=-1), v)
            else:
                a = g.geo_attention(q, k, v, geom, self.alpha, self.beta, self.gamma)
            x = x + self.W_o(a.transpose(1, 2).contiguous().view(weeks, N, dm))
            return x + self.fc2(torch.relu(self.fc1(self.n2(x))))

    class Encoder(nn.Module):
        def __init__(self):
            super().__init__()
            self.embed = nn.Linear(feats, dm)
            self.layers = nn.ModuleList(Layer() for _ in range(layers))
            self.norm = nn.LayerNorm(dm)
            self.head = nn.Linear(dm, 1)

        def forward(self, f):
            x = self.embed(f)
            for layer in self.layers:
                x = layer(x)
            return self.head(self.norm(x))

    model = Encoder().to(dev)
    nparams = sum(p.numel() for p in model.parameters())
    opt = torch.optim.AdamW(model.parameters(), lr=1e-4, fused=True)
    gen = torch.Generator(device=dev).manual_seed(1)
    feat = torch.randn(weeks, N, feats, device=dev, generator=gen)
    target = torch.rand(weeks, N, 1, device=dev, generator=gen)

    def train_step():
        opt.zero_grad(set_to_none=True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = torch.nn.functional.mse_loss(model(feat).float(), target)
        loss.backward()
        opt.step()
        return loss

    def time_steps():
        for _ in range(args.warmup):
            train_step()
        torch.cuda.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(args.steps):
            ls = train_step()
        t1.record()
        torch.cuda.synchronize()
        return t0.elapsed_time(t1) / args.steps, ls

    eager_ms = None
    if not args.no_eager:
        eager[0] = True
        eager_ms, _ = time_steps()
        eager[0] = False
    ms, loss = time_steps()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    # the attention alone at the step's shape (12 layers' fwd+bwd), to report its share of the step
    (qa, ka, va, doa), (a0, b0, c0) = inputs(weeks, 3, "cpu")
    qa, ka, va, doa = (t.to(dev) for t in (qa, ka, va, doa))
    pa = [t.to(dev).requires_grad_(True) for t in (a0, b0, c0)]
    xs = [t.detach().requires_grad_(True) for t in (qa, ka, va)]
    for _ in range(args.warmup):
        g.geo_attention(*xs, geom, *pa).backward(doa)
    torch.cuda.synchronize()
    e0.record()
    for _ in range(args.steps * layers):
        g.geo_attention(*xs, geom, *pa).backward(doa)
    e1.record()
    torch.cuda.synchronize()
    attn_ms = e0.elapsed_time(e1) / args.steps
    attn_flops = layers * flops(weeks)
    dense_flops = 6.0 * nparams * weeks * N
    pk, pk_src = peaks()
    line = {"metric": "geo-attention encoder training step (fwd+bwd+fused AdamW), ms/step", "value": ms,
            "unit": "ms/step", "higher_is_better": False, "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "dtype": "bf16 autocast (fp32 master weights)", "data": "synthetic",
            "config": {"workload": "12-layer pre-LN encoder, d_model 2048, 16 heads x 128, FFN 8192, 24 weeks x 512 "
                                   "stations x 15 features, MSE vs U(0,1) targets, fused AdamW, random init",
                       "params": nparams, "tokens_per_step": weeks * N, "attention_batch": weeks},
            "eager_attention_ms_per_step": eager_ms,
            "attention_ms_per_step": attn_ms, "attention_share": attn_ms / ms,
            "attention_tflops": attn_flops / (attn_ms * 1e-3) / 1e12,
            "model_tflops": (dense_flops + attn_flops) / (ms * 1e-3) / 1e12,
            "model_tensor_frac": (dense_flops + attn_flops) / (ms * 1e-3) / 1e12 / pk, "peak_source": pk_src,
            "loss": float(loss.item())}
    print(json.dumps(line), flush=True)
    return 0


def measure_c5step(args, dev, rank, world, geom):
    """The scaling configuration's whole step on this rank's shard: x [B/world, N, 2048] -> W_qkv -> geo-attention
    (16 heads x 128, the kernels on strided views of the fused projection) -> W_o -> loss, forward and backward under
    bf16 autocast with fp32 weights, and (N > 1) one NCCL all-reduce of dW_qkv, dW_o (67 MB fp32) and
    d(alpha, beta, gamma) after the backward.

    Returns the max-over-ranks device times (CUDA events) of: the step as run (``ms_per_step``); the same step without
    the all-reduce (``compute_ms``); and the all-reduce alone (``allreduce_ms``). Every loop runs the same number of
    times on every rank."""
    import torch.nn as nn
    import foreswe_gpu_optimization_b200 as g
    from foreswe_gpu_optimization_b200.dp import shard
    dist_on = world > 1
    if dist_on:
        import torch.distributed as tdist
    dm = H * D
    s0, s1 = shard(B_TOTAL, world, rank)
    b = s1 - s0

    class Step(nn.Module):
        def __init__(self):
            super().__init__()
            self.W_qkv = nn.Linear(dm, 3 * dm, bias=False)
            self.W_o = nn.Linear(dm, dm, bias=False)
            gp = torch.Generator().manual_seed(7)
            self.alpha = nn.Parameter(torch.rand(H, generator=gp) * 0.9 + 0.1)
            self.beta = nn.Parameter(torch.randn(H, generator=gp) * 0.5)
            self.gamma = nn.Parameter(torch.randn(H, generator=gp) * 0.5)

        def forward(self, x):                   # x [b, N, dm]
            qkv = self.W_qkv(x).view(b, N, 3, H, D)
            q, k, v = (qkv[:, :, i].transpose(1, 2) for i in range(3))   # [b, H, N, D] strided views
            o = g.geo_attention(q, k, v, geom, self.alpha, self.beta, self.gamma)
            return self.W_o(o.transpose(1, 2).reshape(b, N, dm))

    torch.manual_seed(0)
    model = Step().to(dev)
    params = list(model.parameters())
    # every parameter's gradient is a view of one flat fp32 buffer, all-reduced (averaged) in place in one NCCL call
    # once the backward is done. An all-reduce overlapped with the backward (DDP's bucket hooks) competes for SMs
    # with the persistent attention kernels, which hold every SM until they finish: its kernels then wait for SMs,
    # and the next persistent kernel's last CTAs wait for them (measured: 1.37 ms exposed at 4 GPUs against 0.19 ms
    # for the all-reduce alone).
    flat = torch.zeros(sum(p.numel() for p in params), device=dev)
    off = 0
    for p_ in params:
        p_.grad = flat[off:off + p_.numel()].view_as(p_)
        off += p_.numel()
    if dist_on:
        for p_ in params:                       # same initial weights on every rank
            tdist.broadcast(p_.data, src=0)
    gen = torch.Generator(device=dev).manual_seed(100 + rank)
    x = torch.randn(b, N, dm, device=dev, generator=gen)
    target = torch.randn(b, N, dm, device=dev, generator=gen)

    def step(sync=True):
        flat.zero_()
        with torch.autocast("cuda", dtype=torch.bfloat16):
            y = model(x)
        loss = torch.nn.functional.mse_loss(y.float(), target)
        loss.backward()
        if dist_on and sync:
            tdist.all_reduce(flat, op=tdist.ReduceOp.AVG)
        return loss

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        if dist_on:
            tdist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            r = fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / args.steps, r

    ms, loss = timed(step)
    comp_ms, ar_ms = ms, 0.0
    if dist_on:
        comp_ms, _ = timed(lambda: step(sync=False))

        def allreduce():
            tdist.all_reduce(flat, op=tdist.ReduceOp.AVG)
        ar_ms, _ = timed(allreduce)
        tt = torch.tensor([ms, comp_ms, ar_ms], device=dev, dtype=torch.float64)
        tdist.all_reduce(tt, op=tdist.ReduceOp.MAX)
        ms, comp_ms, ar_ms = tt.tolist()
    attn_flops = flops(B_TOTAL)
    proj_flops = 24.0 * B_TOTAL * N * dm * dm          # W_qkv and W_o: forward 8 B N dm^2, backward twice that
    res = {"ms_per_step": ms, "tflops": (attn_flops + proj_flops) / (ms * 1e-3) / 1e12,
           "compute_ms": comp_ms, "allreduce_ms": ar_ms,
           "exposed_allreduce_ms": max(0.0, ms - comp_ms),
           "attention_tflop_per_step": attn_flops / 1e12, "projection_tflop_per_step": proj_flops / 1e12,
           "per_gpu_batch": b, "loss": float(loss.item()),
           "allreduce_payload_mb": flat.numel() * 4 / 1e6,
           "what": "x -> W_qkv -> geo-attention -> W_o -> MSE, fwd+bwd, bf16 autocast, fp32 weights; one NCCL "
                   "all-reduce (average) of dW_qkv, dW_o, d(alpha, beta, gamma) from a flat gradient buffer after the "
                   "backward (N > 1); compute_ms = the same step without it; allreduce_ms = that all-reduce alone; "
                   "max over ranks"}
    del model, flat, params
    torch.cuda.empty_cache()
    return res


def run_c5step(args):
    """The scaling configuration's whole step (``measure_c5step``) as its own JSON line (ms per step)."""
    import datetime
    import foreswe_gpu_optimization_b200 as g
    rank, world = int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist_on = world > 1
    if dist_on:
        import torch.distributed as tdist
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    geom = g.StationGeometry(*stations(0), device=dev)
    r = measure_c5step(args, dev, rank, world, geom)
    if rank == 0:
        dm = H * D
        line = {"metric": "geo-attention scaling step (W_qkv -> geo-attn -> W_o fwd+bwd + gradient all-reduce), ms/step",
                "value": r["ms_per_step"], "unit": "ms/step", "higher_is_better": False, "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "dtype": "bf16 autocast (fp32 weights)", "data": "synthetic",
                "config": {"workload": "%d issue dates sharded over %d GPU(s) x %d stations, d_model %d, %d heads x %d; "
                                       "all-reduce of dW_qkv, dW_o (%.0f MB fp32) and d(alpha, beta, gamma), one call after the backward"
                                       % (B_TOTAL, world, N, dm, H, D, 4 * dm * dm * 4 / 1e6),
                           "per_gpu_batch": r["per_gpu_batch"]},
                "step_tflops": r["tflops"], "step": r}
        print(json.dumps(line), flush=True)
    if dist_on:
        tdist.barrier()
        tdist.destroy_process_group()
    return 0


# (name, issue dates B, heads H, stations N, head dim D, storage dtype, logit scale on q)
CONFIGS = (("c2_tf32", 32, 8, 512, 64, torch.float32, 1.0),
           ("c2_tf32_saturated_x30", 32, 8, 512, 64, torch.float32, 30.0),
           ("c3_bf16", 384, 16, 512, 64, torch.bfloat16, 1.0),
           ("reference_shape_tf32_d192", 1, 16, 512, 192, torch.float32, 1.0),
           ("production_heads_tf32_d192_b32", 32, 16, 512, 192, torch.float32, 1.0),
           ("production_heads_bf16_d192_b32", 32, 16, 512, 192, torch.bfloat16, 1.0))
# the reference's published fwd / bwd / fwd+bwd times (ms) at its production shape [1, 16, 512, 192], TF32, A100
REFERENCE_A100_D192 = {"triton_v2_accurate": [0.491, 1.930, 2.191], "eager_tf32": [0.332, 0.564, 0.857]}


def reference_triton_v2():
    """The reference's fused Triton v2 operator (foreswe_bench/geo_attention_v2.py) from its offline install in
    baseline/_ref (baseline/install_reference.sh), with its default `accurate_experimental` preset; a string saying
    why when it is not installed."""
    ref = os.path.join(REPO, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "foreswe_bench")):
        return "reference not installed in baseline/_ref (sh baseline/install_reference.sh <reference checkout>)"
    if ref not in sys.path:
        sys.path.append(ref)
    try:
        from foreswe_bench import geo_attention_v2 as v2
    except Exception as exc:
        return "import failed: %s: %s" % (type(exc).__name__, str(exc).splitlines()[0][:200])
    v2.use_preset("accurate_experimental")
    return v2


def config_line(args, name, b, h, n, d, dtype, qscale, dev, pk_bf16, pk_src, triton=True):
    """One configuration: fwd, bwd and fwd+bwd ms of the kernels (coordinate prior, per-head alpha/beta/gamma,
    q/k/v ~ N(0,1) D^-1/4, dO ~ N(0,1)), of eager PyTorch on the same GPU and inputs (TF32 matmuls for fp32 storage,
    as the reference's eager TF32 baseline) and, for fp32 storage, of the reference's Triton v2 op; CUDA events,
    after warm-up; peak extra memory of each."""
    import foreswe_gpu_optimization_b200 as g
    gen = torch.Generator().manual_seed(11)
    s = d ** -0.25
    q, k, v = (torch.randn(b, h, n, d, generator=gen) * s for _ in range(3))
    q = q * qscale
    do = torch.randn(b, h, n, d, generator=gen)
    q, k, v, do = (t.to(dev, dtype) for t in (q, k, v, do))
    gp = torch.Generator().manual_seed(7)
    params = [(torch.rand(h, generator=gp) * 0.9 + 0.1), torch.randn(h, generator=gp) * 0.5,
              torch.randn(h, generator=gp) * 0.5]
    params = [t.to(dev).requires_grad_(True) for t in params]
    rng = np.random.default_rng(0)
    geom = g.StationGeometry(rng.uniform(35.0, 49.0, n), rng.uniform(-124.0, -104.0, n),
                             rng.uniform(500.0, 3500.0, n) / 0.3048, device=dev)
    dmat, amat = geom.distance_and_angularity()
    x = [t.detach().requires_grad_(True) for t in (q, k, v)]

    def ours():
        return g.geo_attention(x[0], x[1], x[2], geom, *params)

    def eager():
        s_ = torch.softmax(torch.matmul(x[0], x[1].transpose(-2, -1)) / math.sqrt(d), dim=-1)
        z = (params[0].view(-1, 1, 1) * s_ + params[1].view(-1, 1, 1) / (1 + dmat)
             + params[2].view(-1, 1, 1) / (1 + amat))
        return torch.matmul(torch.softmax(z, dim=-1).to(dtype), x[2])

    def timed(fn, backward):
        def once():
            for t in x + params:
                t.grad = None
            o = fn()
            if backward:
                o.backward(do)
        for _ in range(args.warmup):
            once()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            once()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / args.steps

    def triple(fn):
        try:
            f, fb = timed(fn, False), timed(fn, True)
            return {"fwd": f, "bwd": fb - f, "fwd_bwd": fb}
        except torch.OutOfMemoryError:
            torch.cuda.empty_cache()
            return None

    def mem_of(fn):
        def once():
            for t in x + params:
                t.grad = None
            fn().backward(do)
        try:
            return round(peak_extra_memory(once, dev)["peak_extra_mib"], 1)
        except torch.OutOfMemoryError:
            torch.cuda.empty_cache()
            return None

    mine = triple(ours)
    ref = None if args.no_eager else triple(eager)
    mem = {"ours": mem_of(ours), "eager": None if args.no_eager else mem_of(eager)}
    tri = None
    if triton and not args.no_triton and dtype == torch.float32:
        v2 = reference_triton_v2()
        if isinstance(v2, str):
            tri = {"unavailable": v2}
        else:
            sc = [t[:1] for t in params]   # the Triton v2 op takes scalar alpha, beta, gamma (same work)
            try:
                tri = triple(lambda: v2.fused_geo_attention_v2(x[0], x[1], x[2], dmat, amat, *sc))
                if tri is not None:
                    tri["preset"] = "accurate_experimental"
                    tri["speedup_ours_vs_triton_v2"] = tri["fwd_bwd"] / mine["fwd_bwd"]
                    mem["triton_v2"] = mem_of(lambda: v2.fused_geo_attention_v2(x[0], x[1], x[2], dmat, amat,
                                                                                *sc))
            except Exception as exc:   # a compile or launch error of the reference's kernel is reported
                tri = {"unavailable": "%s: %s" % (type(exc).__name__, str(exc).splitlines()[0][:200])}
    fl = 12.0 * b * h * n * n * d
    line = {"workload": name, "shape_bhnd": [b, h, n, d], "dtype": "bf16" if dtype == torch.bfloat16 else "fp32 (tf32)",
            "steps": args.steps, "warmup": args.warmup, "ms": mine, "eager_ms": ref, "triton_v2_ms": tri,
            "peak_extra_mib_fwd_bwd": mem,
            "tflops": fl / (mine["fwd_bwd"] * 1e-3) / 1e12,
            "speedup_vs_eager": (ref["fwd_bwd"] / mine["fwd_bwd"]) if ref else None,
            "l2": "inputs %s L2 (q,k,v,dO = %.0f MB)" % ("larger than" if 4 * q.numel() * q.element_size() > 126e6
                                                        else "within", 4 * q.numel() * q.element_size() / 1e6)}
    if dtype == torch.bfloat16:
        line["tensor_frac_of_sustained_bf16"] = line["tflops"] / pk_bf16
        line["peak_source"] = pk_src
    if name == "reference_shape_tf32_d192":
        line["reference_a100_ms_fwd_bwd_fwdbwd"] = REFERENCE_A100_D192
    del q, k, v, do, x, geom, dmat, amat
    torch.cuda.empty_cache()
    return line


def run_configs(args):
    """The other configurations of the path, one JSON line each (config_line)."""
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    torch.backends.cuda.matmul.allow_tf32 = True
    pk_bf16, pk_src = peaks()
    for name, b, h, n, d, dtype, qscale in CONFIGS:
        if args.only and name != args.only:
            continue
        if args.batch:
            b = args.batch
        print(json.dumps(config_line(args, name, b, h, n, d, dtype, qscale, dev, pk_bf16, pk_src)), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=("ours", "reference"))
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-eager", action="store_true")
    ap.add_argument("--no-step", action="store_true", help="skip the whole-step (projections + all-reduce) key")
    ap.add_argument("--no-configs", action="store_true", help="skip the C2 / C3 lines of the default run")
    ap.add_argument("--no-triton", action="store_true", help="configs: skip the reference's Triton v2 timing")
    ap.add_argument("--preroll-seconds", type=float, default=0.3,
                    help="busy pre-roll before the timed region (0 for short profiling runs)")
    ap.add_argument("--batch", type=int, default=None, help="override the global batch (small cases for profiling)")
    ap.add_argument("--only", default=None, choices=[c[0] for c in CONFIGS],
                    help="with --workload configs: run this configuration only")
    ap.add_argument("--workload", default="c5", choices=("c5", "c5step", "c4", "configs"),
                    help="c5: the attention scaling configuration (the headline line); c5step: its whole step with the "
                         "W_qkv / W_o projections and their gradient all-reduce; c4: a full encoder training step; "
                         "configs: the other shapes (C2, C3, the reference's published shape), one line each")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    if args.batch and args.workload not in ("configs",):
        global B_TOTAL
        B_TOTAL = args.batch
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "c4":
        return run_c4(args)
    if args.workload == "configs":
        return run_configs(args)
    if args.workload == "c5step":
        return run_c5step(args)

    import foreswe_gpu_optimization_b200 as g
    from foreswe_gpu_optimization_b200 import geo_attention_v2 as gv2

    rank, world = int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist_on = world > 1
    if dist_on:
        import datetime
        import torch.distributed as tdist
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    if B_TOTAL % world:
        raise SystemExit("world size must divide %d" % B_TOTAL)
    from foreswe_gpu_optimization_b200.dp import shard
    s0, s1 = shard(B_TOTAL, world, rank)
    b = s1 - s0
    lat, lon, el = stations(0)
    geom = g.StationGeometry(lat, lon, el, device=dev)
    geom.prior(torch.bfloat16)
    (qh, kh, vh, doh), (a0, b0, c0) = inputs(b, 1000 + rank, "cpu")
    q, k, v, do = (t.to(dev) for t in (qh, kh, vh, doh))
    params = [t.to(dev).requires_grad_(True) for t in (a0, b0, c0)]
    x = [t.detach().requires_grad_(True) for t in (q, k, v)]

    from foreswe_gpu_optimization_b200.dp import allreduce_bias_grads as _allreduce

    def allreduce_bias_grads():
        _allreduce(params)

    def step(qq, kk, vv, dd):
        for t in x + params:
            t.grad = None
        o = g.geo_attention(qq, kk, vv, geom, *params)
        o.backward(dd)
        allreduce_bias_grads()

    phase("inputs ready; warm-up")
    # warm-up
    for _ in range(args.warmup):
        step(x[0], x[1], x[2], do)
    torch.cuda.synchronize()
    mem = peak_extra_memory(lambda: step(x[0], x[1], x[2], do), dev)

    # The step (fwd + bwd and, for N > 1, the bias-gradient all-reduce) captured as one CUDA graph: the timed region
    # replays it, so host-side launch work (autograd, argument packing) does not pace the GPU at small shards.
    graph = None
    try:
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(2):
                step(x[0], x[1], x[2], do)
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        for t in x + params:
            t.grad = None
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            o_g = g.geo_attention(x[0], x[1], x[2], geom, *params)
            o_g.backward(do)
            allreduce_bias_grads()
        del o_g
    except RuntimeError as exc:  # capture unavailable: time eager steps instead
        print("bench: CUDA graph capture failed (%s); timing eager steps" % str(exc).splitlines()[0], file=sys.stderr)
        graph = None
    use_graph = graph is not None
    if dist_on:  # every rank takes the same path
        flag = torch.tensor([1 if use_graph else 0], device=dev)
        tdist.all_reduce(flag, op=tdist.ReduceOp.MIN)
        use_graph = bool(flag.item())

    def run_step():
        if use_graph:
            graph.replay()
        else:
            step(x[0], x[1], x[2], do)

    for _ in range(args.warmup):
        run_step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(3):
        run_step()
    e1.record()
    torch.cuda.synchronize()
    est_ms = e0.elapsed_time(e1) / 3

    # clocks are sampled from a busy pre-roll of ~0.3 s through the timed region and the per-kernel pass below,
    # all the same workload, so even a short timed region has samples under load. Every step holds an all-reduce
    # (N > 1), so the pre-roll length is agreed over the ranks (max of their estimates) before any rank starts it.
    from foreswe_gpu_optimization_b200.dp import agreed_count
    preroll = agreed_count(est_ms, args.preroll_seconds, device=dev) if args.preroll_seconds > 0 else 0
    phase("graph=%s est %.3f ms/step, pre-roll %d steps" % (use_graph, est_ms, preroll))
    clocks = ClockSampler(range(world) if world > 1 else [local])
    if rank == 0:
        clocks.start()
    for _ in range(preroll):
        run_step()
    if dist_on:
        tdist.barrier()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for i in range(args.steps):
        run_step()
    t1.record()
    torch.cuda.synchronize()
    if dist_on:
        tdist.barrier()
    ms = t0.elapsed_time(t1) / args.steps
    phase("timed region done: %.3f ms/step" % ms)

    # per-kernel times for the roofline: the same K steps run eagerly, with events the library records around each
    # kernel on its launching stream (one set per step)
    def mk(n):
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(n)]
        for e in evs:
            e.record()
        return evs
    ev_sets = [(mk(2), mk(4)) for _ in range(args.steps)]
    torch.cuda.synchronize()
    for i in range(args.steps):
        gv2.TIMING_EVENTS["fwd"], gv2.TIMING_EVENTS["bwd"] = ev_sets[i]
        step(x[0], x[1], x[2], do)
    torch.cuda.synchronize()
    gv2.TIMING_EVENTS["fwd"] = gv2.TIMING_EVENTS["bwd"] = None
    clk = clocks.stop() if rank == 0 else None
    del graph
    kt = {"geoattn_fwd_kernel": statistics.mean(f[0].elapsed_time(f[1]) for f, _ in ev_sets),
          "geoattn_bwd_rows_kernel": statistics.mean(bw[0].elapsed_time(bw[1]) for _, bw in ev_sets),
          "geoattn_bwd_cols_kernel": statistics.mean(bw[1].elapsed_time(bw[2]) for _, bw in ev_sets),
          "geoattn_bwd_dq_kernel": statistics.mean(bw[2].elapsed_time(bw[3]) for _, bw in ev_sets)}
    if dist_on:
        tt = torch.tensor([ms] + list(kt.values()), device=dev, dtype=torch.float64)
        tdist.all_reduce(tt, op=tdist.ReduceOp.MAX)
        ms = tt[0].item()
        kt = dict(zip(kt.keys(), tt[1:].tolist()))
    value = flops(B_TOTAL) / (ms * 1e-3) / 1e12

    # end to end through the public API: pinned host inputs copied in every step, bias gradients read back
    phase("per-kernel pass done")
    e2e = None
    if not args.no_e2e:
        from foreswe_gpu_optimization_b200.streaming import HostBatchPipeline
        hq, hk, hv, hd = (t.pin_memory() for t in (qh, kh, vh, doh))
        out = torch.empty(3 * H, dtype=torch.float32).pin_memory()
        pipe = HostBatchPipeline(qh.shape, q.dtype, dev, slices=E2E_SLICES)

        def e2e_step():
            for t in params:
                t.grad = None
            pipe.step(hq, hk, hv, hd, geom, *params)   # copies of slice i+1 overlap fwd+bwd of slice i
            allreduce_bias_grads()
            out.copy_(torch.cat([p.grad for p in params]), non_blocking=True)
        for _ in range(args.warmup):
            e2e_step()
        torch.cuda.synchronize()
        if dist_on:
            tdist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            e2e_step()
        e1.record()
        torch.cuda.synchronize()
        ems = e0.elapsed_time(e1) / args.steps
        if dist_on:
            tt = torch.tensor([ems], device=dev, dtype=torch.float64)
            tdist.all_reduce(tt, op=tdist.ReduceOp.MAX)
            ems = tt.item()
        e2e = {"value": flops(B_TOTAL) / (ems * 1e-3) / 1e12, "unit": UNIT, "ms_per_step": ems,
               "h2d_bytes_per_step": 4 * q.numel() * 2, "d2h_bytes_per_step": 3 * H * 4,
               "pipeline": "HostBatchPipeline: %d slices of issue dates, pinned H2D copies overlapped with fwd+bwd"
                           % E2E_SLICES}
        del hq, hk, hv, hd, pipe

    # the configuration's whole step (projections and their gradient all-reduce), every rank, at every N
    phase("e2e done")
    stepm = None if args.no_step else measure_c5step(args, dev, rank, world, geom)
    phase("whole step done")

    eager = None
    if not args.no_eager and rank == 0:
        dmat, amat = geom.distance_and_angularity()
        e_ms = gpu_eager_ms(q, k, v, do, dmat, amat, *[p.detach() for p in params], steps=3)
        if e_ms is not None:
            eager = {"ms_per_step": e_ms, "value": flops(b) / (e_ms * 1e-3) / 1e12, "unit": UNIT,
                     "what": "eager PyTorch (bf16 storage, cuBLAS + elementwise kernels) on this GPU, same shard"}

    # the TF32 configuration and the temporal-batched bf16 one against eager PyTorch on this GPU (one GPU only), so
    # the default line carries them too
    others = None
    if world == 1 and not args.no_configs:
        import copy
        a2 = copy.copy(args)
        a2.steps, a2.warmup = 5, 3
        tf32_was = torch.backends.cuda.matmul.allow_tf32
        torch.backends.cuda.matmul.allow_tf32 = True
        pk2, src2 = peaks()
        others = [config_line(a2, *cfg, dev, pk2, src2, triton=False) for cfg in CONFIGS
                  if cfg[0] in ("c2_tf32", "c3_bf16")]
        torch.backends.cuda.matmul.allow_tf32 = tf32_was
        phase("other configurations done")

    cpu = None
    if rank == 0 and world == 1:
        threads = os.cpu_count() or 1
        val, reps, el_s = cpu_reference(args.cpu_seconds, threads)
        cpu = {"value": val, "unit": UNIT, "cores": threads, "kind": "port",
               "sample": "fwd+bwd of 1 issue date (H=%d, N=%d, D=%d) fp32 eager on the CPU, %d repetitions in %.1f s"
                         % (H, N, D, reps, el_s), "c1_cpu": cpu_c1(threads)}

    if rank == 0:
        dom = max(kt, key=kt.get)
        # algorithmic flops per launch (recompute not counted): fwd QK^T + PV; row pass dP; key pass dV + dK; dQ GEMM
        unit = 2.0 * b * H * N * N * D
        kflops = {"geoattn_fwd_kernel": 2 * unit, "geoattn_bwd_rows_kernel": unit, "geoattn_bwd_cols_kernel": 2 * unit,
                  "geoattn_bwd_dq_kernel": unit}
        per_launch = kflops[dom]
        ach = per_launch / (kt[dom] * 1e-3) / 1e12
        pk, pk_src = peaks()
        roof = {"bound": "tensor", "kernel": dom, "achieved": ach, "peak": pk, "unit": "TFLOP/s", "frac": ach / pk,
                "peak_source": pk_src, "traffic": traffic_per_launch(dom),
                "kernel_ms": kt, "flops_per_launch": per_launch}
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
                "timing": ("K replays of the step captured as one CUDA graph" if use_graph else "K eager steps")
                          + "; per-kernel times from K eager steps with library events",
                "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": config(world),
                "tensor_peak_frac": value / world / pk, "roofline": roof, "cpu_baseline": cpu, "e2e": e2e,
                "gpu_eager": eager, "step": stepm, "memory": mem, "other_configs": others,
                "gpu_launches": 5 * args.steps, "clocks": clk}
        print(json.dumps(line), flush=True)
    if dist_on:
        tdist.barrier()
        tdist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
