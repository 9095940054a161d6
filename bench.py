#!/usr/bin/env python
"""Benchmark of the VQ2 decode hot path on B200 (one JSON line on stdout, rank 0).

Workload (BASELINE config 2 at M = 1, 2 bpw): one decode step of a 24-layer, hidden-2048
decoder whose linears are VQ-compressed -- per layer q/k/v/o 2048x2048, gate/up 2048->6144,
down 6144->2048 -- plus lm_head 2048->151936, chained through the public runtime API (PackedLinearGroup for q/k/v,
PackedLinear for o -- which consumes v in place of attention -- and PackedSwiGLUMLP for
gate/up/down): 4 kernel launches per layer + lm_head, each with the input rotation fused in
its prologue. ~405 MB of compressed weights per step, more than 3x the 126 MB L2, so no L2
flush is needed.

Metric: compressed bytes (indices + fp16 scales + fp16 x + fp16 y per GEMV) per second.
`value`: the step captured in a CUDA graph, inputs resident in HBM. `e2e`: the same step
through the public API with the token's hidden state copied from pinned host memory and the
logits copied back every step. `roofline`: the GEMV kernel alone (a graph of the 169 matrix
GEMVs, one launch each, on pre-rotated inputs), against the measured HBM copy bandwidth and
against the measured random codebook-gather rate.

Multi-GPU: one process per GPU (torchrun); every rank runs its own replica of the step
(the dense decode path does not shard; "replicas only"); value = all ranks' bytes / max time.

--impl reference: the reference's CPU path (gather + einsum GEMV of
scratch/test_cpu_vq_gemv.py, restated in oracle/cpu_path.py) on the host cores, each step a
bounded sample (one layer's 7 GEMVs + 1/24 of lm_head's rows) of the same seeded workload,
generated on the host with numpy; that arm loads nothing of compressai_b200 and touches no GPU.

The JSON line ends with the MoE (BASELINE configs 3 and 5 shapes, T = 1/8/32/64, expert-parallel
at N > 1 with its outputs checked against a single-GPU block holding all experts) and paged
(config 4) results.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

HIDDEN, INTER, VOCAB = 2048, 6144, 151936
# DRAM bytes of one lm_head GEMV launch (ncu dram__bytes rate x duration) over its algorithmic
# bytes, 81.26 MB / 78.39 MB, from the ncu capture of that launch
NCU_TRAFFIC_RATIO = 1.037
MOE_TOKENS = (1, 8, 32, 64)
METRIC = "VQ GEMV HBM GB/s (compressed bytes)"
UNIT = "GB/s"
WORKLOAD = ("config2 decode step: 24 layers x (q,k,v,o 2048x2048; gate,up 2048->6144; down 6144->2048) "
            "+ lm_head 2048->151936; 2 bpw; M=1")


def gemv_bytes(out, n, M=1, bpw3=False):
    """Algorithmic bytes of one GEMV: indices, fp16 scales, fp16 input rows, fp16 output rows."""
    return out * (n // 8) * (3 if bpw3 else 2) + 2 * out + 2 * M * n + 2 * M * out


def shapes(layers):
    s = []
    for _ in range(layers):
        s += [("q", HIDDEN, HIDDEN), ("k", HIDDEN, HIDDEN), ("v", HIDDEN, HIDDEN), ("o", HIDDEN, HIDDEN),
              ("gate", INTER, HIDDEN), ("up", INTER, HIDDEN), ("down", HIDDEN, INTER)]
    s.append(("lm_head", VOCAB, HIDDEN))
    return s


def step_bytes(layers):
    return sum(gemv_bytes(o, n) for _, o, n in shapes(layers))


def make_config(args, world):
    """The workload description both arms print (identical, so the driver can pair them)."""
    return {"workload": WORKLOAD, "global_batch": world, "seq_len": 1, "bpw": 2, "layers": args.layers,
            "step_weight_bytes": step_bytes(args.layers), "l2": "inputs larger than L2 (no flush)",
            "parallelism": f"dense replicas x{world}" if world > 1 else "single GPU"}


# ------------------------------------------------------------------- host (CPU) workloads
def host_matrix(seed, out, n):
    """Seeded int16 indices and fp32 row scales of one matrix, generated on the host (numpy)."""
    import numpy as np
    rng = np.random.default_rng(seed)
    idx = rng.integers(-32768, 32768, size=(out, n // 8), dtype=np.int16)
    scale = (0.02 * np.exp(0.1 * rng.standard_normal(out))).astype(np.float32)
    return torch.from_numpy(idx), torch.from_numpy(scale)


def host_sample(layer, lm_slice=None, layers=24):
    """One layer's 7 matrices (+ rows [r0, r1) of lm_head) as host tensors."""
    work = []
    for j, (_, out, n) in enumerate(shapes(1)[:7]):
        i, sc = host_matrix([1234, layer, j], out, n)
        work.append((i, sc, n))
    if lm_slice is not None:
        r0, r1 = lm_slice
        i, sc = host_matrix([1234, 999, r0], r1 - r0, HIDDEN)
        work.append((i, sc, HIDDEN))
    return work


def cpu_gemv_sample(work, min_seconds, cb):
    """Time the reference CPU GEMV path (oracle/cpu_path.py) over `work` until min_seconds."""
    from oracle import cpu_path
    xs = {n: torch.randn(n) for _, _, n in work}
    nbytes = sum(gemv_bytes(i.shape[0], n) for i, _, n in work)
    t0 = time.perf_counter()
    reps = 0
    while True:
        for i, s, n in work:
            cpu_path.vq_gemv_cpu_streaming(xs[n], i, cb, s)
        reps += 1
        el = time.perf_counter() - t0
        if el >= min_seconds:
            break
    return nbytes * reps, el, reps


def host_codebook():
    import numpy as np
    return torch.from_numpy(np.random.default_rng(1).standard_normal((1 << 16, 8)).astype(np.float16)).float()


def cpu_moe_sample(min_seconds, cb):
    """One MoE layer (8 routed + the shared expert, SwiGLU 2048 -> 512 -> 2048 at 2 bpw) through the
    reference's CPU expert path (vq_moe_parallel_gate_up_cpu / _down_cpu, restated in
    oracle/cpu_path.py) with the normalised rotations, timed on the host cores until
    min_seconds; tok/s of a 40-layer decode step."""
    import numpy as np

    from oracle import cpu_path
    from oracle import vq2_oracle as O
    rng = np.random.default_rng(11)
    P = 9
    gu_idx = torch.from_numpy(rng.integers(-32768, 32768, size=(P, 1024, 256), dtype=np.int16))
    gu_sc = torch.from_numpy((0.02 * np.exp(0.1 * rng.standard_normal((P, 1024)))).astype(np.float32))
    dn_idx = torch.from_numpy(rng.integers(-32768, 32768, size=(P, 2048, 64), dtype=np.int16))
    dn_sc = torch.from_numpy((0.02 * np.exp(0.1 * rng.standard_normal((P, 2048)))).astype(np.float32))
    rots = {}
    for tag, n in (("moe_expert_2048", 2048), ("moe_expert_512", 512)):
        perm, sign, hb = O.rot_params(tag, n)
        rots[n] = (torch.from_numpy(perm), torch.from_numpy(sign).float(), hb)
    slots = list(range(P))
    w = torch.full((P,), 1.0 / P)
    x = torch.randn(2048)

    def layer():
        xr = cpu_path.rht_cpu(x, *rots[2048])
        y_gu = cpu_path.moe_gate_up_cpu(xr, slots, gu_idx, cb, gu_sc)
        act = torch.nn.functional.silu(y_gu[:, :512]) * y_gu[:, 512:]
        act_r = cpu_path.rht_cpu(act, *rots[512])
        y_dn = cpu_path.moe_down_cpu(act_r, slots, dn_idx, cb, dn_sc)
        return (y_dn * w[:, None]).sum(0)

    layer()
    t0 = time.perf_counter()
    reps = 0
    while True:
        layer()
        reps += 1
        el = time.perf_counter() - t0
        if el >= min_seconds:
            break
    t_layer = el / reps
    return {"value": round(1.0 / (40 * t_layer), 3), "unit": "tok/s (40-layer MoE step, T = 1)",
            "cores": torch.get_num_threads(), "kind": "port", "layer_ms": round(t_layer * 1e3, 2),
            "sample": f"one MoE layer (8 routed + shared expert) x{reps} ({el:.1f} s): Rot.fwd + "
                      "vq_moe_parallel_gate_up_cpu + silu*up + Rot.fwd(512) + vq_moe_parallel_down_cpu + "
                      "weighted sum (scratch/test_cpu_paged_moe.py:31-75, rs = 1)"}


# ------------------------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi sampling of SM clock and throttle reasons while the timed region runs."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        # nvidia-smi numbering can differ from CUDA's (CUDA_VISIBLE_DEVICES); select by UUID
        try:
            u = str(torch.cuda.get_device_properties(device).uuid)
            self.index = u if u.startswith("GPU-") else f"GPU-{u}"
        except (AttributeError, RuntimeError):
            self.index = str(device.index)
        self.rows = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-i", str(self.index), "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except (OSError, ValueError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def __exit__(self, *a):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm = [float(r[1]) for r in self.rows if len(r) >= 9 and r[1].replace(".", "").isdigit()]
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"], "samples": 0}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows if len(r) >= 9 for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": float(self.rows[0][2]),
                "reasons": reasons, "samples": len(sm)}


# ---------------------------------------------------------------------------------- our arm
class DecodeStack:
    """The 24-layer dense decode chain over PackedLinear modules (public API)."""

    def __init__(self, layers, device, seed=0):
        from compressai_b200 import runtime, synth
        g = torch.Generator(device=device).manual_seed(seed)
        cbn = synth.random_codebooks(1)
        self.cbs = {k: torch.from_numpy(v).to(device) for k, v in cbn.items()}
        tags = {"q": "attn_in", "k": "attn_in", "v": "attn_in", "o": "attn_out", "gate": "mlp_in",
                "up": "mlp_in", "down": "mlp_down", "lm_head": "lm_head"}
        self.mods = []
        for name, out, n in shapes(layers):
            idx = torch.randint(-32768, 32768, (out, n // 8), generator=g, device=device, dtype=torch.int16)
            scale = (0.02 * torch.exp(0.1 * torch.randn(out, generator=g, device=device))).half()
            self.mods.append((name, runtime.PackedLinear((out, n), (16,), tags[name], [idx], scale, self.cbs, device)))
        self.layers = layers
        self.qkv, self.o, self.mlp = [], [], []
        for li in range(layers):
            q, k, v, o, gate, up, down = (m for _, m in self.mods[7 * li: 7 * li + 7])
            self.qkv.append(runtime.PackedLinearGroup([q, k, v]))
            self.o.append(o)
            self.mlp.append(runtime.PackedSwiGLUMLP(gate, up, down))

    def __call__(self, h):
        for li in range(self.layers):
            q, k, v = self.qkv[li](h)      # one launch: RHT(h) + 3 GEMVs
            a = self.o[li](v)              # one launch: RHT(v) + GEMV
            h = self.mlp[li](a)            # two launches: RHT + gate/up, SwiGLU + RHT + down
        return self.mods[-1][1](h)

    def launches_per_step(self):
        return 4 * self.layers + 1


def time_graph(graph, steps, stream):
    """Replay `graph` `steps` times on `stream`; device time from CUDA events on that stream."""
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(steps):
            graph.replay()
        e1.record(stream)
    e1.synchronize()
    return e0.elapsed_time(e1) / 1e3


def max_over_ranks(t, dist):
    if dist is None:
        return t
    v = torch.tensor([t], dtype=torch.float64, device="cuda")
    dist.all_reduce(v, op=dist.ReduceOp.MAX)
    return float(v.item())


def barrier(dist):
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()


def run_ours(args, dist, rank, world):
    from compressai_b200 import kernels
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    torch.manual_seed(0)
    stack = DecodeStack(args.layers, dev, seed=1234)
    sh = shapes(args.layers)
    sbytes = step_bytes(args.layers)
    stream = torch.cuda.Stream(dev)
    h_static = torch.randn(1, HIDDEN, device=dev).half()
    # warm-up eagerly (first-call setup), then capture the step; the NVTX range marks the
    # eager steps for the ncu launch list (ncu --nvtx --nvtx-include "decode_step/")
    with torch.cuda.stream(stream):
        for _ in range(2):
            torch.cuda.nvtx.range_push("decode_step")
            stack(h_static)
            torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        logits_static = stack(h_static)
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            g.replay()
    barrier(dist)
    with ClockSampler(dev) as clk:
        t = time_graph(g, args.steps, stream)
        barrier(dist)
        t = max_over_ranks(t, dist)

        # e2e: pinned host input -> device, replay, logits -> pinned host, every step
        h_host = torch.randn(args.steps + args.warmup, 1, HIDDEN).half().pin_memory()
        out_host = torch.empty(VOCAB, dtype=torch.float16).pin_memory()
        for i in range(args.warmup):
            with torch.cuda.stream(stream):
                h_static.copy_(h_host[i], non_blocking=True)
                g.replay()
                out_host.copy_(logits_static.view(-1), non_blocking=True)
            stream.synchronize()
        barrier(dist)
        t0 = time.perf_counter()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        for i in range(args.steps):
            with torch.cuda.stream(stream):
                h_static.copy_(h_host[args.warmup + i], non_blocking=True)
                g.replay()
                out_host.copy_(logits_static.view(-1), non_blocking=True)
            stream.synchronize()
        ev1.record(stream)
        ev1.synchronize()
        t_e2e = max(ev0.elapsed_time(ev1) / 1e3, 0.0)
        t_e2e_wall = time.perf_counter() - t0
        barrier(dist)
        t_e2e = max_over_ranks(max(t_e2e, t_e2e_wall), dist)

        # roofline: GEMV kernels alone on pre-rotated inputs
        xr = {n: torch.randn(1, n, device=dev) for n in (HIDDEN, INTER)}
        ys = [torch.empty(1, m.out, device=dev, dtype=torch.float16) for _, m in stack.mods]
        gg = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            for (_, m), y in zip(stack.mods, ys):
                kernels.vq_gemv(xr[m.n], m.idx0, stack.cbs["16"], m.scale, y=y, out_dtype=torch.float16)
        torch.cuda.synchronize()
        with torch.cuda.graph(gg, stream=stream):
            for (_, m), y in zip(stack.mods, ys):
                kernels.vq_gemv(xr[m.n], m.idx0, stack.cbs["16"], m.scale, y=y, out_dtype=torch.float16)
        with torch.cuda.stream(stream):
            for _ in range(args.warmup):
                gg.replay()
        barrier(dist)
        t_gemv = max_over_ranks(time_graph(gg, args.steps, stream), dist)
        gather_ceiling = kernels.gather_rate(stack.cbs["16"])
    clocks = clk.summary()
    step_idx = sum(o * (n // 8) for _, o, n in sh)

    peaks = load_peaks()
    n_gemv = len(sh)
    per_launch_s = t_gemv / (args.steps * n_gemv)
    achieved = sbytes / n_gemv / per_launch_s / 1e9
    res = {
        "metric": METRIC, "value": round(world * sbytes * args.steps / t / 1e9, 2), "unit": UNIT,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(t / args.steps * 1e3, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32 (fp16 in/out, int16 indices)",
        "data": "synthetic: seeded uniform 16-bit indices, fp16 scales ~0.02, N(0,1) fp16 codebook and input",
        "config": make_config(args, world),
        "e2e": {"value": round(world * sbytes * args.steps / t_e2e / 1e9, 2), "unit": UNIT,
                "h2d_bytes_per_step": HIDDEN * 2, "d2h_bytes_per_step": VOCAB * 2,
                "ms_per_step": round(t_e2e / args.steps * 1e3, 4)},
        "roofline": {"bound": "hbm", "kernel": "vq_gemv_kernel", "achieved": round(achieved, 1),
                     "peak": peaks[0], "unit": "GB/s", "frac": round(achieved / peaks[0], 4),
                     "peak_source": peaks[1],
                     "traffic": round(NCU_TRAFFIC_RATIO * sbytes / n_gemv, 0),
                     "traffic_source": "ncu dram bytes of one lm_head launch / its algorithmic bytes = "
                                       f"{NCU_TRAFFIC_RATIO}, x the mean algorithmic bytes per launch",
                     "avg_launch_us": round(per_launch_s * 1e6, 3), "launches_per_step": n_gemv,
                     "gather_ceiling": {"measured_gathers_per_s": round(gather_ceiling, 0),
                                        "achieved_gathers_per_s": round(step_idx / (t_gemv / args.steps), 0),
                                        "frac": round(step_idx / (t_gemv / args.steps) / gather_ceiling, 4),
                                        "note": "each 2-byte index needs one random 16-byte codebook gather"}},
        "gpu_launches": stack.launches_per_step() * args.steps * 2 + n_gemv * args.steps,
        "clocks": clocks,
    }
    return res, stack


# ------------------------------------------------------------------------------ MoE (config 3/5)
def run_moe(args, dev, dist, world, steps, warmup, tokens=MOE_TOKENS):
    """Decode step of a 40-layer stack of MoE blocks (256 routed experts + 1 shared, top-8,
    SwiGLU 2048->512->2048 at 2 bpw, all resident) on device logits, one vq2_moe_layer call per
    layer, the 40 layers in one CUDA graph. N = 1: MoEBlock. N > 1: expert parallel -- rank r
    holds experts [r*256/N, (r+1)*256/N) of every layer plus the shared expert (its token t on
    rank t % N); replicated router; the rank sum in the combine kernel over NVLink peer memory
    (NCCL all_reduce when symmetric memory is unavailable). Every rank also builds the
    single-GPU block over all experts and checks the expert-parallel output against it, layer by
    layer, and that all ranks hold the same output. Expert bytes per layer = (distinct experts +
    shared) x 792,576 B, all ranks together."""
    from compressai_b200 import ep, moe, synth, vq
    L, E = args.moe_layers, 256
    rank = dist.get_rank() if dist is not None else 0
    g = torch.Generator(device=dev).manual_seed(4321)      # identical expert data on every rank
    cb = torch.from_numpy(synth.random_codebooks(1)["16"]).to(dev)
    gl = torch.Generator(device=dev).manual_seed(999)      # identical router inputs on every rank
    lo, hi = ep.partition(E, world, rank)
    r_in, r_mid = vq.get_rot("moe_expert_2048", HIDDEN, dev), vq.get_rot("moe_expert_512", 512, dev)
    Tmax = max(tokens)
    peer_ctx = None
    if world > 1:  # one symmetric buffer for the rank sums of all layers (see ep.py)
        try:
            peer_ctx = ep.PeerReduceContext(None, dev, max_tokens=Tmax, hidden=HIDDEN)
        except Exception:
            peer_ctx = None
    blocks, ref_blocks, gates = [], [], []
    for _ in range(L):
        full = moe.ExpertRecordPool(E + 1, dev)
        w16 = full.raw.view(torch.int16)
        w16.copy_(torch.randint(-32768, 32768, w16.shape, generator=g, device=dev, dtype=torch.int16))
        full.gu_scale.copy_(0.02 * torch.exp(0.1 * torch.randn(full.gu_scale.shape, generator=g, device=dev)))
        full.dn_scale.copy_(0.02 * torch.exp(0.1 * torch.randn(full.dn_scale.shape, generator=g, device=dev)))
        gate = 0.02 * torch.randn(HIDDEN, generator=gl, device=dev)
        ref = moe.MoEBlock(moe.PackedMoEExpertUniversal(full, cb, dev, shared=True), shared_gate=gate)
        if world > 1:
            pool = moe.ExpertRecordPool(hi - lo + 1, dev)
            pool.raw[: hi - lo].copy_(full.raw[lo:hi])
            pool.raw[hi - lo].copy_(full.raw[E])
            blocks.append(ep.ExpertParallelMoEBlock(pool, cb, E, r_in, r_mid, shared_gate=gate,
                                                    reduce="peer" if peer_ctx is not None else "nccl",
                                                    peer_ctx=peer_ctx, max_tokens=Tmax))
            ref_blocks.append(ref)
        else:
            blocks.append(ref)
    peak = load_peaks()[0]
    results = []
    for T in tokens:
        logits = [torch.randn(T, E, generator=gl, device=dev) for _ in range(L)]
        h0 = torch.randn(T, HIDDEN, generator=gl, device=dev).half()

        def step(h):
            for blk, lg in zip(blocks, logits):
                h = blk(h, lg)
            return h

        distinct = sum(int(torch.unique(moe.route(lg, 8)[0]).numel()) + 1 for lg in logits)
        sbytes = distinct * synth.EXPERT_BYTES
        stream = torch.cuda.Stream(dev)
        with torch.cuda.stream(stream):
            step(h0)
        torch.cuda.synchronize()
        gr, graphed = None, True
        try:
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=stream):
                out = step(h0)
        except Exception:  # capture of the NCCL all_reduce refused: time the eager step instead
            gr, graphed = None, False
            torch.cuda.synchronize()
        barrier(dist)

        def replay():
            if gr is not None:
                gr.replay()
            else:
                step(h0)

        with torch.cuda.stream(stream):
            for _ in range(warmup):
                replay()
        barrier(dist)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(steps):
                replay()
            e1.record(stream)
        e1.synchronize()
        t = max_over_ranks(e0.elapsed_time(e1) / 1e3, dist)
        ach = sbytes * steps / t / 1e9
        # router kernel, gate_up, down (+ the peer combine at N > 1, or the separate combine kernel
        # above 64 (token, expert) problems)
        per_layer = 4 if (world > 1 and blocks[0].reduce_kind == "peer") or T * 9 > 64 else 3
        res = {"T": T, "tok_s": round(T * steps / t, 2), "ms_per_step": round(t / steps * 1e3, 4),
               "us_per_layer": round(t / steps / L * 1e6, 2), "distinct_experts_per_layer": round(distinct / L, 2),
               "roofline": {"bound": "hbm", "achieved": round(ach, 1), "peak": peak * world, "unit": "GB/s",
                            "frac": round(ach / (peak * world), 4)},
               "launches_per_step": per_layer * L, "graph": graphed}
        # parity: the output of one eager step
        torch.cuda.synchronize()
        if world > 1:
            worst, h = 0.0, h0
            for blk, rb, lg in zip(blocks, ref_blocks, logits):
                y = blk(h, lg)
                r = rb(h, lg)
                worst = max(worst, float((y.float() - r.float()).abs().max() / r.float().abs().max()))
                h = y
            mine = h.contiguous()
            allv = [torch.empty_like(mine) for _ in range(world)]
            dist.all_gather(allv, mine)
            res["max_rel_err_vs_single_gpu"] = round(max_over_ranks(worst, dist), 7)
            res["ranks_identical"] = all(bool(torch.equal(allv[0], v)) for v in allv[1:])
            res["finite"] = bool(torch.isfinite(mine.float()).all())
        else:
            with torch.cuda.stream(stream):
                out = step(h0)
            torch.cuda.synchronize()
            res["finite"] = bool(torch.isfinite(out.float()).all())
        del gr
        results.append(res)
    summary = {"layers": L, "experts": f"{E} routed + 1 shared, top-8, 2 bpw, all resident",
               "bytes_per_layer": "(distinct + 1) x 792,576", "per_T": results,
               "parallelism": (f"expert-parallel x{world}, rank sum: " +
                               ("combine kernel over NVLink peer memory" if blocks[0].reduce_kind == "peer"
                                else "NCCL all_reduce")) if world > 1 else "single GPU"}
    if peer_ctx is not None:
        peer_ctx.check()
    del blocks, ref_blocks
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return summary


# ------------------------------------------------------------------------------ config 5 stack
def run_stack(args, dev, dist, world, batches=(1, 8, 64)):
    """the 35B-A3B-shaped Qwen3.5-MoE text model (40 layers: 30 Gated-DeltaNet
    + 10 full-attention, hidden 2048, 256 experts + 1 shared, top-8, expert inter 512, vocab
    248320), random-init, every linear VQ 2 bpw, attention / DeltaNet / norms the transformers
    modules (torch fallback path: no fla / causal-conv1d kernels in the image), the MoE blocks
    on this library's kernels -- expert-parallel across the N ranks at N > 1 (every rank runs
    the same batch; experts split; rank sum over NVLink peer memory). Greedy decode through the
    HF cache, eager (no graph); tokens/s of the whole group."""
    from compressai_b200 import stack
    group = dist.group.WORLD if dist is not None else None
    t0 = time.perf_counter()
    model = stack.build_vq2_moe_model(None, dev, seed=11, group=group, max_tokens=max(batches))
    build_s = time.perf_counter() - t0
    res = {"model": "Qwen3.5-MoE 35B-A3B shape, random-init, VQ 2 bpw", "build_s": round(build_s, 1),
           "parallelism": f"expert-parallel x{world}" if world > 1 else "single GPU", "per_batch": []}
    for B in batches:
        barrier(dist)
        t, ids = stack.decode(model, batch=B, prompt_len=4, steps=args.stack_steps, warmup=2, seed=B)
        t = max_over_ranks(t, dist)
        entry = {"batch": B, "ms_per_step": round(t * 1e3, 3), "tok_s": round(B / t, 2)}
        if world > 1:
            allv = [torch.empty_like(ids) for _ in range(world)]
            dist.all_gather(allv, ids.contiguous())
            entry["ranks_identical"] = all(bool(torch.equal(allv[0], v)) for v in allv[1:])
        res["per_batch"].append(entry)
    del model
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return res


# ------------------------------------------------------------------------ row-sharded lm_head (N > 1)
def run_sharded_head(args, dev, dist, world):
    """Greedy lm_head (151936 x 2048, 2 bpw) for one token per rank: every rank running the full
    matrix on its own token (replicas) against the row-sharded head (all-gather of the N hidden
    rows over peer memory, the fused-argmax GEMV over this rank's V/N rows for all N tokens, the
    cross-rank key maximum). Both in CUDA graphs; ids checked against the full matrix."""
    from compressai_b200 import runtime, shard, synth
    rank = dist.get_rank()
    g = torch.Generator(device=dev).manual_seed(77)          # the same matrix on every rank
    cbs = {k: torch.from_numpy(v).to(dev) for k, v in synth.random_codebooks(1).items()}
    idx = torch.randint(-32768, 32768, (VOCAB, HIDDEN // 8), generator=g, device=dev, dtype=torch.int16)
    scale = (0.02 * torch.exp(0.1 * torch.randn(VOCAB, generator=g, device=dev))).half()
    full = runtime.PackedLinear((VOCAB, HIDDEN), (16,), "lm_head", [idx], scale, cbs, dev)
    lo, hi = shard.shard_rows(VOCAB, world, rank)
    sh = runtime.PackedLinear((hi - lo, HIDDEN), (16,), "lm_head", [idx[lo:hi].clone()], scale[lo:hi].clone(), cbs,
                              dev)
    ex = shard.PeerExchange(None, dev, max_bytes=8 * HIDDEN * 2)
    head = shard.ShardedLMHead(sh, lo, VOCAB, ex)
    gx = torch.Generator(device=dev).manual_seed(5)
    xs = torch.randn(world, 1, HIDDEN, generator=gx, device=dev).half()   # every rank's token, known to all
    x = xs[rank].clone()
    stream = torch.cuda.Stream(dev)
    res = {"vocab": VOCAB, "rows_per_rank": hi - lo}
    for name, fn in (("replicated", lambda: full.greedy(x)), ("sharded", lambda: head.greedy(x))):
        with torch.cuda.stream(stream):
            fn()
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=stream):
            out = fn()
        barrier(dist)
        with torch.cuda.stream(stream):
            for _ in range(args.warmup):
                gr.replay()
        barrier(dist)
        t = max_over_ranks(time_graph(gr, args.steps, stream), dist)
        res[f"us_{name}"] = round(t / args.steps * 1e6, 2)
        if name == "sharded":
            want = full.greedy(xs.reshape(world, HIDDEN))
            res["ids_equal_full_matrix"] = bool(torch.equal(out.reshape(-1), want))
        del gr
    res["tok_s_replicated"] = round(world / (res["us_replicated"] * 1e-6), 1)
    res["tok_s_sharded"] = round(world / (res["us_sharded"] * 1e-6), 1)
    ex.check()
    return res


# ------------------------------------------------------------------------------ paging (config 4)
def run_paged(args, dev, coding="raw"):
    """40 MoE layers x 256 experts in a pinned host .vq2m image (8.12 GB raw); one PagedMoEExpert
    per layer with 39 slots (1.25 GB of HBM: floor(1.25e9 / (40 x 792,576))); 512 decode steps
    whose top-8 routing is the seeded Zipf(1.1) trace; hidden state chained through the layers.
    coding "vq2a": the ANS-coded container (64 distinct skewed-index experts tiled over the
    grid); each miss copies the compressed record and decodes it on the GPU."""
    import numpy as np

    from compressai_b200 import container, paged_runtime, synth
    L, E, steps, cap = 40, 256, args.paged_steps, 39
    t0 = time.perf_counter()
    if coding == "raw":
        nbytes = container.RESERVED_HEADER_BYTES + L * E * synth.EXPERT_BYTES
        pinned = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
        container.synthetic_vq2m_image(L, E, seed=5, out=pinned.numpy())
    else:
        nbytes = container.ans_image_size(L, E, seed=5)
        pinned = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
        container.synthetic_ans_vq2m_image(L, E, seed=5, out=pinned.numpy())
    store = paged_runtime.PagedModelStore.from_image(pinned, device=dev)
    setup_s = time.perf_counter() - t0
    cb = torch.from_numpy(synth.random_codebooks(1)["16"]).to(dev)
    copy_stream = torch.cuda.Stream(dev)
    mods = [paged_runtime.PagedMoEExpert(ln, store, cb, capacity=cap, device=dev, copy_stream=copy_stream)
            for ln in range(L)]
    trace = synth.zipf_trace(steps, L, seed=0)
    ids_host = [[torch.from_numpy(trace[s, ln][None].astype(np.int64)) for ln in range(L)] for s in range(steps)]
    w = torch.full((1, 8), 1.0 / 8, device=dev)  # router weights stay on the device; ids come to the host
    h = torch.randn(1, HIDDEN, device=dev).half()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t1 = time.perf_counter()
    e0.record()
    for s in range(steps):
        for ln in range(L):
            h = mods[ln](h, ids_host[s][ln], w)
    e1.record()
    e1.synchronize()
    wall = time.perf_counter() - t1
    hits = sum(m.hits for m in mods)
    misses = sum(m.misses for m in mods)
    # H2D link bandwidth on the same pinned source, for the fraction
    buf = torch.empty(64 << 20, dtype=torch.uint8, device=dev)
    src = pinned[: 64 << 20]
    c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    c0.record()
    for _ in range(10):
        buf.copy_(src, non_blocking=True)
    c1.record()
    c1.synchronize()
    h2d = 10 * buf.numel() / (c0.elapsed_time(c1) / 1e3) / 1e9
    paged_gbs = store.bytes_paged / wall / 1e9
    res = {"steps": steps, "layers": L, "capacity_per_layer": cap, "hbm_budget_bytes": L * cap * synth.EXPERT_BYTES,
           "hit_rate": round(hits / (hits + misses), 4), "hits": hits, "misses": misses,
           "bytes_paged": store.bytes_paged, "tok_s": round(steps / wall, 2), "ms_per_step": round(wall / steps * 1e3, 3),
           "device_ms_per_step": round(e0.elapsed_time(e1) / steps, 3),
           "paging_GBs": round(paged_gbs, 2), "h2d_link_GBs": round(h2d, 2), "link_frac": round(paged_gbs / h2d, 4),
           "container_bytes": nbytes, "setup_s": round(setup_s, 1), "source": "pinned host image",
           "index_coding": coding}
    if coding != "raw":
        store.check_decode_status()
        res["record_bytes_vs_raw"] = round(store.bytes_paged / (misses * synth.EXPERT_BYTES), 4)
        res["indices"] = "skewed |N(0, 3000)| (synth_expert_skewed), 64 distinct experts tiled"
    else:
        del mods
        res["device_resident"] = run_paged_device(store, cb, trace, dev, steps, cap, hits, misses)
    del store, pinned
    torch.cuda.empty_cache()
    return res


def run_paged_device(store, cb, trace, dev, steps, cap, host_hits, host_misses):
    """The same trace through DeviceResidentPagedMoE: per layer the LRU kernel, the zero-copy
    fetch of missed records from the pinned image and the expert FFN, all 40 layers of a step in
    one CUDA graph; the step's ids (40 x 8 int32) are copied into the graph's input buffer from
    pinned memory before each replay. No host decision inside a step."""
    import numpy as np

    from compressai_b200 import paged_runtime
    L = store.num_layers
    dr = paged_runtime.DeviceResidentPagedMoE(store, cb, capacity=cap, device=dev)
    ids_pin = torch.from_numpy(trace.astype(np.int32)).pin_memory()   # [steps, L, 8]
    ids_buf = torch.zeros(L, 8, dtype=torch.int32, device=dev)
    w = torch.full((1, 8), 1.0 / 8, device=dev)
    h_in = torch.randn(1, HIDDEN, device=dev).half()
    h_out = torch.empty_like(h_in)
    st = torch.cuda.Stream(dev)
    st.wait_stream(torch.cuda.current_stream(dev))
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(st):
        with torch.cuda.graph(g, stream=st):
            h = h_in
            for ln in range(L):
                h = dr.layer(ln, h, ids_buf[ln], w)
            h_out.copy_(h)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t1 = time.perf_counter()
    with torch.cuda.stream(st):
        e0.record(st)
        for s in range(steps):
            ids_buf.copy_(ids_pin[s], non_blocking=True)
            g.replay()
            h_in.copy_(h_out)
        e1.record(st)
    e1.synchronize()
    wall = time.perf_counter() - t1
    views = [dr.lru_view(ln) for ln in range(L)]
    hits, misses = sum(v[0] for v in views), sum(v[1] for v in views)
    del g
    return {"tok_s": round(steps / wall, 2), "ms_per_step": round(wall / steps * 1e3, 3),
            "device_ms_per_step": round(e0.elapsed_time(e1) / steps, 3), "hits": hits, "misses": misses,
            "same_lru_as_host": hits == host_hits and misses == host_misses and not any(v[4] for v in views),
            "fetch": "SM zero-copy reads of the pinned image", "graph": "one CUDA graph per 40-layer step",
            "finite": bool(torch.isfinite(h_out).all())}


# ------------------------------------------------------------------------------ config-2 sweep
def run_sweep(dev, Ms=(1, 4, 16, 64), reps=10):
    """Per-launch device time of each config-2 shape x {2, 3} bpw x M on pre-rotated inputs,
    over a rotating pool of distinct weight copies of >= 4x L2, in a CUDA graph."""
    import math

    from compressai_b200 import kernels, synth
    cbn = synth.random_codebooks(1)
    cb0, cb1 = (torch.from_numpy(cbn[k]).to(dev) for k in ("16", "16_8"))
    g = torch.Generator(device=dev).manual_seed(77)
    st = torch.cuda.Stream(dev)
    out = []
    for (rows, n) in [(HIDDEN, HIDDEN), (INTER, HIDDEN), (HIDDEN, INTER), (VOCAB, HIDDEN)]:
        for bits in (2, 3):
            nbytes = rows * (n // 8) * (3 if bits == 3 else 2)
            copies = max(2, min(64, math.ceil(4 * 126e6 / nbytes)))
            i0s = [torch.randint(-32768, 32768, (rows, n // 8), generator=g, device=dev, dtype=torch.int16)
                   for _ in range(copies)]
            i1s = [torch.randint(0, 256, (rows, n // 8), generator=g, device=dev, dtype=torch.uint8)
                   for _ in range(copies)] if bits == 3 else [None] * copies
            sc = (0.02 * torch.ones(rows, device=dev)).half()
            for M in Ms:
                xr = torch.randn(M, n, generator=g, device=dev)
                y = torch.empty(M, rows, device=dev, dtype=torch.float16)

                def body():
                    for c in range(copies):
                        kernels.vq_gemv(xr, i0s[c], cb0, sc, i1=i1s[c], cb1=cb1 if bits == 3 else None, y=y,
                                        out_dtype=torch.float16)
                with torch.cuda.stream(st):
                    body()
                torch.cuda.synchronize()
                gr = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gr, stream=st):
                    body()
                with torch.cuda.stream(st):
                    gr.replay()
                t = time_graph(gr, reps, st) / (reps * copies)
                alg = gemv_bytes(rows, n, M, bits == 3)
                tc = M >= 4 or (M >= 2 and rows >= 16384)
                out.append({"out": rows, "n": n, "bpw": bits, "M": M, "us": round(t * 1e6, 2),
                            "GBs": round(alg / t / 1e9, 1), "gathers_per_s": round(rows * n / 8 / t, 0),
                            "path": ("tcgen05" if rows // 128 >= 148 else "mma.sync split-K") if tc
                            else "CUDA cores"})
                del gr
            del i0s, i1s
            torch.cuda.empty_cache()
    return out


def sweep_summary(sweep):
    """{"<out>x<n>": {"b<bpw>": {"<M>": us}}} -- the compact form printed in the JSON line."""
    d = {}
    for e in sweep:
        d.setdefault(f"{e['out']}x{e['n']}", {}).setdefault(f"b{e['bpw']}", {})[str(e["M"])] = e["us"]
    return d


def load_peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback 6.65 TB/s"


def run_reference(args, rank, world):
    """The reference's CPU path on the host cores, rank 0 only: each step one layer's 7 GEMVs and
    1/24 of lm_head's rows of the seeded workload, generated here on the host. Loads nothing of
    compressai_b200 and touches no GPU."""
    if rank != 0:
        return None
    torch.set_num_threads(os.cpu_count())
    cb = host_codebook()
    rows_per = (VOCAB + args.layers - 1) // args.layers
    total_b, total_t = 0, 0.0
    for s in range(args.warmup + args.steps):
        li = s % args.layers
        r0 = li * rows_per
        work = host_sample(li, (r0, min(VOCAB, r0 + rows_per)))
        b, t, _ = cpu_gemv_sample(work, 0.0, cb)
        if s >= args.warmup:
            total_b += b
            total_t += t
    v = round(total_b / total_t / 1e9, 3)
    return {"metric": METRIC, "value": v, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(total_t / args.steps * 1e3, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "impl": "reference",
            "data": "synthetic: seeded uniform 16-bit indices, fp16 scales ~0.02, N(0,1) codebook and input",
            "config": make_config(args, world),
            "cpu_baseline": {"value": v, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
                             "sample": f"per step: one layer's 7 GEMVs + 1/{args.layers} of lm_head rows (a bounded "
                                       "sample of the step; the metric is a rate), gather+einsum fp32 "
                                       "(scratch/test_cpu_vq_gemv.py:53-70)",
                             "moe": cpu_moe_sample(args.cpu_seconds, cb)},
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--layers", type=int, default=24)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--moe-layers", type=int, default=40)
    ap.add_argument("--paged-steps", type=int, default=512)
    ap.add_argument("--dense-only", action="store_true")
    ap.add_argument("--sweep-json", default=None, help="write the full config-2 sweep here")
    ap.add_argument("--stack-steps", type=int, default=6, help="timed decode steps of the config-5 stack")
    ap.add_argument("--no-stack", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":  # host cores only: no process group, no GPU
        res = run_reference(args, rank, world)
        if res is not None:
            print(json.dumps(res), flush=True)
        return
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as tdist
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
        dist = tdist
    try:
        res, stack = run_ours(args, dist, rank, world)
        if rank == 0 and world == 1:
            torch.set_num_threads(os.cpu_count())
            cb = host_codebook()
            b, t, reps = cpu_gemv_sample(host_sample(0), args.cpu_seconds, cb)
            res["cpu_baseline"] = {"value": round(b / t / 1e9, 3), "unit": UNIT,
                                   "cores": torch.get_num_threads(), "kind": "port",
                                   "sample": f"one layer's 7 GEMVs x{reps} ({t:.1f} s), gather+einsum fp32 "
                                             "(scratch/test_cpu_vq_gemv.py:53-70)",
                                   "moe": cpu_moe_sample(args.cpu_seconds, cb)}
        if not args.dense_only:
            dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
            del stack
            torch.cuda.empty_cache()
            if world == 1:
                sweep = run_sweep(dev)
                res["sweep_us"] = sweep_summary(sweep)
                if args.sweep_json:
                    with open(args.sweep_json, "w") as f:
                        json.dump(sweep, f, indent=1)
                res["paged"] = run_paged(args, dev)
                res["paged_ans"] = run_paged(args, dev, coding="vq2a")
            if world > 1:
                res["lm_head_sharded"] = run_sharded_head(args, dev, dist, world)
            if not args.no_stack:
                res["stack35b"] = run_stack(args, dev, dist, world)
            res["moe"] = run_moe(args, dev, dist, world, args.steps, args.warmup)
        if rank == 0 and res is not None:
            print(json.dumps(res), flush=True)
    finally:
        if dist is not None:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
