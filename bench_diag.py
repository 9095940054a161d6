"""Small, self-contained GPU workloads for profiling and measurement (ncu-sized): the commands
behind the launch lists and captures summarised in profiles/. Not part of the package.

  python bench_diag.py gather
      random codebook-row gather rates (global / shared / cluster-shared memory)
  python bench_diag.py gemv --out 151936 --n 2048 --M 1 --bpw 2 --reps 3 [--swiglu | --argmax]
      `reps` launches of one VQ GEMV (input RHT fused in the prologue) on a seeded matrix;
      with --swiglu the input is an fp32 [gate | up] row of 2n and SwiGLU + RHT run in the
      prologue (the MLP down projection); with --argmax the fused greedy argmax (keys only)
  python bench_diag.py moe --T 1 --reps 3 [--graph --layers 40] [--shared] [--world 8 --rank 0]
      `reps` MoE layers (router + expert FFN) over 256 resident seeded experts; with --graph,
      `reps` replays of a CUDA graph of `layers` chained layers (each its own router logits); with
      --world N, rank `rank`'s share of an expert-parallel layer (its E/N experts + the shared
      expert, the rank-sum exchange into local buffers whose peer waits give up after one poll)
  python bench_diag.py rans --n 16777216 --reps 2
      `reps` GPU decodes of one VQ2A stream of n skewed index bytes, then `reps` decodes of one
      ANS-coded expert record (vq2_rans_decode_segments)
  python bench_diag.py paged --layers 2 --experts 64 --steps 8 --T 1 [--coding vq2a]
      native paged MoE steps (vq2_paged_moe_step) over a pinned synthetic .vq2m image
  python bench_diag.py reftriton --reps 50
      the reference's own Triton kernels (vq2/kernels.py, from the offline install under
      baseline/_ref) beside this library's drop-ins of the same functions: same arguments, same
      rotating weight copies (at least 4x L2 of indices per shape), both timed in CUDA graphs

Each prints one JSON line with the measured device time per launch/layer.
"""
import argparse
import json
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
from compressai_b200 import kernels, moe, runtime, synth  # noqa: E402


def _cbs(dev):
    return {k: torch.from_numpy(v).to(dev) for k, v in synth.random_codebooks(1).items()}


def _time(fn, reps):
    fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    e1.synchronize()
    return e0.elapsed_time(e1) / 1e3 / reps


def cmd_gather(a):
    dev = torch.device("cuda", 0)
    cb = _cbs(dev)["16"]
    clk = torch.cuda.get_device_properties(dev)
    sms = clk.multi_processor_count
    rows = [("global, 65536 rows (L2)", 0, 65536), ("global, 4096 rows (L1)", 0, 4096),
            ("shared memory, 12288 rows", 1, 65536), ("cluster shared memory (8 CTAs)", 2, 65536),
            ("bucketed entry: codeword + fp32 x from shared memory", 3, 65536),
            ("bucketed entry: codeword + fp16 x from shared memory", 4, 65536)]
    out = []
    for name, mode, r in rows:
        g = kernels.gather_rate(cb, mode=mode, rows=r)
        out.append({"path": name, "gathers_per_s": round(g, 0), "per_sm_per_s": round(g / sms, 0)})
    print(json.dumps({"gather": out, "sms": sms}))


def cmd_gemv(a):
    dev = torch.device("cuda", 0)
    cbs = _cbs(dev)
    bits = (16,) if a.bpw == 2 else (16, 8)
    idx, scale = synth.random_matrix(a.seed, a.out, a.n, bits)
    lin = runtime.PackedLinear((a.out, a.n), bits, "diag", [torch.from_numpy(i) for i in idx],
                               torch.from_numpy(scale), cbs, dev)
    if a.argmax:  # fused greedy argmax (no logits written), keys as the row-sharded head uses them
        x = torch.randn(a.M, a.n, device=dev).half()
        cb0, cb1 = lin.codebooks()
        t = _time(lambda: kernels.gemv_argmax(x, lin.mat(), cb0, cb1, rot=lin.rot, keys=True), a.reps)
        xbytes = 2 * a.M * a.n
    elif a.swiglu:
        from compressai_b200 import _lib
        x = torch.randn(a.M, 2 * a.n, device=dev)
        cb0, cb1 = lin.codebooks()
        t = _time(lambda: kernels.gemv_multi(x, [lin.mat()], cb0, cb1, rot=lin.rot, mode=_lib.VQ2_ACT_SWIGLU_RHT,
                                             out_dtype=torch.float16), a.reps)
        xbytes = 4 * a.M * 2 * a.n
    else:
        x = torch.randn(a.M, a.n, device=dev).half()
        t = _time(lambda: lin(x), a.reps)
        xbytes = 2 * a.M * a.n
    nbytes = a.out * a.n // 8 * (2 if a.bpw == 2 else 3) + 2 * a.out + xbytes + 2 * a.M * a.out
    print(json.dumps({"gemv": [a.out, a.n, a.M, a.bpw], "us": round(t * 1e6, 2), "GBs": round(nbytes / t / 1e9, 1)}))


class _LoneRankPeers:
    """The fields moe.moe_layer reads from ep.PeerReduceContext, backed by local buffers that no
    other rank writes: one GPU runs rank `rank`'s share of an expert-parallel layer, and every
    wait for a peer gives up after `max_polls` polls (the partial of this rank is what remains)."""

    def __init__(self, dev, world, rank, max_tokens, hidden, max_polls=1):
        from compressai_b200 import _lib
        nbytes = _lib.load().vq2_moe_peer_buffer_bytes(max_tokens, hidden, world)
        self.bufs = [torch.zeros(nbytes, dtype=torch.uint8, device=dev) for _ in range(world)]
        self.ptrs = torch.tensor([b.data_ptr() for b in self.bufs], dtype=torch.int64, device=dev)
        self.peers_dev = self.ptrs.data_ptr()
        self.rank, self.world, self.max_tokens, self.max_polls = rank, world, max_tokens, max_polls
        self.epochs = torch.zeros(4, dtype=torch.int32, device=dev)
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)


def cmd_moe(a):
    dev = torch.device("cuda", 0)
    cbs = _cbs(dev)
    if a.world > 1:  # one rank of an expert-parallel layer: its expert slice + the shared expert
        from compressai_b200 import vq
        lo, hi = a.rank * a.E // a.world, (a.rank + 1) * a.E // a.world
        pool = moe.ExpertRecordPool(hi - lo + 1, dev)
        g = torch.Generator(device=dev).manual_seed(a.seed)
        pool.raw.view(torch.int16).copy_(torch.randint(-32768, 32768, pool.raw.view(torch.int16).shape, generator=g,
                                                       device=dev, dtype=torch.int16))
        pool.gu_scale.fill_(0.02)
        pool.dn_scale.fill_(0.02)
        peer = _LoneRankPeers(dev, a.world, a.rank, a.T, 2048)
        r_in, r_mid = vq.get_rot("moe_expert_2048", 2048, dev), vq.get_rot("moe_expert_512", 512, dev)
        gate = 0.02 * torch.randn(2048, device=dev)
        h = torch.randn(a.T, 2048, device=dev).half()
        lg = [torch.randn(a.T, a.E, device=dev) for _ in range(a.layers)]

        def step():
            x = h
            for li in range(a.layers):
                x = moe.moe_layer(x, lg[li], pool, cbs["16"], r_in, r_mid, 8, shared_gate=gate, lo=lo, hi=hi,
                                  rank=a.rank, world=a.world, peer=peer)
            return x
        step()
        torch.cuda.synchronize()
        if not a.graph:
            t = _time(step, a.reps) / a.layers
        else:
            st = torch.cuda.Stream(dev)
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=st):
                step()
            t = _time(gr.replay, a.reps) / a.layers
        print(json.dumps({"moe_T": a.T, "world": a.world, "rank": a.rank, "layers": a.layers,
                          "us_per_layer": round(t * 1e6, 2), "peer_waits_gave_up": bool(peer.err.item())}))
        return
    pool = moe.ExpertRecordPool(a.E, dev)
    g = torch.Generator(device=dev).manual_seed(a.seed)
    pool.raw.view(torch.int16).copy_(torch.randint(-32768, 32768, pool.raw.view(torch.int16).shape, generator=g,
                                                   device=dev, dtype=torch.int16))
    pool.gu_scale.copy_(0.02 * torch.ones_like(pool.gu_scale))
    pool.dn_scale.copy_(0.02 * torch.ones_like(pool.dn_scale))
    if a.shared:  # the last pool row serves as the shared expert, with a seeded gate vector
        ex = moe.PackedMoEExpertUniversal(pool, cbs["16"], dev, shared=True)
        blk = moe.MoEBlock(ex, shared_gate=0.02 * torch.randn(2048, device=dev))
    else:
        ex = moe.PackedMoEExpertUniversal(pool, cbs["16"], dev)
        blk = moe.MoEBlock(ex)
    h = torch.randn(a.T, 2048, device=dev).half()
    logits = torch.randn(a.T, a.E, device=dev)
    if a.graph:  # `layers` chained layers, each with its own router logits, in one CUDA graph
        lg = [torch.randn(a.T, a.E, device=dev) for _ in range(a.layers)]

        def step():
            x = h
            for li in range(a.layers):
                x = blk(x, lg[li])
            return x
        step()
        torch.cuda.synchronize()
        st = torch.cuda.Stream(dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            step()
        t = _time(g.replay, a.reps) / a.layers
        print(json.dumps({"moe_T": a.T, "graph_layers": a.layers, "us_per_layer": round(t * 1e6, 2),
                          "tok_s": round(a.T / (t * a.layers), 1)}))
        return
    t = _time(lambda: blk(h, logits), a.reps)
    ids, _ = moe.route(logits, 8)
    distinct = int(torch.unique(ids).numel())
    nbytes = distinct * pool.record_bytes
    print(json.dumps({"moe_T": a.T, "us": round(t * 1e6, 2), "distinct_experts": distinct,
                      "expert_GBs": round(nbytes / t / 1e9, 1), "tok_s": round(a.T / t, 1)}))


def cmd_rans(a):
    import numpy as np

    from compressai_b200 import ans, container
    dev = torch.device("cuda", 0)
    x = np.minimum(np.abs(np.random.default_rng(a.seed).normal(0, 3000, a.n // 2)), 65535).astype(np.uint16)
    enc = torch.from_numpy(ans.encode(x)).to(dev)
    out = torch.empty(a.n, dtype=torch.uint8, device=dev)
    status = ans.new_status(dev)
    t = _time(lambda: ans.decode(enc, a.n, out, status), a.reps)
    ans.check_status(status)
    ok = bool(torch.equal(out.cpu(), torch.from_numpy(x.view(np.uint8))))
    img, _ = container.synthetic_ans_vq2m_image(1, 2, seed=a.seed, distinct=2)
    lay = container.parse_header(memoryview(img[:container.RESERVED_HEADER_BYTES]))
    off, nb = lay.record(0, 1)
    src = torch.from_numpy(img[off:off + nb].copy()).to(dev)
    dst = torch.empty(lay.expert_bytes, dtype=torch.uint8, device=dev)
    segs = lay.segments(0, 1)
    tr = _time(lambda: ans.decode_segments(src, segs, dst, status), a.reps)
    ans.check_status(status)
    print(json.dumps({"rans_bytes": a.n, "encoded": enc.numel(), "us": round(t * 1e6, 2),
                      "decoded_GBs": round(a.n / t / 1e9, 1), "bit_exact": ok, "record_bytes": nb,
                      "record_us_eager": round(tr * 1e6, 2)}))


def cmd_paged(a):
    import time

    import numpy as np

    from compressai_b200 import container, paged_runtime
    dev = torch.device("cuda", 0)
    if a.coding == "raw":
        img, _ = container.synthetic_vq2m_image(a.layers, a.experts, seed=a.seed)
    else:
        img, _ = container.synthetic_ans_vq2m_image(a.layers, a.experts, seed=a.seed, distinct=min(a.experts, 16))
    store = paged_runtime.PagedModelStore.from_image(torch.from_numpy(img).pin_memory(), device=dev)
    cb = _cbs(dev)["16"]
    cs = torch.cuda.Stream(dev)
    mods = [paged_runtime.PagedMoEExpert(ln, store, cb, capacity=a.capacity, device=dev, copy_stream=cs)
            for ln in range(a.layers)]
    rng = np.random.default_rng(a.seed)
    trace = [[torch.from_numpy(np.stack([rng.choice(a.experts, 8, replace=False) for _ in range(a.T)]))
              for _ in range(a.layers)] for _ in range(a.steps)]
    w = torch.full((a.T, 8), 1.0 / 8, device=dev)
    h = torch.randn(a.T, 2048, device=dev).half()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for s in range(a.steps):
        for ln in range(a.layers):
            h = mods[ln](h, trace[s][ln], w)
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    if store.ans_coded:
        store.check_decode_status()
    print(json.dumps({"paged_steps": a.steps, "layers": a.layers, "T": a.T, "coding": a.coding,
                      "native": all(m.native for m in mods), "misses": sum(m.misses for m in mods),
                      "ms_per_step": round(wall / a.steps * 1e3, 3), "finite": bool(torch.isfinite(h).all())}))


def _rotating(fn, copies, reps):
    """Device time per call of fn(c), c cycling over the weight copies, from a CUDA graph of
    `copies` calls replayed `reps` times (no host launch cost in the measurement)."""
    for c in range(copies):  # warm-up (Triton autotuning, first-call set-up) outside the capture
        fn(c)
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for c in range(copies):
            fn(c)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    e1.synchronize()
    return e0.elapsed_time(e1) / 1e3 / (reps * copies)


def cmd_reftriton(a):
    ref_root = os.path.join(os.path.dirname(os.path.abspath(__file__)), "baseline", "_ref")
    if not os.path.isfile(os.path.join(ref_root, "vq2", "kernels.py")):
        print(json.dumps({"reference_triton": "unavailable", "why": "the reference is not installed in baseline/_ref"}))
        return
    sys.path.insert(0, ref_root)
    import vq2.kernels as RK  # the reference package, unmodified
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(a.seed)
    cb = _cbs(dev)["16"].to(torch.bfloat16)
    budget = 4 * 126 * 2 ** 20
    out = []
    for rows, n in ((2048, 2048), (6144, 2048), (2048, 6144), (151936, 2048)):
        ng = n // 8
        copies = max(2, -(-budget // (rows * ng * 2)))
        idx = torch.randint(-32768, 32768, (copies, rows, ng), generator=g, device=dev, dtype=torch.int16)
        sc = (0.02 * torch.ones(copies, rows, device=dev)).to(torch.bfloat16)
        x = torch.randn(n, generator=g, device=dev).to(torch.bfloat16)
        y_ref = RK.vq_gemv_16(x, idx[0], cb, sc[0], rows, n)
        y_own = kernels.vq_gemv_16(x, idx[0], cb, sc[0], rows, n)
        err = float((y_own.float() - y_ref.float()).abs().max() / y_ref.float().abs().max())
        reps = max(1, a.reps * 8 // copies)
        t_ref = _rotating(lambda c: RK.vq_gemv_16(x, idx[c], cb, sc[c], rows, n), copies, reps)
        t_own = _rotating(lambda c: kernels.vq_gemv_16(x, idx[c], cb, sc[c], rows, n), copies, reps)
        out.append({"vq_gemv_16": [rows, n], "copies": copies, "ref_us": round(t_ref * 1e6, 2),
                    "own_us": round(t_own * 1e6, 2), "speedup": round(t_ref / t_own, 2), "max_rel_diff": err})
        del idx, sc
    # one top-8 MoE layer's two expert GEMVs (gate_up on the shared input, down on 8 activations)
    E, copies = 256, 2
    gu = torch.randint(-32768, 32768, (copies, E, 1024, 256), generator=g, device=dev, dtype=torch.int16)
    dn = torch.randint(-32768, 32768, (copies, E, 2048, 64), generator=g, device=dev, dtype=torch.int16)
    gus = (0.02 * torch.ones(copies, E, 1024, device=dev)).to(torch.bfloat16)
    dns = (0.02 * torch.ones(copies, E, 2048, device=dev)).to(torch.bfloat16)
    sets = [torch.randperm(E, generator=g, device=dev)[:8].to(torch.int32) for _ in range(64)]
    x = torch.randn(2048, generator=g, device=dev).to(torch.bfloat16)
    act = torch.randn(8, 512, generator=g, device=dev).to(torch.bfloat16)
    y_gu = torch.empty(8, 1024, device=dev, dtype=torch.bfloat16)
    y_dn = torch.empty(8, 2048, device=dev, dtype=torch.bfloat16)
    own_gu, own_dn = torch.empty_like(y_gu), torch.empty_like(y_dn)

    def ref_layer(c, mod=RK, a_gu=y_gu, a_dn=y_dn):
        ids = sets[c % 64]
        w = c % copies
        mod.vq_moe_parallel_gate_up(x, ids, gu[w], cb, gus[w], a_gu)
        mod.vq_moe_parallel_down(act, ids, dn[w], cb, dns[w], a_dn)
    ref_layer(0)
    ref_layer(0, kernels, own_gu, own_dn)
    err = max(float((own_gu.float() - y_gu.float()).abs().max() / y_gu.float().abs().max()),
              float((own_dn.float() - y_dn.float()).abs().max() / y_dn.float().abs().max()))
    t_ref = _rotating(ref_layer, 128, max(1, a.reps // 10))
    t_own = _rotating(lambda c: ref_layer(c, kernels, own_gu, own_dn), 128, max(1, a.reps // 10))
    out.append({"moe_gate_up_plus_down_top8": [E, 1024, 2048], "ref_us": round(t_ref * 1e6, 2),
                "own_us": round(t_own * 1e6, 2), "speedup": round(t_ref / t_own, 2), "max_rel_diff": err})
    print(json.dumps({"reference_triton": out, "triton": __import__("triton").__version__}))


def main(argv=None):
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="cmd", required=True)
    sub.add_parser("gather")
    g = sub.add_parser("gemv")
    g.add_argument("--out", type=int, default=151936)
    g.add_argument("--n", type=int, default=2048)
    g.add_argument("--M", type=int, default=1)
    g.add_argument("--bpw", type=int, default=2, choices=(2, 3))
    g.add_argument("--reps", type=int, default=3)
    g.add_argument("--seed", type=int, default=0)
    g.add_argument("--swiglu", action="store_true")
    g.add_argument("--argmax", action="store_true")
    m = sub.add_parser("moe")
    m.add_argument("--T", type=int, default=1)
    m.add_argument("--E", type=int, default=256)
    m.add_argument("--reps", type=int, default=3)
    m.add_argument("--seed", type=int, default=0)
    m.add_argument("--graph", action="store_true")
    m.add_argument("--layers", type=int, default=40)
    m.add_argument("--shared", action="store_true", help="the last pool row as a shared expert (9 problems)")
    m.add_argument("--world", type=int, default=1, help="> 1: one rank of an expert-parallel layer on this GPU")
    m.add_argument("--rank", type=int, default=0)
    r = sub.add_parser("rans")
    r.add_argument("--n", type=int, default=1 << 24)
    r.add_argument("--reps", type=int, default=2)
    r.add_argument("--seed", type=int, default=0)
    pg = sub.add_parser("paged")
    pg.add_argument("--layers", type=int, default=2)
    pg.add_argument("--experts", type=int, default=64)
    pg.add_argument("--capacity", type=int, default=16)
    pg.add_argument("--steps", type=int, default=8)
    pg.add_argument("--T", type=int, default=1)
    pg.add_argument("--coding", choices=("raw", "vq2a"), default="raw")
    pg.add_argument("--seed", type=int, default=0)
    rt = sub.add_parser("reftriton")
    rt.add_argument("--reps", type=int, default=50)
    rt.add_argument("--seed", type=int, default=0)
    a = ap.parse_args(argv)
    {"gather": cmd_gather, "gemv": cmd_gemv, "moe": cmd_moe, "rans": cmd_rans, "paged": cmd_paged,
     "reftriton": cmd_reftriton}[a.cmd](a)


if __name__ == "__main__":
    main()
