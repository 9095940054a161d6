"""Small, self-contained GPU workloads for profiling and measurement (ncu-sized).

  python -m compressai_b200.diag gather
      random codebook-row gather rates (global / shared / cluster-shared memory)
  python -m compressai_b200.diag gemv --out 151936 --n 2048 --M 1 --bpw 2 --reps 3
      `reps` launches of one VQ GEMV (input RHT fused in the prologue) on a seeded matrix
  python -m compressai_b200.diag moe --T 1 --reps 3
      `reps` MoE layers (router + expert FFN) over 256 resident seeded experts

Each prints one JSON line with the measured device time per launch/layer.
"""
import argparse
import json

import torch

from . import kernels, moe, runtime, synth


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
            ("shared memory, 12288 rows", 1, 65536), ("cluster shared memory (8 CTAs)", 2, 65536)]
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
    x = torch.randn(a.M, a.n, device=dev).half()
    t = _time(lambda: lin(x), a.reps)
    nbytes = a.out * a.n // 8 * (2 if a.bpw == 2 else 3) + 2 * a.out + 2 * a.M * (a.n + a.out)
    print(json.dumps({"gemv": [a.out, a.n, a.M, a.bpw], "us": round(t * 1e6, 2), "GBs": round(nbytes / t / 1e9, 1)}))


def cmd_moe(a):
    dev = torch.device("cuda", 0)
    cbs = _cbs(dev)
    pool = moe.ExpertRecordPool(a.E, dev)
    g = torch.Generator(device=dev).manual_seed(a.seed)
    pool.raw.view(torch.int16).copy_(torch.randint(-32768, 32768, pool.raw.view(torch.int16).shape, generator=g,
                                                   device=dev, dtype=torch.int16))
    pool.gu_scale.copy_(0.02 * torch.ones_like(pool.gu_scale))
    pool.dn_scale.copy_(0.02 * torch.ones_like(pool.dn_scale))
    ex = moe.PackedMoEExpertUniversal(pool, cbs["16"], dev)
    blk = moe.MoEBlock(ex)
    h = torch.randn(a.T, 2048, device=dev).half()
    logits = torch.randn(a.T, a.E, device=dev)
    t = _time(lambda: blk(h, logits), a.reps)
    ids, _ = moe.route(logits, 8)
    distinct = int(torch.unique(ids).numel())
    nbytes = distinct * pool.record_bytes
    print(json.dumps({"moe_T": a.T, "us": round(t * 1e6, 2), "distinct_experts": distinct,
                      "expert_GBs": round(nbytes / t / 1e9, 1), "tok_s": round(a.T / t, 1)}))


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
    m = sub.add_parser("moe")
    m.add_argument("--T", type=int, default=1)
    m.add_argument("--E", type=int, default=256)
    m.add_argument("--reps", type=int, default=3)
    m.add_argument("--seed", type=int, default=0)
    a = ap.parse_args(argv)
    {"gather": cmd_gather, "gemv": cmd_gemv, "moe": cmd_moe}[a.cmd](a)


if __name__ == "__main__":
    main()
