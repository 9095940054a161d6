"""Expert parallelism on 2..8 GPUs (as many as the box has): the EP block's output (rank sum over
NVLink peer memory inside the combine kernel, and the NCCL all_reduce baseline) equals a
single-GPU MoE block holding all experts, identically on every rank, also when the layer stack
runs from a CUDA graph. Skipped with fewer than 2 GPUs; NVLS is off (plain peer loads/stores)."""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

E, T = 256, 4


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results):
    import datetime

    import torch.distributed as dist

    from compressai_b200 import ep, moe, synth, vq
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        cb = torch.from_numpy(synth.random_codebooks(4)["16"]).to(dev)
        shared = synth.synth_expert(31, 0)
        full = moe.ExpertRecordPool(E + 1, dev)
        for e in range(E):
            full.set_expert(e, *[torch.from_numpy(a) for a in synth.synth_expert(30, e)])
        full.set_expert(E, *[torch.from_numpy(a) for a in shared])
        lo, hi = ep.partition(E, world, rank)
        loc = moe.ExpertRecordPool(hi - lo + 1, dev)   # this rank's experts + the shared expert
        loc.raw[: hi - lo].copy_(full.raw[lo:hi])
        loc.raw[hi - lo].copy_(full.raw[E])
        gate = torch.from_numpy((0.05 * np.random.default_rng(1).standard_normal(2048)).astype(np.float32)).to(dev)
        r_in, r_mid = vq.get_rot("moe_expert_2048", 2048, dev), vq.get_rot("moe_expert_512", 512, dev)
        blk = ep.ExpertParallelMoEBlock(loc, cb, E, r_in, r_mid, shared_gate=gate)            # peer reduce
        nccl = ep.ExpertParallelMoEBlock(loc, cb, E, r_in, r_mid, shared_gate=gate, reduce="nccl")
        assert blk.reduce_kind == "peer", getattr(blk, "peer_error", "")
        ref_blk = moe.MoEBlock(moe.PackedMoEExpertUniversal(full, cb, dev, shared=True), shared_gate=gate)
        out = {}
        for t_ in (T, 1):
            h = torch.from_numpy(np.random.default_rng(2 + t_).standard_normal((t_, 2048)).astype(np.float16)).to(dev)
            lg = torch.from_numpy(np.random.default_rng(3 + t_).standard_normal((t_, E)).astype(np.float32)).to(dev)
            ref = ref_blk(h, lg).float().cpu().numpy()
            y = blk(h, lg).float().cpu().numpy()
            yn = nccl(h, lg).float().cpu().numpy()
            out[t_] = (float(np.abs(y - ref).max() / np.abs(ref).max()),
                       float(np.abs(yn - ref).max() / np.abs(ref).max()), y)
        # several layers in one CUDA graph (no NCCL inside): replays equal the eager chain
        h = torch.from_numpy(np.random.default_rng(9).standard_normal((1, 2048)).astype(np.float16)).to(dev)
        lgs = [torch.from_numpy(np.random.default_rng(10 + i).standard_normal((1, E)).astype(np.float32)).to(dev)
               for i in range(3)]
        eager = h
        for lg in lgs:
            eager = blk(eager, lg)
        st = torch.cuda.Stream(dev)
        st.wait_stream(torch.cuda.current_stream(dev))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(st):
            with torch.cuda.graph(g, stream=st):
                x = h
                for lg in lgs:
                    x = blk(x, lg)
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        graph_equal = bool(torch.equal(x, eager))
        blk.peer.check()
        del g
        # row-sharded greedy lm_head: every rank gets the full matrix's greedy ids of every rank's token
        from compressai_b200 import runtime, shard
        V, n = 20000, 2048
        idx, scale = synth.random_matrix(123, V, n)
        cbd = {"16": cb}
        full = runtime.PackedLinear((V, n), (16,), "lm_head", [torch.from_numpy(idx[0])], torch.from_numpy(scale),
                                    cbd, dev)
        lo, hi = shard.shard_rows(V, world, rank)
        sh = runtime.PackedLinear((hi - lo, n), (16,), "lm_head", [torch.from_numpy(idx[0][lo:hi])],
                                  torch.from_numpy(scale[lo:hi]), cbd, dev)
        ex = shard.PeerExchange(None, dev, max_bytes=4 * n * 2)
        head = shard.ShardedLMHead(sh, lo, V, ex)
        xs = torch.from_numpy(np.random.default_rng(77).standard_normal((world, 2, n)).astype(np.float16)).to(dev)
        ids = head.greedy(xs[rank])
        want = full.greedy(xs.reshape(-1, n)).reshape(world, 2)
        ex.check()
        sharded_ok = bool(torch.equal(ids, want))
        results[rank] = (out, graph_equal, sharded_ok)
        torch.cuda.synchronize()
    finally:
        dist.destroy_process_group()


def test_expert_parallel_matches_single_gpu():
    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    mgr = mp.get_context("spawn").Manager()
    results = mgr.dict()
    mp.start_processes(_worker, args=(world, _free_port(), results), nprocs=world, join=True, start_method="spawn")
    for r in range(world):
        out, graph_equal, sharded_ok = results[r]
        assert sharded_ok, r
        for t_, (err_peer, err_nccl, _) in out.items():
            assert err_peer < 2e-3 and err_nccl < 2e-3, (r, t_, err_peer, err_nccl)  # fp16 outputs
        assert graph_equal, r
    for r in range(1, world):
        for t_ in results[0][0]:
            assert np.array_equal(results[0][0][t_][2], results[r][0][t_][2])   # identical on every rank
