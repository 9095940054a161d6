"""Expert parallelism on 2 GPUs (NCCL): the EP block's output equals a single-GPU MoE block
holding all experts. Skipped with fewer than 2 GPUs."""
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
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        cb = torch.from_numpy(synth.random_codebooks(4)["16"]).to(dev)
        shared = synth.synth_expert(31, 0)
        full = moe.ExpertRecordPool(E + 1, dev)
        for e in range(E):
            full.set_expert(e, *[torch.from_numpy(a) for a in synth.synth_expert(30, e)])
        full.set_expert(E, *[torch.from_numpy(a) for a in shared])
        lo, hi = ep.partition(E, world, rank)
        n_local = hi - lo + (1 if rank == 0 else 0)
        loc = moe.ExpertRecordPool(n_local, dev)
        loc.raw[: hi - lo].copy_(full.raw[lo:hi])
        if rank == 0:
            loc.raw[hi - lo].copy_(full.raw[E])
        gate = torch.from_numpy((0.05 * np.random.default_rng(1).standard_normal(2048)).astype(np.float32)).to(dev)
        r_in, r_mid = vq.get_rot("moe_expert_2048", 2048, dev), vq.get_rot("moe_expert_512", 512, dev)
        blk = ep.ExpertParallelMoEBlock(loc, cb, E, r_in, r_mid, shared_gate=gate)
        ref_blk = moe.MoEBlock(moe.PackedMoEExpertUniversal(full, cb, dev, shared=True), shared_gate=gate)
        h = torch.from_numpy(np.random.default_rng(2).standard_normal((T, 2048)).astype(np.float16)).to(dev)
        lg = torch.from_numpy(np.random.default_rng(3).standard_normal((T, E)).astype(np.float32)).to(dev)
        y = blk(h, lg).float().cpu().numpy()
        ref = ref_blk(h, lg).float().cpu().numpy()
        results[rank] = (float(np.abs(y - ref).max() / np.abs(ref).max()), y)
        torch.cuda.synchronize()
    finally:
        dist.destroy_process_group()


def test_expert_parallel_two_gpus_matches_single_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    mgr = mp.get_context("spawn").Manager()
    results = mgr.dict()
    mp.start_processes(_worker, args=(2, _free_port(), results), nprocs=2, join=True, start_method="spawn")
    for r in range(2):
        err, _ = results[r]
        assert err < 2e-3, (r, err)   # fp16 outputs of two fp32 sums in different orders
    assert np.array_equal(results[0][1], results[1][1])
