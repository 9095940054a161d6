"""Expert-parallel host logic on CPU ranks (gloo, world size 2 and 4): partitioning, local id
mapping, the shared expert's tokens spread over the ranks (token t on rank t % N), all_reduce of
the partials -- against the single-process oracle. The per-rank expert compute is a test stand-in built from the oracle (the product's
compute is the CUDA expert FFN)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from compressai_b200 import ep, synth
from oracle import vq2_oracle as O

E, T, K, SEED = 16, 3, 4, 9


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cbs():
    return synth.random_codebooks(2)


def _oracle_ffn_factory(rank_experts, cb16, rot2048, rot512):
    """ffn(h, ids [T, k] local rows, w [T, k], k) over this rank's expert list, fp64 -> fp32."""
    def ffn(h, ids, w, k):
        hn = h.double().numpy()
        out = np.zeros((hn.shape[0], hn.shape[1]))
        for t in range(hn.shape[0]):
            rows = [int(r) for r in ids[t]]
            valid = [(r, float(wt)) for r, wt in zip(rows, w[t]) if 0 <= r < len(rank_experts)]
            if valid:
                out[t] = O.moe_layer_ref(hn[t:t + 1], np.array([[r for r, _ in valid]]), np.array([[x for _, x in valid]]),
                                         lambda r: rank_experts[r], cb16, rot2048, rot512)[0]
        return torch.from_numpy(out.astype(np.float32))
    return ffn


def _router(logits, k, hidden=None, gate=None):
    ids, w = O.router_ref(logits.numpy(), k)
    ids_t, w_t = torch.from_numpy(ids), torch.from_numpy(w)
    if gate is None:
        return ids_t, w_t
    sw = 1 / (1 + np.exp(-(hidden.double().numpy() @ gate.double().numpy())))
    return ids_t, w_t, torch.from_numpy(sw.astype(np.float32))


def _worker(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cbs = _cbs()
        r2048, r512 = O.rot_params("moe_expert_2048", 2048), O.rot_params("moe_expert_512", 512)
        lo, hi = ep.partition(E, world, rank)
        experts = [synth.synth_expert(SEED, e) for e in range(lo, hi)]
        experts.append(synth.synth_expert(SEED + 1, 0))   # every rank holds the shared expert
        gate = torch.from_numpy((0.05 * np.random.default_rng(1).standard_normal(2048)).astype(np.float32))
        blk = ep.ExpertParallelMoEBlock(None, None, E, None, None, shared_gate=gate, top_k=K,
                                        ffn=_oracle_ffn_factory(experts, cbs["16"], r2048, r512), router=_router)
        h = torch.from_numpy(np.random.default_rng(2).standard_normal((T, 2048)).astype(np.float32))
        logits = torch.from_numpy(np.random.default_rng(3).standard_normal((T, E)).astype(np.float32))
        y = blk(h, logits)
        results[rank] = y.numpy()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_expert_parallel_matches_single_process(world):
    mgr = mp.get_context("spawn").Manager()
    results = mgr.dict()
    mp.start_processes(_worker, args=(world, _free_port(), results), nprocs=world, join=True, start_method="spawn")
    cbs = _cbs()
    r2048, r512 = O.rot_params("moe_expert_2048", 2048), O.rot_params("moe_expert_512", 512)
    h = np.random.default_rng(2).standard_normal((T, 2048)).astype(np.float32)
    logits = np.random.default_rng(3).standard_normal((T, E)).astype(np.float32)
    gate = (0.05 * np.random.default_rng(1).standard_normal(2048)).astype(np.float32)
    ids, w = O.router_ref(logits, K)
    sw = 1 / (1 + np.exp(-(h.astype(np.float64) @ gate.astype(np.float64))))
    ref = O.moe_layer_ref(h, ids, w, lambda e: synth.synth_expert(SEED, e), cbs["16"], r2048, r512,
                          shared=synth.synth_expert(SEED + 1, 0), shared_w=sw)
    for r in range(world):
        y = results[r]
        assert np.abs(y - ref).max() / np.abs(ref).max() < 1e-5, r
    assert np.array_equal(results[0], results[world - 1])


def test_partition_and_local_ids():
    assert ep.partition(256, 8, 3) == (96, 128)
    with pytest.raises(ValueError):
        ep.partition(256, 3, 0)
    ids = torch.tensor([[0, 5, 9, 15], [8, 7, 6, 12]])
    w = torch.rand(2, 4)
    loc, lw = ep.local_problems(ids, w, 8, 16, shared_id=8, shared_w=torch.tensor([0.3, 0.7]))
    assert loc.tolist() == [[-1, -1, 1, 7, 8], [0, -1, -1, 4, 8]]
    assert torch.allclose(lw[:, 4], torch.tensor([0.3, 0.7]))
    # the shared expert's problem of token t is local on rank t % world only
    ids3 = torch.tensor([[0, 9], [9, 1], [2, 12]])
    for rank in range(2):
        loc, _ = ep.local_problems(ids3, torch.rand(3, 2), 8 * rank, 8 * rank + 8, shared_id=8,
                                   shared_w=torch.rand(3), rank=rank, world=2)
        assert loc[:, 2].tolist() == [8 if t % 2 == rank else -1 for t in range(3)]


# ------------------------------------------------------------------------ a rank that leaves
def _leaving_worker(rank, world, port, results):
    """Step 0 runs on every rank; then the last rank leaves between steps (no collective of its
    in flight) and the others' next all_reduce must end with an error within the group timeout."""
    import datetime
    import time
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    # the group timeout also bounds rendezvous and step 0, which a loaded host can stretch (spawned
    # ranks import torch and run the fp64 stand-in); the leaving rank's closed connection is
    # reported to its peers at once, well inside it
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    cbs = _cbs()
    r2048, r512 = O.rot_params("moe_expert_2048", 2048), O.rot_params("moe_expert_512", 512)
    lo, hi = ep.partition(E, world, rank)
    experts = [synth.synth_expert(SEED, e) for e in range(lo, hi)]
    blk = ep.ExpertParallelMoEBlock(None, None, E, None, None, top_k=K,
                                    ffn=_oracle_ffn_factory(experts, cbs["16"], r2048, r512), router=_router)
    h = torch.from_numpy(np.random.default_rng(2).standard_normal((1, 2048)).astype(np.float32))
    lg = torch.from_numpy(np.random.default_rng(3).standard_normal((1, E)).astype(np.float32))
    blk(h, lg)
    if rank == world - 1:
        results[rank] = "left"
        return  # leaves without destroying the group: its peers must notice on their own
    t0 = time.time()
    try:
        blk(h, lg)
        results[rank] = "no error"
    except Exception as exc:  # gloo reports the lost peer / the timeout as a RuntimeError
        results[rank] = (type(exc).__name__, round(time.time() - t0, 1))


def test_rank_leaving_between_steps_is_detected_by_the_others():
    world = 4
    mgr = mp.get_context("spawn").Manager()
    results = mgr.dict()
    mp.start_processes(_leaving_worker, args=(world, _free_port(), results), nprocs=world, join=True,
                       start_method="spawn")
    assert results[world - 1] == "left"
    for r in range(world - 1):
        res = results[r]
        assert isinstance(res, tuple), (r, res)
        assert res[1] < 40, (r, res)   # ended by the error, not by hanging
