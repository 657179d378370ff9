"""GPU tests of the context split's peer exchange (al_xchg_*, al_context_threshold_peer, al_lse_merge_peer): the two
all-gathers of the C4 protocol replaced by pushes into every rank's gather area over NVLink, epoch flags stored into
the peers' regions, and consumers that wait for the flags and read their own gather area.

- one rank: the step through a PeerExchange equals the step without one, bit for bit;
- a wait whose flag nothing sets gives up after its poll limit, sets error bit 2 and leaves the context usable;
- two GPUs (when present): the peer path equals the NCCL path bit for bit on consecutive steps, launched eagerly and
  replayed from a captured CUDA graph (the epoch counters advance on the device).
"""
from __future__ import annotations

import os
from datetime import timedelta

import numpy as np
import pytest
import torch

from test_gpu_context import _free_port, _inputs

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _shard(t, plan):
    cs_ = plan.shard_capacity
    sl = lambda x, dim: x.narrow(dim, plan.start, cs_).contiguous()
    return sl(t["k"], 2), sl(t["v"], 2), sl(t["zT"], 3)


def test_peer_exchange_on_one_rank_equals_the_plain_step():
    from attention_lab_b200 import context_split as csplit
    from attention_lab_b200.selection import fixed_budget
    L = cap = 8192
    t = _inputs(1, 8, 4, cap, L, seed=3)
    plan = csplit.plan_shard(L, fixed_budget(L, 1 / 32), 0, 1, cap)
    K, V, Z = _shard(t, plan)
    Z2 = Z.clone()
    want = csplit.context_split_decode_step(t["q"], t["q_pre"], K, V, Z, t["wq_t"], t["wk"], plan,
                                            k_pre_new=t["k_pre_new"])
    x = csplit.PeerExchange(1, 8, plan.k, 4, device=DEV)
    try:
        for _ in range(2):
            got = csplit.context_split_decode_step(t["q"], t["q_pre"], K, V, Z2, t["wq_t"], t["wk"], plan,
                                                   k_pre_new=t["k_pre_new"], exchange=x)
            torch.cuda.synchronize()
            assert torch.equal(got, want)
        assert torch.equal(Z2, Z), "the z column must be written the same way"
    finally:
        x.close()


def test_a_wait_on_a_flag_nothing_sets_gives_up_with_an_error_bit():
    """Two ranks' tables on one GPU, both entries this process's own region: this rank pushes (its counter reaches 1)
    but 'rank 1' never does, so the consumers' waits run out after `spin` polls."""
    from attention_lab_b200 import _lib, ops
    B, G, k, h, d = 1, 2, 64, 4, 128
    base, _ = ops.xchg_create(1 << 20, DEV)
    try:
        _lib.device_status()                                   # clear earlier bits
        flags, counter, done = base, base + 512, base + 520
        peer_flags = torch.tensor([base, base], dtype=torch.int64, device=DEV)
        gkeys = ops.device_view(base + 4096, (2, B, G, k), torch.int64, DEV)
        dst = torch.tensor([base + 4096, base + 4096], dtype=torch.int64, device=DEV)
        ops.xchg_push(torch.ones(B, G, k, dtype=torch.int64, device=DEV), dst, 0, done, counter, peer_flags)
        torch.cuda.synchronize()
        assert int(gkeys[0].sum()) == B * G * k and int(gkeys[1].sum()) == 0, "the push fills slot 0 only"
        rows = torch.arange(B * G * k, dtype=torch.int64, device=DEV).view(B, G, k)
        ops.context_threshold_peer(gkeys, flags, counter, rows, 0, k, 0, k, spin=200)
        assert _lib.device_status() & 2, "the threshold wait must give up and flag it"
        gparts = ops.device_view(base + 65536, (2, B, G, h, d + 2), torch.float32, DEV)
        ops.lse_merge_peer(gparts, flags, counter, 0, torch.float32, spin=200)
        assert _lib.device_status() & 2, "the merge wait must give up and flag it"
        x = torch.ones(1000, device=DEV)                       # the context is still usable
        assert float((x * 2).sum()) == 2000.0
        assert _lib.device_status() == 0
    finally:
        ops.xchg_destroy(base, DEV)


def _xchg_worker(rank, world, port, L, cap, result_dir):
    import torch.distributed as dist
    from attention_lab_b200 import context_split as csplit
    from attention_lab_b200.selection import fixed_budget
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    x = None
    try:
        plan = csplit.plan_shard(L, fixed_budget(L, 1 / 32), rank, world, cap)
        x = csplit.PeerExchange(1, 8, plan.k, 4, device=dev)
        res = {}
        for step in range(3):                                 # consecutive steps: the epochs advance
            t = _inputs(1, 8, 4, cap, L, seed=11 + step, device=dev)
            K, V, Z = _shard(t, plan)
            Z2 = Z.clone()
            a = csplit.context_split_decode_step(t["q"], t["q_pre"], K, V, Z, t["wq_t"], t["wk"], plan,
                                                 k_pre_new=t["k_pre_new"])
            b = csplit.context_split_decode_step(t["q"], t["q_pre"], K, V, Z2, t["wq_t"], t["wk"], plan,
                                                 k_pre_new=t["k_pre_new"], exchange=x)
            torch.cuda.synchronize()
            res[f"nccl{step}"], res[f"peer{step}"] = a.float().cpu().numpy(), b.float().cpu().numpy()
            res[f"z{step}"] = bool(torch.equal(Z, Z2))
        # a captured step replayed twice (fresh epochs on the device each time) equals the eager step
        t = _inputs(1, 8, 4, cap, L, seed=21, device=dev)
        K, V, Z = _shard(t, plan)
        eager = csplit.context_split_decode_step(t["q"], t["q_pre"], K, V, Z, t["wq_t"], t["wk"], plan, exchange=x)
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            dist.barrier()
            torch.cuda.synchronize()
            with torch.cuda.graph(g, stream=s):
                out = csplit.context_split_decode_step(t["q"], t["q_pre"], K, V, Z, t["wq_t"], t["wk"], plan,
                                                       exchange=x)
        torch.cuda.current_stream(dev).wait_stream(s)
        reps = []
        for _ in range(2):
            torch.cuda.synchronize()
            dist.barrier()
            g.replay()
            torch.cuda.synchronize()
            reps.append(bool(torch.equal(out, eager)))
        res["graph"] = reps
        del g
        np.save(os.path.join(result_dir, f"xchg{rank}.npy"), np.array([res], dtype=object), allow_pickle=True)
    finally:
        torch.cuda.synchronize()
        if x is not None:
            x.close()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_peer_exchange_on_two_gpus_equals_the_nccl_path(tmp_path):
    import torch.multiprocessing as mp
    L = cap = 16384
    mp.spawn(_xchg_worker, args=(2, _free_port(), L, cap, str(tmp_path)), nprocs=2, join=True)
    for rank in range(2):
        res = np.load(tmp_path / f"xchg{rank}.npy", allow_pickle=True)[0]
        for step in range(3):
            assert np.array_equal(res[f"peer{step}"], res[f"nccl{step}"]), f"rank {rank} step {step}"
            assert res[f"z{step}"], f"rank {rank} step {step}: z column"
        assert res["graph"] == [True, True], f"rank {rank}: graph replays {res['graph']}"
