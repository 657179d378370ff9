"""GPU tests of the context split (config C4) through the C ABI: al_context_local_topk, al_context_threshold,
al_gathered_attend_partial and al_lse_merge.

Ranks are emulated on one GPU (each shard's caches are separate tensors; the all-gathers become stacks), and the
result is compared with the single-device fused step on the unsplit caches: the kept rows must be exactly the fused
kernel's rows (the same fp32 scores, the same (score desc, position asc) order), the z column written by the owning
shard must equal the fused kernel's, and the merged output must match within the bf16 tolerance of tests/parity.py.
A second test runs the real orchestration (NCCL all-gathers) on two GPUs when the machine has them.
"""
from __future__ import annotations

import math
import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch

from oracle import oracle as orc
from parity import check_out, check_topk_float64

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _inputs(B, G, h, C, L, seed, mirror=False, device=DEV):
    gen = torch.Generator().manual_seed(seed)
    d, r = 128, 32
    bf = torch.bfloat16
    t = dict(
        q=torch.randn(B, G, h, 1, d, generator=gen).to(bf),
        q_pre=torch.randn(B, G, h, 1, d, generator=gen).to(bf),
        k=torch.randn(B, G, C, d, generator=gen).to(bf),
        v=torch.randn(B, G, C, d, generator=gen).to(bf),
        zT=(torch.randn(B, G, r, C, generator=gen) * 0.25).to(bf),
        wq_t=(torch.randn(G, h * d, r, generator=gen) * 0.004).to(bf),
        wk=(torch.randn(G, r, d, generator=gen) * 0.02).to(bf),
        k_pre_new=torch.randn(B, G, 1, d, generator=gen).to(bf),
    )
    if mirror:                                   # every candidate score has a twin half a sequence later
        t["zT"][..., L // 2:L - 1] = t["zT"][..., : L - 1 - L // 2]
    return {k_: v_.to(device) for k_, v_ in t.items()}


def _fused(t, L, k0):
    import attention_lab_b200 as al
    from attention_lab_b200.selection import build_step_plan
    B, G, C = t["k"].shape[0], t["k"].shape[1], t["k"].shape[2]
    plan = build_step_plan(B, G, C, L, k0, t["k"].device)
    zT = t["zT"].clone()
    out, rows = al.sparse_decode_step_kernel(t["q"], t["q_pre"], t["k"], t["v"], zT, t["wq_t"], t["wk"], plan.fixed_rows,
                                             plan.off_lo, plan.lo, plan.hi, plan.k, plan.selected_count,
                                             k_pre_new=t["k_pre_new"], write_col=plan.write_col, return_rows=True)
    pos = (rows.view(B, G, -1) - (torch.arange(B * G, device=rows.device) * C).view(B, G, 1)).cpu().numpy()
    return out, pos, zT


def _emulate(t, L, k0, world, cap):
    """Every rank's device steps on one GPU; returns (merged out, kept global positions [B][G] sets, zT shards)."""
    from attention_lab_b200 import context_split as csplit
    from attention_lab_b200 import ops
    B, G, h = t["q"].shape[:3]
    plans = [csplit.plan_shard(L, k0, r, world, cap) for r in range(world)]
    cs_ = plans[0].shard_capacity
    pad = cs_ * world - t["k"].shape[2]

    def shard(x, dim, p):
        if pad:
            x = torch.cat([x, torch.zeros(x.shape[:dim] + (pad,) + x.shape[dim + 1:], dtype=x.dtype, device=x.device)], dim)
        return x.narrow(dim, p.start, cs_).contiguous()
    loc = []
    for p in plans:
        K, V, zT = shard(t["k"], 2, p), shard(t["v"], 2, p), shard(t["zT"], 3, p)
        if p.selected_count > 0:
            rows, keys = csplit.CudaContextOps.local_topk(t["q_pre"], zT, t["wq_t"], t["wk"], p,
                                                          k_pre_new=t["k_pre_new"])     # gated by the plan
        else:
            rows = torch.empty(B, G, 0, dtype=torch.int64, device=DEV)
            keys = torch.zeros(B, G, p.k, dtype=torch.int64, device=DEV)
        loc.append((p, K, V, zT, rows, keys))
    all_keys = torch.stack([x[5] for x in loc]).contiguous()
    parts, kept = [], [[set() for _ in range(G)] for _ in range(B)]
    for p, K, V, zT, rows, _ in loc:
        if p.selected_count > 0:
            rows = csplit.CudaContextOps.threshold(all_keys, rows, p)
        parts.append(csplit.CudaContextOps.attend_partial(t["q"], K, V, rows, None))
        rr = rows.cpu().numpy()
        for b in range(B):
            for g in range(G):
                x = rr[b, g]
                x = x[x >= 0] - (b * G + g) * cs_
                kept[b][g] |= set((x + p.start).tolist())
    out = ops.lse_merge(torch.stack(parts).contiguous(), t["q"].dtype)
    torch.cuda.synchronize()
    return out, kept, [x[3] for x in loc], plans


def _oracle_out(t, pos):
    B, G = pos.shape[:2]
    q = t["q"].float().cpu().numpy()
    K, V = t["k"].float().cpu().numpy(), t["v"].float().cpu().numpy()
    out = np.zeros(q.shape)
    for b in range(B):
        for g in range(G):
            sel = np.sort(pos[b, g])
            out[b, g] = orc.subset_attention(q[b:b + 1, g:g + 1], K[b:b + 1, g:g + 1, sel], V[b:b + 1, g:g + 1, sel],
                                             1 / math.sqrt(128))[0, 0]
    return out


@pytest.mark.parametrize("world,cap,L,mirror", [(2, 8192, 8192, False), (4, 8192, 8192, False),
                                                (2, 8192, 8192, True), (4, 12288, 8192, False),
                                                (8, 4096, 3600, False)])
def test_context_split_kernels_equal_the_fused_step(world, cap, L, mirror):
    """(4, 12288, 8192): the last rank lies past the legal range; (8, 4096, 3600): F's recent window [3536, 3600)
    straddles the last shard boundary, so the last shard holds F rows and no candidate (k_local = 0)."""
    from attention_lab_b200 import _lib
    from attention_lab_b200.selection import fixed_budget, selection_layout
    k0 = fixed_budget(L, 1 / 32)
    t = _inputs(2, 8, 4, cap, L, seed=world * 10 + int(mirror), mirror=mirror)
    out_f, pos_f, zT_f = _fused(t, L, k0)
    out_c, kept, zT_sh, plans = _emulate(t, L, k0, world, cap)
    assert _lib.device_status() == 0
    B, G = 2, 8
    for b in range(B):
        for g in range(G):
            assert kept[b][g] == set(pos_f[b, g].tolist()), f"segment ({b},{g})"
    # the fused rows (and so the kept rows) against the float64 oracle's top-k of the same inputs
    lay = selection_layout(L)
    f64 = lambda x: x.double().cpu().numpy()
    u64 = orc.project_queries(f64(t["q_pre"]), f64(t["wq_t"]))
    s64 = orc.candidate_scores(u64, f64(t["zT"]), lay.candidate_lo, lay.candidate_hi)[:, :, 0, :]
    check_topk_float64(pos_f[..., lay.fixed_count:] - lay.candidate_lo, s64, lay.clamp_k(k0), "split top-k")
    # the newest key's z column, written by the shard that owns position L-1
    owner = [p for p in plans if p.write_col >= 0][0]
    zc = zT_sh[owner.rank][..., owner.write_col]
    assert torch.equal(zc.view(torch.int16), zT_f[..., L - 1].view(torch.int16))
    want = _oracle_out(t, pos_f)
    check_out(out_c.float().cpu().numpy(), want, "bfloat16", "merged out")
    check_out(out_f.float().cpu().numpy(), want, "bfloat16", "fused out")


def test_partial_and_merge_edge_cases():
    """A partial over no rows (all skipped) is empty and the merge ignores it; merging one partial normalises it."""
    from attention_lab_b200 import ops
    t = _inputs(1, 2, 2, 256, 256, seed=3)
    rows = torch.full((1, 2, 5), -1, dtype=torch.int64, device=DEV)
    empty = ops.gathered_attend_partial(t["q"], t["k"], t["v"], rows)
    assert torch.isinf(empty[..., 0]).all() and (empty[..., 1] == 0).all() and (empty[..., 2:] == 0).all()
    rows2 = torch.arange(0, 10, device=DEV).view(1, 1, 10).repeat(1, 2, 1) + torch.tensor([0, 256], device=DEV).view(1, 2, 1)
    full = ops.gathered_attend_partial(t["q"], t["k"], t["v"], rows2.contiguous())
    out = ops.lse_merge(torch.stack([empty, full, empty]).contiguous(), torch.float32)
    ref = ops.gathered_decode_step_kernel(t["q"], t["k"], t["v"], rows2.reshape(-1), 10)
    assert torch.allclose(out.float(), ref.float(), atol=2e-2, rtol=2e-2)
    with pytest.raises(ValueError):
        ops.context_threshold(torch.zeros(2, 1, 2, 4, dtype=torch.int64, device=DEV), rows, 2, 4, 1, 4)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, world, port, L, cap, result_dir):
    import torch.distributed as dist
    from attention_lab_b200 import context_split as csplit
    from attention_lab_b200.selection import fixed_budget
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        t = _inputs(1, 8, 4, cap, L, seed=5, device=dev)
        plan = csplit.plan_shard(L, fixed_budget(L, 1 / 32), rank, world, cap)
        cs_ = plan.shard_capacity
        sl = lambda x, dim: x.narrow(dim, plan.start, cs_).contiguous()
        out = csplit.context_split_decode_step(t["q"], t["q_pre"], sl(t["k"], 2), sl(t["v"], 2), sl(t["zT"], 3),
                                               t["wq_t"], t["wk"], plan, k_pre_new=t["k_pre_new"])
        torch.cuda.synchronize()
        np.save(os.path.join(result_dir, f"out{rank}.npy"), out.float().cpu().numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_context_split_on_two_gpus_equals_the_fused_step(tmp_path):
    import torch.multiprocessing as mp
    from attention_lab_b200.selection import fixed_budget
    L = cap = 32768
    mp.spawn(_nccl_worker, args=(2, _free_port(), L, cap, str(tmp_path)), nprocs=2, join=True)
    t = _inputs(1, 8, 4, cap, L, seed=5)
    out_f, pos_f, _ = _fused(t, L, fixed_budget(L, 1 / 32))
    want = _oracle_out(t, pos_f)
    for rank in range(2):
        got = np.load(tmp_path / f"out{rank}.npy")
        check_out(got, want, "bfloat16", f"rank {rank}")
