"""Context split across ranks (config C4) on CPU: the shard plans, and the whole protocol of
attention_lab_b200.context_split run on gloo ranks (world 2 and 4) with the oracle standing in for the kernels.

The orchestration under test is the product's own `context_split_decode_step` (plans, the two all-gathers, the
threshold, the partial attend and the merge); `OracleOps` gives it float64 numpy restatements of the four device
steps. The result must equal the single-device decode step of decode.py:145-163 on the unsplit caches: the same
top-k set (score desc, position asc) and the same attention output.
"""
from __future__ import annotations

import math
import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from attention_lab_b200 import context_split as csplit
from attention_lab_b200.selection import fixed_budget, selection_layout
from oracle import oracle as orc


@pytest.mark.parametrize("L,cap,world", [(1000, 1000, 2), (1000, 1000, 4), (1000, 2048, 4), (8193, 8448, 8),
                                         (131072, 131072, 2), (70, 70, 2)])
def test_shard_plans_partition_the_step(L, cap, world):
    k0 = fixed_budget(L, 1 / 32)
    lay = selection_layout(L)
    plans = [csplit.plan_shard(L, k0, r, world, cap) for r in range(world)]
    cands, fixed, owners = [], [], []
    for p in plans:
        assert p.start == p.rank * p.shard_capacity and p.shard_capacity % csplit.SHARD_ALIGN == 0
        cands += [p.start + c for c in range(p.lo, p.hi)]
        fixed += [p.start + c for c in p.fixed_local]
        assert p.k == lay.clamp_k(k0) and p.k_local == min(p.k, p.hi - p.lo)
        if p.write_col >= 0:
            owners.append(p.rank)
            assert p.start + p.write_col == L - 1
    assert cands == list(range(lay.candidate_lo, lay.candidate_hi))      # each candidate on exactly one shard, in order
    assert fixed == lay.fixed_positions()                                 # F in its global order
    assert len(owners) == 1                                               # one rank writes the new z column
    assert sum(p.k_local for p in plans) >= plans[0].k                   # the union holds the global top-k


def _order_key(s32: np.ndarray) -> np.ndarray:
    """float32 -> uint32 preserving order; NaN above +inf, -0 == +0 (the kernels' score key)."""
    u = s32.astype(np.float32).view(np.uint32).copy()
    u[s32 == 0] = 0
    key = np.where(u & 0x80000000, ~u, u | 0x80000000).astype(np.uint64)
    key[np.isnan(s32)] = 0xFFFFFFFF
    return key


def _scores32(u, zT, lo, hi):
    """float32 scores of columns [lo, hi), computed column by column (the same value on any shard)."""
    return (u[:, :, 0, :, None] * zT[:, :, :, lo:hi].astype(np.float64)).sum(axis=2).astype(np.float32)


class OracleOps:
    """The four device steps of context_split, restated on CPU (float64; partials in the natural-log domain)."""

    def __init__(self, wq_t):
        self.wq_t = wq_t

    def local_topk(self, q_pre, zT, wq_t_scaled, wk, plan, *, k_pre_new=None):
        B, G = q_pre.shape[:2]
        if k_pre_new is not None:       # the z column of the newest key (decode.py:156-157), owning shard only
            assert plan.write_col >= 0, "k_pre_new reached a shard that does not own position L - 1"
            zT[..., plan.write_col] = torch.from_numpy(orc.project_keys(k_pre_new.numpy(), wk.numpy())[..., 0])
        u = orc.project_queries(q_pre.numpy(), wq_t_scaled.numpy())
        s = _scores32(u, zT.numpy(), plan.lo, plan.hi)                       # [B,G,M_local]
        pos = plan.start + np.arange(plan.lo, plan.hi)
        keys = np.zeros((B, G, plan.k), dtype=np.uint64)
        rows = np.zeros((B, G, plan.selected_count), dtype=np.int64)
        for b in range(B):
            for g in range(G):
                off = (b * G + g) * plan.shard_capacity
                nan = np.isnan(s[b, g])
                order = np.lexsort((pos, -np.where(nan, 0.0, s[b, g]), ~nan))[:plan.k_local]
                chosen = np.sort(order)                                      # ascending position
                k64 = (_order_key(s[b, g][chosen]) << np.uint64(32)) | (np.uint64(0xFFFFFFFF) - pos[chosen].astype(np.uint64))
                keys[b, g, :plan.k_local] = k64
                rows[b, g, :plan.fixed_count] = off + np.array(plan.fixed_local, dtype=np.int64)
                rows[b, g, plan.fixed_count:] = off + plan.lo + chosen
        return torch.from_numpy(rows), torch.from_numpy(keys.view(np.int64))

    def threshold(self, all_keys, rows, plan):
        keys = all_keys.numpy().view(np.uint64)                              # [world,B,G,k]
        out = rows.numpy().copy()
        _, B, G, _ = keys.shape
        for b in range(B):
            for g in range(G):
                tau = np.sort(keys[:, b, g, :].ravel())[::-1][plan.k - 1]
                mine = keys[plan.rank, b, g, :plan.k_local]
                out[b, g, plan.fixed_count:][mine < tau] = -1
        return torch.from_numpy(out)

    def attend_partial(self, q_main, k_cache, v_cache, rows, scale):
        B, G, h, _, d = q_main.shape
        kf = k_cache.numpy().reshape(-1, d)
        vf = v_cache.numpy().reshape(-1, d)
        part = np.zeros((B, G, h, d + 2))
        r = rows.numpy().reshape(B, G, -1)
        for b in range(B):
            for g in range(G):
                sel = r[b, g][r[b, g] >= 0]
                m, l, acc = orc.partial_attention(q_main.numpy()[b, g, :, 0, :], kf[sel], vf[sel], scale)
                part[b, g, :, 0], part[b, g, :, 1], part[b, g, :, 2:] = m, l, acc
        return torch.from_numpy(part)

    def lse_merge(self, all_parts, dtype):
        p = all_parts.numpy()
        W, B, G, h, d2 = p.shape
        out = np.zeros((B, G, h, 1, d2 - 2))
        for b in range(B):
            for g in range(G):
                out[b, g, :, 0, :] = orc.lse_merge(p[:, b, g, :, 0], p[:, b, g, :, 1], p[:, b, g, :, 2:])
        return torch.from_numpy(out)


def _problem(seed, B, G, h, d, r, C, L, mirror=False):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((B, G, h, 1, d))
    q_pre = rng.standard_normal((B, G, h, 1, d))
    K = rng.standard_normal((B, G, C, d))
    V = rng.standard_normal((B, G, C, d))
    zT = rng.standard_normal((B, G, r, C)).astype(np.float32)
    zT[..., 700:720] = zT[..., 100:120]               # exact score ties across shards
    if mirror:                                        # every score has a twin half a sequence later
        zT[..., L // 2:L] = zT[..., :L - L // 2]
    wq_t = (rng.standard_normal((G, h * d, r)) * 0.02).astype(np.float32)
    wk = (rng.standard_normal((G, r, d)) * 0.02).astype(np.float32)
    k_pre_new = rng.standard_normal((B, G, 1, d)).astype(np.float32)
    return q, q_pre, K, V, zT, wq_t, wk, k_pre_new


def _single_device(q, q_pre, K, V, zT, wq_t, L, k0):
    """decode.py:145-163 on the unsplit caches with float32 scores, ties to the smaller position."""
    lay = selection_layout(L)
    k = lay.clamp_k(k0)
    u = orc.project_queries(q_pre, wq_t)
    s = _scores32(u, zT, lay.candidate_lo, lay.candidate_hi)
    B, G = q.shape[:2]
    out = np.zeros(q.shape)
    chosen_all = []
    for b in range(B):
        for g in range(G):
            top = orc.topk_indices(s[b, g].astype(np.float64)[None], k)[0] + lay.candidate_lo
            chosen_all.append(sorted(top.tolist()))
            sel = np.array(lay.fixed_positions() + sorted(top.tolist()))
            out[b, g] = orc.subset_attention(q[b:b + 1, g:g + 1], K[b:b + 1, g:g + 1, sel], V[b:b + 1, g:g + 1, sel],
                                             1 / math.sqrt(q.shape[-1]))[0, 0]
    return out, chosen_all


def _worker(rank, world, port, cap, L, mirror, result_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        B, G, h, d, r = 1, 2, 2, 128, 32
        q, q_pre, K, V, zT, wq_t, wk, k_pre_new = _problem(7, B, G, h, d, r, cap, L, mirror)
        k0 = fixed_budget(L, 1 / 16)
        plan = csplit.plan_shard(L, k0, rank, world, cap)
        cs_, st = plan.shard_capacity, plan.start
        pad = cs_ * world - cap

        def shard(x, axis):
            x = np.concatenate([x, np.zeros(x.shape[:axis] + (pad,) + x.shape[axis + 1:], x.dtype)], axis=axis)
            return torch.from_numpy(np.ascontiguousarray(np.take(x, range(st, st + cs_), axis=axis)))
        ops = OracleOps(wq_t)
        z_shard = shard(zT, 3)
        # every rank passes the newest key; the protocol lets only the owner of position L - 1 write its z column
        out = csplit.context_split_decode_step(torch.from_numpy(q), torch.from_numpy(q_pre), shard(K, 2), shard(V, 2),
                                               z_shard, torch.from_numpy(wq_t), torch.from_numpy(wk), plan, ops=ops,
                                               k_pre_new=torch.from_numpy(k_pre_new), scale=1 / math.sqrt(d))
        np.save(os.path.join(result_dir, f"out{rank}.npy"), out.numpy())
        np.save(os.path.join(result_dir, f"z{rank}.npy"), z_shard.numpy())
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world,cap,L,mirror", [(2, 1000, 1000, False), (2, 1000, 1000, True),
                                                (4, 2048, 1000, False), (4, 2048, 1000, True)])
def test_context_split_on_gloo_ranks_equals_single_device(world, cap, L, mirror, tmp_path):
    """world-size gloo ranks run the product orchestration; every rank's output equals the single-device step
    (world 4 with capacity 2048 leaves two ranks past the legal range, holding nothing; `mirror` makes every
    selection a tie decided by position across shards)."""
    mp.spawn(_worker, args=(world, _free_port(), cap, L, mirror, str(tmp_path)), nprocs=world, join=True)
    q, q_pre, K, V, zT, wq_t, wk, k_pre_new = _problem(7, 1, 2, 2, 128, 32, cap, L, mirror)
    want, _ = _single_device(q, q_pre, K, V, zT, wq_t, L, fixed_budget(L, 1 / 16))
    z_new = orc.project_keys(k_pre_new, wk)[..., 0].astype(np.float32)        # [B,G,r]
    for rank in range(world):
        got = np.load(tmp_path / f"out{rank}.npy")
        assert np.abs(got - want).max() < 1e-10, f"rank {rank}"
        plan = csplit.plan_shard(L, fixed_budget(L, 1 / 16), rank, world, cap)
        z_got = np.load(tmp_path / f"z{rank}.npy")
        z_orig = np.concatenate([zT, np.zeros(zT.shape[:3] + (plan.shard_capacity * world - cap,), zT.dtype)],
                                axis=3)[..., plan.start:plan.start + plan.shard_capacity]
        changed = np.nonzero((z_got != z_orig).any(axis=(0, 1, 2)))[0].tolist()
        if plan.write_col >= 0:
            assert changed in ([plan.write_col], []) and np.array_equal(z_got[..., plan.write_col], z_new)
        else:
            assert changed == [], f"rank {rank} does not own position L - 1 but changed its index table"
