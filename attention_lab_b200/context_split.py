"""Context split of one decode step across the ranks of a process group (config C4: one long sequence, one GPU per
contiguous shard of its positions).

attention-lab's decode step (decode.py:145-163) runs on one device. Split across P ranks, each rank holds positions
[start, start + shard_capacity) of every cache (K, V, zT) and, per layer:

    1. scores its own candidates and takes a local top-k (a 64-bit key per candidate: the score's order key above
       the inverted position, so (score desc, position asc) is plain integer order and no two candidates tie);
    2. all-gathers the keys (P * k * 8 bytes per (batch, group));
    3. finds the global k-th key and keeps its candidates at or above it: exactly the single-device top-k set;
    4. attends over F's rows on its shard plus its kept candidates into an unnormalised partial (m, l, acc);
    5. all-gathers the partials (P * h * 130 floats per (batch, group)) and merges them by log-sum-exp.

Every rank ends with the same output. F's prefix lives on the first shard, its recent window on the shard(s) that
hold the last positions; the newest key's z column is written by the shard that owns position L - 1.

The device work goes through an `ops` object (default: `CudaContextOps`, the sm_100a kernels). Tests hand the same
orchestration CPU stand-ins to check the protocol over gloo ranks; the CUDA path itself has no CPU fallback.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch
import torch.distributed as dist

from . import ops as _ops
from .selection import row_offsets, selection_layout

SHARD_ALIGN = 16   # positions; keeps every shard's zT rows 16-byte aligned for the vector scan


@dataclass(frozen=True)
class ShardPlan:
    """One rank's view of a decode step whose legal range is [0, legal_length)."""

    rank: int
    world: int
    legal_length: int
    k: int                      # global top-k size (selection.py rules)
    start: int                  # global position of local column 0
    shard_capacity: int         # positions held per rank
    lo: int                     # local candidate columns [lo, hi)
    hi: int
    fixed_local: tuple          # local columns of F on this shard (global F order)
    k_local: int                # min(k, hi - lo)
    _dev: dict = field(default_factory=dict, compare=False, repr=False)   # device tensors, built once per shape

    @property
    def fixed_count(self) -> int:
        return len(self.fixed_local)

    @property
    def selected_count(self) -> int:
        return self.fixed_count + self.k_local

    @property
    def write_col(self) -> int:
        """Local column of position legal_length - 1, or -1 when another shard owns it."""
        c = self.legal_length - 1 - self.start
        return c if 0 <= c < self.shard_capacity else -1

    def fixed_rows(self, batch: int, groups: int, device) -> torch.Tensor:
        key = ("fixed", batch, groups, str(device))
        if key not in self._dev:
            off = row_offsets(batch, groups, self.shard_capacity, device)
            pos = torch.tensor(self.fixed_local, dtype=torch.long, device=device).view(1, 1, -1)
            self._dev[key] = (pos + off).contiguous()
        return self._dev[key]

    def off_lo(self, batch: int, groups: int, device) -> torch.Tensor:
        key = ("off_lo", batch, groups, str(device))
        if key not in self._dev:
            self._dev[key] = (row_offsets(batch, groups, self.shard_capacity, device) + self.lo).contiguous()
        return self._dev[key]


def shard_capacity(capacity: int, world: int) -> int:
    """Positions per rank: an equal, aligned share of the global capacity."""
    if world < 1:
        raise ValueError("world must be >= 1")
    per = -(-capacity // world)
    return -(-per // SHARD_ALIGN) * SHARD_ALIGN


def plan_shard(legal_length: int, k0: int, rank: int, world: int, capacity: int) -> ShardPlan:
    """The selection rules of selection.py:21-86 for the whole sequence, restricted to rank's shard."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside [0, {world})")
    cs = shard_capacity(capacity, world)
    if legal_length > cs * world:
        raise ValueError(f"legal length {legal_length} exceeds the shards' capacity {cs * world}")
    lay = selection_layout(legal_length)
    k = lay.clamp_k(k0)
    start, end = rank * cs, (rank + 1) * cs
    lo = min(max(lay.candidate_lo, start), end) - start
    hi = max(min(lay.candidate_hi, end), start) - start
    hi = max(hi, lo)
    fixed = tuple(p - start for p in lay.fixed_positions() if start <= p < end)
    return ShardPlan(rank=rank, world=world, legal_length=int(legal_length), k=int(k), start=start,
                     shard_capacity=cs, lo=lo, hi=hi, fixed_local=fixed, k_local=min(int(k), hi - lo))


class CudaContextOps:
    """The four device steps on the sm_100a kernels (C ABI entries al_context_local_topk, al_context_threshold,
    al_gathered_attend_partial, al_lse_merge)."""

    @staticmethod
    def local_topk(q_pre, zT, wq_t_scaled, wk, plan: ShardPlan, *, k_pre_new=None):
        B, G = q_pre.shape[:2]
        dev = q_pre.device
        return _ops.context_local_topk(q_pre, zT, wq_t_scaled, wk, plan.fixed_rows(B, G, dev), plan.off_lo(B, G, dev),
                                       plan.lo, plan.hi, plan.k_local, key_pos=plan.start, key_stride=plan.k,
                                       k_pre_new=k_pre_new if plan.write_col >= 0 else None,
                                       write_col=plan.write_col)

    @staticmethod
    def threshold(all_keys, rows, plan: ShardPlan):
        return _ops.context_threshold(all_keys, rows, plan.rank, plan.k, plan.fixed_count, plan.k_local)

    @staticmethod
    def attend_partial(q_main, k_cache, v_cache, rows, scale):
        return _ops.gathered_attend_partial(q_main, k_cache, v_cache, rows, scale=scale)

    @staticmethod
    def lse_merge(all_parts, dtype):
        return _ops.lse_merge(all_parts, dtype)


class PeerExchange:
    """The protocol's two exchanges over peer memory instead of NCCL all-gathers.

    Every rank allocates one region on its GPU (`ops.xchg_create`), the 64-byte CUDA IPC handles travel once over the
    process group (`all_gather_object`), and every rank maps the others' regions (`ops.xchg_open`). Region layout: a
    header with, per channel (0: keys, 1: partials), a flag word per rank (written by that rank, over NVLink), an epoch
    counter and a done counter; then this rank's keys [B,G,k] and partials [B,G,h,d+2], and per channel a gather area
    with one slot per rank. Per layer a rank writes its keys, pushes them into its slot of every rank's gather area
    (`ops.xchg_push`: remote stores, then the epoch flags), and the threshold kernel waits for every peer's flag and
    reads its own gather area; the same for the partials and the merge. Waits are bounded (`spin` polls of a flag); a
    wait that gives up sets error bit 2 (`_lib.device_status`). Collective: every rank constructs it with the same
    shapes, and `close()` on every rank releases it."""

    FLAGS = 256          # bytes per channel's flag array (64 ranks)

    def __init__(self, B: int, G: int, k: int, h: int, d: int = 128, *, group=None, device=None, spin: int = 1 << 22):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if self.world > 64:
            raise ValueError("at most 64 ranks")
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.shape = (int(B), int(G), int(k), int(h), int(d))
        self.spin = int(spin)
        keys_b, parts_b = B * G * k * 8, B * G * h * (d + 2) * 4
        al = lambda x: (x + 255) // 256 * 256
        self.keys_off = 1024
        self.parts_off = al(self.keys_off + keys_b)
        self.gkeys_off = al(self.parts_off + parts_b)
        self.gparts_off = al(self.gkeys_off + self.world * keys_b)
        nbytes = self.gparts_off + self.world * parts_b
        self.base, handle = _ops.xchg_create(nbytes, self.device)
        handles = [None] * self.world
        if self.world > 1:
            dist.all_gather_object(handles, handle, group=group)
        else:
            handles[0] = handle
        self.peers = [self.base if q == self.rank else _ops.xchg_open(handles[q], self.device) for q in range(self.world)]
        dev = self.device
        tab = lambda off: torch.tensor([b + off for b in self.peers], dtype=torch.int64, device=dev)
        self.peer_flags = [tab(0), tab(self.FLAGS)]               # channel c's flag arrays on every rank
        self.peer_gather = [tab(self.gkeys_off), tab(self.gparts_off)]
        self.flags = [self.base, self.base + self.FLAGS]         # this rank's flag arrays
        self.counters = [self.base + 2 * self.FLAGS, self.base + 2 * self.FLAGS + 4]
        self.done = [self.base + 2 * self.FLAGS + 8, self.base + 2 * self.FLAGS + 12]
        self.keys = _ops.device_view(self.base + self.keys_off, (B, G, k), torch.int64, dev)
        self.parts = _ops.device_view(self.base + self.parts_off, (B, G, h, d + 2), torch.float32, dev)
        self.gather_keys = _ops.device_view(self.base + self.gkeys_off, (self.world, B, G, k), torch.int64, dev)
        self.gather_parts = _ops.device_view(self.base + self.gparts_off, (self.world, B, G, h, d + 2), torch.float32,
                                             dev)

    def push(self, channel: int) -> None:
        src = self.keys if channel == 0 else self.parts
        _ops.xchg_push(src, self.peer_gather[channel], self.rank, self.done[channel], self.counters[channel],
                       self.peer_flags[channel])

    def close(self) -> None:
        """Collective: unmap the peers' regions, wait for every rank to have done the same, then free this rank's
        region (synchronises the device first)."""
        if self.base is None:
            return
        torch.cuda.synchronize(self.device)
        for q, ptr in enumerate(self.peers):
            if q != self.rank:
                _ops.xchg_close(ptr, self.device)
        if self.world > 1:
            dist.barrier(group=self.group)
        _ops.xchg_destroy(self.base, self.device)
        self.base, self.peers = None, []


def _all_gather(t: torch.Tensor, world: int, group) -> torch.Tensor:
    if world == 1:
        return t.unsqueeze(0).contiguous()
    t = t.contiguous()
    buf = torch.empty((world * t.shape[0],) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
    dist.all_gather_into_tensor(buf, t, group=group)            # one call, ranks concatenated along dim 0
    return buf.view((world,) + tuple(t.shape))


def context_split_decode_step(q_main, q_pre, k_cache, v_cache, zT, wq_t_scaled, wk, plan: ShardPlan, *,
                              group=None, k_pre_new=None, scale=None, ops=None, exchange: PeerExchange | None = None):
    """One layer's sparse decode step with the sequence split over the group's ranks (this rank holds the shard of
    `plan`: caches [B,G,shard_capacity,d] and zT [B,G,r,shard_capacity]). Every rank calls it with the same global
    step and gets the full output [B,G,h,1,d]; it equals decode.py:145-163 run on the unsplit caches. `k_pre_new`
    ([B,G,1,d], the newest key before RoPE) may be given on every rank: the rank whose shard holds position
    legal_length - 1 writes its index column, the others ignore it. With `exchange` (a PeerExchange of this group and
    shape) the keys and partials move over peer memory instead of NCCL all-gathers."""
    if exchange is not None:
        return _peer_step(q_main, q_pre, k_cache, v_cache, zT, wq_t_scaled, wk, plan, exchange, k_pre_new, scale)
    ops = CudaContextOps if ops is None else ops
    world = plan.world
    if world > 1 and dist.get_world_size(group) != world:
        raise ValueError(f"plan is for {world} ranks, the group has {dist.get_world_size(group)}")
    B, G, h, _, d = q_main.shape
    # every rank may pass the newest key's pre-RoPE features; only the shard that owns position L - 1 writes its z
    kpn = k_pre_new if plan.write_col >= 0 else None
    if plan.selected_count > 0:
        rows, keys = ops.local_topk(q_pre, zT, wq_t_scaled, wk, plan, k_pre_new=kpn)
    else:   # a shard past the legal range: nothing to score, nothing to attend
        rows = torch.empty((B, G, 0), dtype=torch.int64, device=q_main.device)
        keys = torch.zeros((B, G, plan.k), dtype=torch.int64, device=q_main.device)
    if plan.k > 0:   # the same on every rank
        all_keys = _all_gather(keys, world, group)
        if plan.selected_count > 0:
            rows = ops.threshold(all_keys, rows, plan)
    part = ops.attend_partial(q_main, k_cache, v_cache, rows, scale)
    all_parts = _all_gather(part, world, group)
    return ops.lse_merge(all_parts, q_main.dtype)


def _peer_step(q_main, q_pre, k_cache, v_cache, zT, wq_t_scaled, wk, plan: ShardPlan, x: PeerExchange, k_pre_new,
               scale):
    """context_split_decode_step with the exchanges over peer memory (the same kernels around them)."""
    B, G, h, _, d = q_main.shape
    if x.world != plan.world or x.shape != (B, G, plan.k, h, d):
        raise ValueError(f"exchange is for world {x.world} and shape {x.shape}, the step for world {plan.world} and "
                         f"{(B, G, plan.k, h, d)}")
    dev = q_main.device
    kpn = k_pre_new if plan.write_col >= 0 else None
    if plan.selected_count > 0:
        rows, _ = _ops.context_local_topk(q_pre, zT, wq_t_scaled, wk, plan.fixed_rows(B, G, dev), plan.off_lo(B, G, dev),
                                          plan.lo, plan.hi, plan.k_local, key_pos=plan.start, key_stride=plan.k,
                                          k_pre_new=kpn, write_col=plan.write_col, keys_out=x.keys)
    else:   # a shard past the legal range: nothing to score, nothing to attend
        rows = torch.empty((B, G, 0), dtype=torch.int64, device=dev)
        x.keys.zero_()
    if plan.k > 0:   # the same on every rank
        x.push(0)
        if plan.selected_count > 0:
            rows = _ops.context_threshold_peer(x.gather_keys, x.flags[0], x.counters[0], rows, plan.rank, plan.k,
                                               plan.fixed_count, plan.k_local, spin=x.spin)
    _ops.gathered_attend_partial(q_main, k_cache, v_cache, rows, scale=scale, part_out=x.parts)
    x.push(1)
    return _ops.lse_merge_peer(x.gather_parts, x.flags[1], x.counters[1], plan.rank, q_main.dtype, spin=x.spin)
