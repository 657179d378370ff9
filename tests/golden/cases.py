"""Seeded synthetic inputs for the parity cases (shared by `make_golden.py`, the CPU oracle tests and the GPU tests).

Inputs are drawn from torch's CPU generator so that the reference (which defines its random tensors through that
generator) and this repository see bit-identical values. Shapes follow the reference's conventions:
q/q_pre [B,G,h,1,d], K/V/k_pre [B,G,C,d], zT [B,G,r,C], wq_t_scaled [G,h*d,r], wk [G,r,d].

Config C1 of the build (one Qwen3-0.6B-shape layer, B=1, G=8, h=2, d=128, L=2048, r=32, k=64) is `CASES["c1"]`;
the others are the edge cases the reference's contract tests exercise (k=0, short history, full selection,
capacity above the legal length, batch > 1, bf16 index keys, canonical order).
"""
from __future__ import annotations

import hashlib
import math
from dataclasses import dataclass, field

import numpy as np
import torch

ROPE_THETA = 1.0e6


@dataclass(frozen=True)
class Case:
    name: str
    B: int = 1
    G: int = 8
    h: int = 2
    d: int = 128
    r: int = 32
    C: int = 2048          # capacity
    L: int = 2048          # legal length (query at L-1)
    rho: float = 1 / 32
    k0: int | None = None  # overrides the rho rule (k0 = capacity forces a full selection)
    kv_dtype: str = "float32"
    idx_dtype: str = "float32"
    canonical: bool = False
    poison_tail: bool = False   # NaN into every slot at or beyond L (K, V, k_pre, zT)
    seed: int = 0
    extra: dict = field(default_factory=dict)


CASES = {c.name: c for c in [
    Case("c1"),                                                               # config C1, fp32 K/V
    Case("c1_bf16kv", kv_dtype="bfloat16"),                                   # config C1 as stated: bf16 K/V, fp32 index
    Case("k0_fixed_only", C=512, L=512, rho=0.0, seed=1),                     # k = 0 reads exactly F
    Case("short_history", C=128, L=60, seed=2),                               # L <= 68: F covers everything
    Case("full_selection", C=320, L=300, k0=320, seed=3),                     # every candidate selected = dense
    Case("capacity_gt_legal", C=640, L=600, rho=1 / 8, poison_tail=True, seed=4),
    Case("batch2_h4", B=2, G=4, h=4, C=384, L=300, rho=1 / 8, seed=5),
    Case("bf16_index", C=1024, L=1000, rho=1 / 8, kv_dtype="bfloat16", idx_dtype="bfloat16", seed=6),
    Case("canonical", C=1024, L=1000, rho=1 / 8, canonical=True, seed=7),
    Case("odd_capacity", C=601, L=585, rho=1 / 8, seed=8),                   # unaligned capacity (scalar scan path)
]}


def _dt(name: str):
    return getattr(torch, name)


def rope(x: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
    """Rotate-half RoPE with theta 1e6 (the Qwen3 convention), float64. x [..., n, d], positions [n]."""
    d = x.shape[-1]
    inv = 1.0 / (ROPE_THETA ** (torch.arange(0, d, 2, dtype=torch.float64) / d))
    ang = positions.to(torch.float64)[:, None] * inv[None, :]
    cos = torch.cat([ang.cos(), ang.cos()], dim=-1)
    sin = torch.cat([ang.sin(), ang.sin()], dim=-1)
    half = d // 2
    rot = torch.cat([-x[..., half:], x[..., :half]], dim=-1)
    return x * cos + rot * sin


def indexer_weights(G, h, d, r, seed):
    """GroupedIndexer init (attention-lab src/attention_lab/indexer.py:35-45): float64 draws from Generator(seed)."""
    gen = torch.Generator().manual_seed(int(seed))
    wq = torch.randn(G, r, h * d, generator=gen, dtype=torch.float64) * 0.02
    wk = torch.randn(G, r, d, generator=gen, dtype=torch.float64) * 0.02
    wq_t = (wq / math.sqrt(r)).transpose(1, 2).contiguous()
    return wq, wk, wq_t


def build(case: Case) -> dict:
    """All inputs of one decode step as CPU torch tensors in their working dtypes (plus float64 weights)."""
    B, G, h, d, r, C, L = case.B, case.G, case.h, case.d, case.r, case.C, case.L
    gen = torch.Generator().manual_seed(case.seed)
    q = torch.randn(B, G, h, 1, d, generator=gen, dtype=torch.float64)
    k = torch.randn(B, G, C, d, generator=gen, dtype=torch.float64)
    v = torch.randn(B, G, C, d, generator=gen, dtype=torch.float64)
    q_pre = torch.randn(B, G, h, 1, d, generator=gen, dtype=torch.float64)
    k_pre = torch.randn(B, G, C, d, generator=gen, dtype=torch.float64)
    pos = torch.arange(C)
    k = rope(k, pos)                                  # the cache holds rotated keys at their own positions
    q = rope(q, torch.tensor([L - 1]))                # the query sits at position L-1
    kvd, idd = _dt(case.kv_dtype), _dt(case.idx_dtype)
    wq, wk, wq_t = indexer_weights(G, h, d, r, case.seed)
    q, k, v = q.to(kvd), k.to(kvd), v.to(kvd)
    q_pre, k_pre = q_pre.to(idd), k_pre.to(idd)
    wk_w, wq_t_w = wk.to(idd), wq_t.to(idd)
    # the index table of the history: z = Wk . k_pre, columns [0, L-1); column L-1 is written by the step itself
    zT = torch.matmul(wk_w.unsqueeze(0), k_pre.transpose(-1, -2)).contiguous()    # [B,G,r,C] in the index dtype
    zT[..., L - 1:] = float("nan")                                                   # not yet written
    if case.poison_tail:
        for x in (k, v, k_pre):
            x[:, :, L:] = float("nan")
    k_pre_new = k_pre[:, :, L - 1:L].contiguous()
    return {"q": q.contiguous(), "k": k.contiguous(), "v": v.contiguous(), "q_pre": q_pre.contiguous(),
            "k_pre": k_pre.contiguous(), "k_pre_new": k_pre_new, "zT": zT, "wq": wq, "wk": wk_w.contiguous(),
            "wq_t": wq_t_w.contiguous(), "wk64": wk, "wq_t64": wq_t}


def step_constants(case: Case) -> dict:
    """prepare_request (attention-lab src/attention_lab/decode.py:61-83) restated for a query at L-1."""
    import sys
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parents[2]))
    from oracle import oracle as orc
    plan = orc.make_plan(case.B, case.G, case.C, legal=case.L, rho=case.rho)
    k = plan.k if case.k0 is None else plan.layout.clamp_k(case.k0)
    return {"lo": plan.lo, "hi": plan.hi, "k": k, "S": plan.layout.fixed_count + k, "write_col": case.L - 1,
            "fixed_rows": plan.fixed_rows, "off_lo": plan.off_lo, "fixed_count": plan.layout.fixed_count}


def sha256_of(tensors: dict, keys=("q", "k", "v", "q_pre", "k_pre", "zT", "wk", "wq_t")) -> str:
    h = hashlib.sha256()
    for key in keys:
        t = tensors[key]
        h.update(key.encode())
        h.update(t.contiguous().view(torch.uint8).numpy().tobytes() if t.dtype == torch.bfloat16
                 else t.contiguous().numpy().tobytes())
    return h.hexdigest()


def to_np(t: torch.Tensor) -> np.ndarray:
    """float64 numpy view of a tensor (bf16 values are exact in float64)."""
    return t.detach().to(torch.float64).numpy()
