"""Host-side selection rules and the per-step plan of a sparse decode step.

The rules are attention-lab's (src/attention_lab/selection.py:17-86): a key position j is legal for the query at
p when 0 <= j < valid_length and j <= p; F = the first 4 and last 64 legal positions; the candidate domain is the
contiguous range [lo, hi) between them; k0 = min(round(rho * N0), candidates(N0)) with Python's round (ties to
even) is fixed per request; at every step k = min(k0, candidates now). The step plan (qwen_wrap.py:145-181) turns
these into the device tensors the kernels take: F as flat row ids [B,G,F] and the flat row of candidate 0, [B,G,1].
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

FIXED_PREFIX = 4
FIXED_RECENT = 64


def legal_length(query_position: int, valid_length: int) -> int:
    query_position, valid_length = int(query_position), int(valid_length)
    if query_position < 0 or valid_length < 0:
        raise ValueError(f"negative query_position={query_position} or valid_length={valid_length}")
    n = min(valid_length, query_position + 1)
    if n <= 0:
        raise ValueError(f"no legal key position for query_position={query_position}, valid_length={valid_length}")
    return n


@dataclass(frozen=True)
class SelectionLayout:
    legal_length: int
    fixed_prefix: int
    recent_start: int

    @property
    def candidate_lo(self) -> int:
        return self.fixed_prefix

    @property
    def candidate_hi(self) -> int:
        return self.recent_start

    @property
    def candidate_count(self) -> int:
        return self.recent_start - self.fixed_prefix

    @property
    def fixed_count(self) -> int:
        return self.fixed_prefix + (self.legal_length - self.recent_start)

    def fixed_positions(self) -> list[int]:
        return list(range(self.fixed_prefix)) + list(range(self.recent_start, self.legal_length))

    def clamp_k(self, k: int) -> int:
        if k < 0:
            raise ValueError("k must be non-negative")
        return min(int(k), self.candidate_count)

    def selected_count(self, k: int) -> int:
        return self.fixed_count + self.clamp_k(k)


def selection_layout(legal: int, fixed_prefix: int = FIXED_PREFIX, fixed_recent: int = FIXED_RECENT) -> SelectionLayout:
    legal = int(legal)
    if legal <= 0:
        raise ValueError("legal length must be positive")
    if fixed_prefix < 0 or fixed_recent < 0:
        raise ValueError("fixed set sizes must be non-negative")
    prefix = min(fixed_prefix, legal)
    return SelectionLayout(legal, prefix, max(prefix, legal - fixed_recent))


def fixed_budget(n0: int, rho: float, fixed_prefix: int = FIXED_PREFIX, fixed_recent: int = FIXED_RECENT) -> int:
    rho = float(rho)
    if math.isnan(rho) or not 0.0 <= rho <= 1.0:
        raise ValueError("rho must be in [0, 1]")
    return min(round(rho * int(n0)), selection_layout(n0, fixed_prefix, fixed_recent).candidate_count)


def row_offsets(batch: int, groups: int, capacity: int, device) -> torch.Tensor:
    """[B,G,1] int64 flat-row offsets (b*G+g)*C."""
    return (torch.arange(batch * groups, device=device, dtype=torch.long) * capacity).view(batch, groups, 1)


@dataclass
class StepPlan:
    """One decode step's selection constants, shared by every layer of the step."""

    legal_length: int
    k0: int
    k: int
    lo: int
    hi: int
    fixed_count: int
    selected_count: int
    fixed_rows: torch.Tensor   # [B,G,F] int64 flat rows
    off_lo: torch.Tensor       # [B,G,1] int64

    @property
    def write_col(self) -> int:
        return self.legal_length - 1

    @property
    def candidate_count(self) -> int:
        return self.hi - self.lo


def build_step_plan(batch: int, groups: int, capacity: int, legal_length: int, k0: int, device) -> StepPlan:
    """F and the candidate domain for a step whose legal range is [0, legal_length)."""
    if legal_length > capacity:
        raise ValueError(f"legal length {legal_length} exceeds allocated capacity {capacity}")
    lay = selection_layout(legal_length)
    k = lay.clamp_k(k0)
    off = row_offsets(batch, groups, capacity, device)
    pos = torch.tensor(lay.fixed_positions(), dtype=torch.long, device=device).view(1, 1, -1)
    return StepPlan(legal_length=int(legal_length), k0=int(k0), k=int(k), lo=lay.candidate_lo, hi=lay.candidate_hi,
                    fixed_count=lay.fixed_count, selected_count=lay.fixed_count + k,
                    fixed_rows=(pos + off).contiguous(), off_lo=(off + lay.candidate_lo).contiguous())
