"""The reference's sparse decode step restated with the same torch operators -- TEST AND BASELINE INFRASTRUCTURE ONLY.

attention-lab's path is device-agnostic torch code; this module restates its hot-path functions operator for operator
(matmul, topk, cat, index_select, scaled_dot_product_attention, copy_) so that the reference's own CPU cost can be
timed on the GPU box's host cores, where the reference itself is not installed. It is pinned to the reference's
golden outputs by tests/test_oracle_golden.py. Only `bench.py`'s reference arm / cpu_baseline leg and the tests use it;
the product (`attention_lab_b200`) never imports it.

Each function cites the reference function it restates (paths relative to the attention-lab project root).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def project_keys(k_pre: torch.Tensor, wk: torch.Tensor) -> torch.Tensor:
    """src/attention_lab/indexer.py:15-17: k_pre [B,G,C,d], wk [G,r,d] -> [B,G,r,C]."""
    return torch.matmul(wk.unsqueeze(0), k_pre.transpose(-1, -2))


def project_queries(q_pre: torch.Tensor, wq_t_scaled: torch.Tensor) -> torch.Tensor:
    """src/attention_lab/indexer.py:20-24: q_pre [B,G,h,T,d] -> u [B,G,T,r]."""
    B, G, h, T, d = q_pre.shape
    return torch.matmul(q_pre.permute(0, 1, 3, 2, 4).reshape(B, G, T, h * d), wq_t_scaled.unsqueeze(0))


def candidate_scores(u: torch.Tensor, zT: torch.Tensor, lo: int, hi: int) -> torch.Tensor:
    """src/attention_lab/indexer.py:27-29: u [B,G,T,r] . zT[..., lo:hi] -> [B,G,T,hi-lo]."""
    return torch.matmul(u, zT[..., lo:hi])


def select_rows_kernel(u, zT, fixed_rows, off_lo, lo: int, hi: int, k: int) -> torch.Tensor:
    """src/attention_lab/decode.py:86-93: one matmul, one topk, merge with F -> flat rows [B*G*S]."""
    B, G = fixed_rows.shape[:2]
    if k <= 0:
        return fixed_rows.reshape(-1)
    top = torch.topk(candidate_scores(u, zT, lo, hi), k, dim=-1).indices.view(B, G, k)
    return torch.cat([fixed_rows, top + off_lo], dim=-1).view(-1)


def gathered_decode_step_kernel(q_main, k_cache, v_cache, rows, selected_count: int, *, scale=None):
    """src/attention_lab/decode.py:131-142 with sparse.py:40-60 (backend "sdpa"): two flattened index_selects,
    then SDPA with the h query heads of a group folded into the sequence axis."""
    B, G, h, T, d = q_main.shape
    k_sub = k_cache.view(-1, d).index_select(0, rows).view(B, G, selected_count, d)
    v_sub = v_cache.view(-1, d).index_select(0, rows).view(B, G, selected_count, d)
    out = F.scaled_dot_product_attention(q_main.reshape(B, G, h * T, d), k_sub, v_sub, scale=scale)
    return out.view(B, G, h, T, d)


def sparse_decode_step_kernel(q_main, q_pre, k_cache, v_cache, zT, wq_t_scaled, wk, fixed_rows, off_lo, lo: int,
                              hi: int, k: int, selected_count: int, *, k_pre_new=None, write_col: int = -1,
                              scale=None, canonical_order: bool = False):
    """src/attention_lab/decode.py:145-163: z of the newest key into its column, u, select, (sort), attend.
    Returns (out [B,G,h,1,d], rows [B*G*S])."""
    B, G, h, T, d = q_main.shape
    if k_pre_new is not None:
        zT[..., write_col:write_col + 1].copy_(project_keys(k_pre_new, wk))
    u = project_queries(q_pre, wq_t_scaled)
    rows = select_rows_kernel(u, zT, fixed_rows, off_lo, lo, hi, k)
    if canonical_order:
        rows = rows.view(B, G, selected_count).sort(dim=-1).values.reshape(-1)
    return gathered_decode_step_kernel(q_main, k_cache, v_cache, rows, selected_count, scale=scale), rows


def append_kv(k_cache, v_cache, start: int, k_new, v_new) -> None:
    """The K/V copies of src/attention_lab/qwen_wrap.py:90-106 (LabCache.append) for new rows [B,G,T,d]."""
    T = k_new.shape[2]
    k_cache[:, :, start:start + T].copy_(k_new)
    v_cache[:, :, start:start + T].copy_(v_new)
