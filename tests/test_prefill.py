"""Batched prefill scorer (config C5): `ops.prefill_score_topk` / al_prefill_score_topk against the oracle's
`prefill_topk`, the decode-time selection (selection.py:71-79, decode.py:86-93) applied to every query row of a
prefill chunk.

CPU tests pin the oracle with hand-worked answers. GPU tests check the kernel's fp32 scores against float64 within the
fp32 summation bound of a 32-term dot product (|err| <= 32 * 2^-24 * sum_j |u_j z_j|), then require the chosen
positions to equal the oracle's selection on the kernel's own scores exactly (ties to the smaller position).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle as orc

DEV = "cuda:0"


def test_oracle_known_answers():
    """zT row 0 holds c % 5 and u = e_0, so the scores are c % 5: every top-k is decided by ties, smaller position first."""
    C = 128
    zT = np.zeros((1, 32, C))
    zT[0, 0] = np.arange(C) % 5
    u = np.zeros((1, 6, 32))
    u[0, :, 0] = 1.0
    got = orc.prefill_topk(u, zT, q_pos0=66, k=4, kcap=5)
    # rows at positions 66..71: legal lengths 67..72; candidates [4, L-64) are empty up to L = 68
    assert (got[0, 0] == -1).all() and (got[0, 1] == -1).all()
    assert got[0, 2].tolist() == [4, -1, -1, -1, -1]                # L = 69: one candidate
    assert got[0, 5].tolist() == [4, 5, 6, 7, -1]                   # L = 72: M = 4 = k, all taken
    got = orc.prefill_topk(u, zT, q_pos0=80, k=4)
    # L = 81: candidates 4..16, scores c % 5: the 4s at 4, 9, 14, then the first 3 (position 8)
    assert got[0, 0].tolist() == [4, 8, 9, 14]
    assert got[0, 5].tolist() == [4, 9, 14, 19]                     # L = 86: candidates up to 21, a fourth 4 at 19
    assert (orc.prefill_topk(u, zT, q_pos0=80, k=0, kcap=2) == -1).all()


def _inputs(H, T, C, seed, ties=0):
    g = torch.Generator().manual_seed(seed)
    u = torch.randn(H, T, 32, generator=g).to(torch.bfloat16)
    zT = torch.randn(H, 32, C, generator=g).to(torch.bfloat16)
    if ties:                                    # every column repeats one of `ties` vectors: scores tie exactly
        zT = zT[:, :, :ties].repeat(1, 1, C // ties + 1)[:, :, :C].contiguous()
    return u, zT


def _check(u, zT, q_pos0, k, kcap, idx, scores):
    u64, z64 = u.double().numpy(), zT.double().numpy()
    H, T, _ = u64.shape
    s = scores.cpu().numpy()
    for t in range(T):
        lay = orc.selection_layout(q_pos0 + t + 1)
        if lay.candidates == 0:
            continue
        with np.errstate(invalid="ignore", over="ignore"):
            want = np.einsum("hj,hjc->hc", u64[:, t], z64[:, :, lay.lo:lay.hi])
            bound = 32 * 2.0 ** -24 * np.einsum("hj,hjc->hc", np.abs(u64[:, t]), np.abs(z64[:, :, lay.lo:lay.hi])) + 1e-30
        got = s[:, t, lay.lo:lay.hi]
        fin = np.isfinite(want)
        err = np.abs(got[fin] - want[fin])
        assert (err <= bound[fin]).all(), f"row {t}: score error {err.max():.3e} above the fp32 bound"
        assert (np.isnan(got[~fin]) == np.isnan(want[~fin])).all(), f"row {t}: NaN scores differ"
        inf = ~fin & ~np.isnan(want)
        assert (got[inf] == want[inf]).all(), f"row {t}: infinite scores differ"
    want = orc.prefill_topk(u64, z64, q_pos0, k, kcap, scores=s)
    got = idx.cpu().numpy()
    bad = np.argwhere((got != want).any(axis=-1))
    assert bad.size == 0, f"{len(bad)} rows differ, first (head, row) {tuple(bad[0])}"


@pytest.mark.gpu
@pytest.mark.parametrize("H,T,q_pos0,C,k,kcap,ties", [
    (2, 600, 0, 1024, 256, 256, 0),        # rows with no candidates, M <= k and M > k; T not a multiple of 16
    (3, 200, 3000, 3200, 256, 300, 0),     # a chunk later in the sequence, kcap > k
    (1, 1000, 7000, 8192, 64, 64, 0),      # long rows, small k
    (2, 300, 1500, 2048, 256, 256, 3),     # three distinct scores per row: position decides every tie
    (1, 64, 500, 1024, 100, 100, 1),       # all scores equal
    (2, 100, 200, 512, 0, 4, 0),           # k = 0: nothing chosen
])
def test_prefill_topk_matches_the_oracle(H, T, q_pos0, C, k, kcap, ties):
    from attention_lab_b200 import ops
    u, zT = _inputs(H, T, C, seed=T + C + ties, ties=ties)
    scores = torch.full((H, T, C), float("nan"), dtype=torch.float32, device=DEV)
    idx = ops.prefill_score_topk(u.to(DEV), zT.to(DEV), k, q_pos0=q_pos0, kcap=kcap, scores_out=scores)
    torch.cuda.synchronize()
    if ties:
        s = scores.cpu().numpy()
        lay = orc.selection_layout(q_pos0 + T)
        for c in range(ties):
            col = s[:, -1, lay.lo + c:lay.hi:ties]
            assert (col == col[:, :1]).all(), "equal columns must score equally"
    _check(u, zT, q_pos0, k, kcap, idx, scores)
    again = ops.prefill_score_topk(u.to(DEV), zT.to(DEV), k, q_pos0=q_pos0, kcap=kcap)
    assert torch.equal(idx, again), "the selection must not depend on the diagnostic scores output"


def _shaped(H, T, C, seed, kind):
    """Inputs that drive the scorer's less common paths: `neg` (most scores negative: thresholds below zero),
    `outlier` (a few huge columns at the start of every row: the first histogram's window starts far too high),
    `zero` (all-zero query rows: every score of those rows is 0), `nonfinite` (NaN and infinite scores)."""
    g = torch.Generator().manual_seed(seed)
    u = torch.randn(H, T, 32, generator=g)
    zT = torch.randn(H, 32, C, generator=g)
    if kind == "neg":
        u = u.abs()
        zT = -zT.abs() + 0.3 * torch.randn(H, 32, C, generator=g)
    elif kind == "outlier":
        zT[:, :, 4:12] *= 4096.0
    elif kind == "zero":
        u[:, ::3] = 0.0
    elif kind == "nonfinite":
        zT[:, :, 40:44] = float("inf")          # +-inf or NaN (0 * inf, inf - inf) depending on u
        zT[:, 5, 300:302] = float("nan")
        u[:, 7::50, 3] = float("inf")
        u[:, 11::50] = float("nan")
    return u.to(torch.bfloat16), zT.to(torch.bfloat16).contiguous()


@pytest.mark.gpu
@pytest.mark.parametrize("kind,H,T,q_pos0,C,k,kcap", [
    ("neg", 2, 700, 0, 1024, 256, 256),
    ("outlier", 2, 500, 900, 1536, 128, 128),
    ("zero", 1, 400, 300, 768, 256, 256),
    ("nonfinite", 2, 600, 100, 1024, 200, 256),
    ("plain", 1, 700, 600, 1408, 400, 450),        # k > 256: positions written straight to the output rows
])
def test_prefill_topk_uncommon_paths_match_the_oracle(kind, H, T, q_pos0, C, k, kcap):
    from attention_lab_b200 import ops
    if kind == "plain":
        u, zT = _inputs(H, T, C, seed=3)
    else:
        u, zT = _shaped(H, T, C, seed=T + C, kind=kind)
    scores = torch.full((H, T, C), float("nan"), dtype=torch.float32, device=DEV)
    idx = ops.prefill_score_topk(u.to(DEV), zT.to(DEV), k, q_pos0=q_pos0, kcap=kcap, scores_out=scores)
    torch.cuda.synchronize()
    _check(u, zT, q_pos0, k, kcap, idx, scores)
    again = ops.prefill_score_topk(u.to(DEV), zT.to(DEV), k, q_pos0=q_pos0, kcap=kcap)
    assert torch.equal(idx, again), "the selection must not depend on the diagnostic scores output"


@pytest.mark.gpu
def test_prefill_topk_full_c5_shape():
    """Config C5 at full size (8 heads x 8192 rows x 8192 columns, k = 256): every row holds min(256, M) ascending
    candidate positions, and sampled rows equal the oracle's selection on the kernel's scores."""
    from attention_lab_b200 import ops
    H, T, C, k = 8, 8192, 8192, 256
    u, zT = _inputs(H, T, C, seed=5)
    scores = torch.full((H, T, C), float("nan"), dtype=torch.float32, device=DEV)
    idx = ops.prefill_score_topk(u.to(DEV), zT.to(DEV), k, scores_out=scores)
    torch.cuda.synchronize()
    got = idx.cpu()
    L = torch.arange(1, T + 1)
    M = (L - 64 - 4).clamp(min=0)
    count = (got >= 0).sum(-1)
    assert torch.equal(count, M.clamp(max=k).expand(H, T).to(count.dtype))
    valid = got >= 0
    assert (got[..., 1:][valid[..., 1:]] > got[..., :-1][valid[..., 1:]]).all(), "positions must ascend"
    assert (got[valid] >= 4).all()
    assert ((got.long() < (L - 64).view(1, T, 1)) | ~valid).all()
    rows = [0, 67, 68, 69, 300, 331, 332, 333, 4095, 8191] + list(range(1000, 8192, 997))
    s = scores[:, rows].cpu().numpy()
    for j, t in enumerate(rows):
        want = orc.prefill_topk(u[:, t:t + 1].double().numpy(), zT.double().numpy(), t, k,
                                scores=s[:, j:j + 1])
        assert np.array_equal(got[:, t:t + 1].numpy(), want), f"row {t}"
