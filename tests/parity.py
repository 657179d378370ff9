"""Parity rules shared by the CPU oracle tests and the GPU tests.

Tolerances (fixed before the first GPU run, never loosened to pass):
- top-k sets, float32 index: equal to the reference's set, except elements whose float64 score lies within
  TIE_TOL = 1e-6 (relative to max(1, |k-th score|)) of the k-th score (ties and rounding at the boundary);
- top-k sets, bfloat16 index: every chosen candidate scores at least the k-th score minus one bf16 rounding of the
  largest score (the reference's own bf16 rule, tests/test_attention_contracts.py:273-277);
- float32 attention outputs: max |diff| <= 5e-5 and relative norm <= 1e-5 against the float64 oracle
  (tests/test_metal_attend.py:168 of the reference);
- bfloat16 attention outputs: relative norm <= 2e-3 and every element within one bf16 ulp (2^-8 relative) plus 1e-6
  of the float64 oracle rounded once (2e-3 relative);
- float32 scores: max |diff| <= 1e-5 and relative norm <= 1e-5 (tests/test_metal_score.py:27 of the reference);
- against an output the reference itself rounded to bfloat16 (two independent roundings): the reference's preset
  bf16 tolerance, max |diff| <= 5e-2 and relative norm <= 2e-2 (tests/test_attention_contracts.py:28-32).
"""
from __future__ import annotations

import numpy as np

TIE_TOL = 1e-6
F32_OUT = {"atol": 5e-5, "rel_norm": 1e-5}
BF16_OUT = {"rel_norm": 2e-3, "ulp": 2.0 ** -8}
BF16_VS_BF16 = {"atol": 5e-2, "rel_norm": 2e-2}
F32_SCORES = {"atol": 1e-5, "rel_norm": 1e-5}


def candidate_sets(rows, fixed_rows, off_lo, B, G):
    rows = np.asarray(rows).reshape(B, G, -1)
    out = {}
    for b in range(B):
        for g in range(G):
            f = set(np.asarray(fixed_rows)[b, g].tolist())
            out[(b, g)] = {int(x) - int(np.asarray(off_lo)[b, g, 0]) for x in rows[b, g].tolist() if int(x) not in f}
    return out


def check_topk_sets(rows_a, rows_b, scores64, case, const):
    """rows_a vs rows_b (flat int64 row lists) under the tie rules above. scores64 [B,G,M] float64."""
    B, G, k = case.B, case.G, const["k"]
    A = candidate_sets(rows_a, const["fixed_rows"], const["off_lo"], B, G)
    R = candidate_sets(rows_b, const["fixed_rows"], const["off_lo"], B, G)
    for key in A:
        a, r = A[key], R[key]
        assert len(a) == k and len(r) == k, f"{key}: {len(a)} / {len(r)} candidates, want {k}"
        if k == 0:
            continue
        s = scores64[key[0], key[1]]
        kth = np.sort(s)[::-1][k - 1]
        if case.idx_dtype == "float32":
            for m in a ^ r:
                assert abs(s[m] - kth) <= TIE_TOL * max(1.0, abs(kth)), \
                    f"{key}: candidate {m} differs (score {s[m]:.9g}, k-th {kth:.9g})"
        else:
            tol = 2.0 ** -8 * np.abs(s).max() + 1e-6
            for m in a:
                assert s[m] >= kth - tol, f"{key}: chosen candidate {m} scores {s[m]:.6g} < k-th {kth:.6g}"


def check_out(got, want64, dtype: str, what: str = "out"):
    got = np.asarray(got, dtype=np.float64)
    want64 = np.asarray(want64, dtype=np.float64)
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    diff = np.abs(got - want64)
    rel = np.linalg.norm(got - want64) / (np.linalg.norm(want64) + 1e-30)
    if dtype == "float32":
        assert diff.max() <= F32_OUT["atol"], f"{what}: max |diff| {diff.max():.3e}"
        assert rel <= F32_OUT["rel_norm"], f"{what}: rel norm {rel:.3e}"
    elif dtype == "bfloat16_vs_bfloat16":
        assert diff.max() <= BF16_VS_BF16["atol"], f"{what}: max |diff| {diff.max():.3e}"
        assert rel <= BF16_VS_BF16["rel_norm"], f"{what}: rel norm {rel:.3e}"
    else:
        assert rel <= BF16_OUT["rel_norm"], f"{what}: rel norm {rel:.3e}"
        assert (diff <= BF16_OUT["ulp"] * np.abs(want64) + 1e-6).all(), \
            f"{what}: element off by more than one bf16 ulp (max {diff.max():.3e})"


def check_scores(got, want64, what="scores"):
    got = np.asarray(got, dtype=np.float64)
    diff = np.abs(got - want64)
    rel = np.linalg.norm(got - want64) / (np.linalg.norm(want64) + 1e-30)
    assert diff.max() <= F32_SCORES["atol"], f"{what}: max |diff| {diff.max():.3e}"
    assert rel <= F32_SCORES["rel_norm"], f"{what}: rel norm {rel:.3e}"


def check_topk_float64(chosen, scores64, k, what="top-k"):
    """chosen [..., k] candidate indices (any order) against the float64 top-k of scores64 [..., M] under
    (score desc, index asc): the sets must be equal except for candidates whose float64 score lies within TIE_TOL
    (relative to max(1, |k-th score|)) of the k-th score -- the north-star rule for identical inputs computed in
    fp32. Returns the number of segments whose sets differ (inside the tolerance)."""
    from oracle import oracle as orc
    chosen = np.asarray(chosen)
    s = np.asarray(scores64, dtype=np.float64)
    want = orc.topk_indices(s, k)
    kth = np.sort(s, axis=-1)[..., ::-1][..., k - 1]
    n_diff = 0
    for idx in np.ndindex(*s.shape[:-1]):
        diff = set(chosen[idx].tolist()) ^ set(want[idx].tolist())
        assert len(set(chosen[idx].tolist())) == k, f"{what} {idx}: duplicate or missing candidates"
        for m in diff:
            assert abs(s[idx][m] - kth[idx]) <= TIE_TOL * max(1.0, abs(kth[idx])), \
                f"{what} {idx}: candidate {m} (score {s[idx][m]:.9g}) differs from the float64 top-k " \
                f"(k-th {kth[idx]:.9g}) beyond the tie tolerance"
        n_diff += len(diff) > 0
    return n_diff
