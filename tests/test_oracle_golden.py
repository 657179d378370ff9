"""Pin the CPU oracle against the reference's own outputs (tests/golden/*.npz, made by make_golden.py).

CPU only. For every golden case: the seeded inputs hash to the recorded sha256 (same generator stream here as where
the fixtures were made), the oracle's scores match the reference's, its top-k set equals the reference's (ties
within 1e-6 excepted for fp32; the bf16 rule of the reference's own test otherwise), and its attention, dense read
and z column match within the reference's preset float32 tolerances.
"""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

import cases as cs
from oracle import oracle as orc
from parity import check_topk_sets

NAMES = sorted(cs.CASES)


def load(name):
    from pathlib import Path
    return np.load(Path(cs.__file__).parent / f"{name}.npz")


@pytest.mark.parametrize("name", NAMES)
def test_inputs_reproduce(name):
    t = cs.build(cs.CASES[name])
    assert cs.sha256_of(t) == str(load(name)["inputs_sha256"]), "seeded inputs differ from the fixture's"


@pytest.mark.parametrize("name", NAMES)
def test_oracle_matches_reference(name):
    case, g = cs.CASES[name], load(name)
    t = cs.build(case)
    c = cs.step_constants(case)
    assert (c["lo"], c["hi"], c["k"], c["S"]) == (int(g["lo"]), int(g["hi"]), int(g["k"]), int(g["S"]))
    n = cs.to_np
    zT = n(t["zT"]).copy()
    out, rows = orc.sparse_decode_step(n(t["q"]), n(t["q_pre"]), n(t["k"]), n(t["v"]), zT, n(t["wq_t"]), n(t["wk"]),
                                       c["fixed_rows"], c["off_lo"], c["lo"], c["hi"], c["k"], c["S"],
                                       k_pre_new=n(t["k_pre_new"]), write_col=c["write_col"],
                                       scale=1 / math.sqrt(case.d), canonical_order=case.canonical)
    # z column: float64 oracle vs the reference's value in the index dtype (one bf16 ulp; fp32: a 128-term dot
    # product's rounding, 1e-6 absolute)
    zc = zT[..., c["write_col"]]
    tol = 2.0 ** -8 * np.abs(zc) + 1e-7 if case.idx_dtype == "bfloat16" else 1e-6
    assert np.all(np.abs(g["zcol"] - zc) <= tol)
    # scores: the reference's matmul in its dtype vs the oracle over the same (rounded) z column
    u = orc.project_queries(n(t["q_pre"]), n(t["wq_t"]))
    zr = zT.copy()
    zr[..., c["write_col"]] = g["zcol"]
    s64 = orc.candidate_scores(u, zr, c["lo"], c["hi"])[:, :, 0, :]
    if s64.size == 0:
        assert g["scores"].size == 0
    elif case.idx_dtype == "float32":
        assert np.abs(g["scores"] - s64).max() <= 1e-5
        if g["scores_ref64"].size:
            assert np.abs(g["scores_ref64"] - s64).max() <= 1e-5
    else:   # bf16 matmul output is rounded to bf16: within 2^-8 relative (+ the rounding of u)
        assert np.abs(g["scores"] - s64).max() <= 2.0 ** -7 * np.abs(s64).max() + 1e-4
    # top-k sets: the oracle's choice against the reference's
    check_topk_sets(rows, g["rows"], s64, case, c)
    # attention over the reference's own rows, float64 vs the reference run in float32
    out_ref_rows = orc.gathered_decode_step(n(t["q"]), n(t["k"]), n(t["v"]), g["rows"], c["S"], 1 / math.sqrt(case.d))
    assert np.abs(out_ref_rows - g["out_f32"]).max() <= 1e-4
    rel = np.linalg.norm(out_ref_rows - g["out_f32"]) / np.linalg.norm(g["out_f32"])
    assert rel <= 1e-5
    if case.kv_dtype == "float32":
        assert np.abs(out_ref_rows - g["out"]).max() <= 1e-4
    else:
        assert np.abs(out_ref_rows - g["out"]).max() <= 5e-2
    # the oracle's own rows give the same answer (same set up to ties); a bf16 index ties so often that the
    # reference's own bf16 rule only bounds the chosen scores (checked above), not the set
    if case.idx_dtype == "float32":
        assert np.abs(out - out_ref_rows).max() <= 1e-4
    dense = orc.dense_decode_step(n(t["q"]), n(t["k"]), n(t["v"]), case.L, 1 / math.sqrt(case.d))
    assert np.abs(dense - g["dense"]).max() <= (1e-4 if case.kv_dtype == "float32" else 5e-2)
    assert np.isfinite(out).all()


def test_known_answers_selection_rules():
    """Known answers of the reference's contract tests (test_attention_contracts.py:309-335)."""
    assert [orc.fixed_budget(8192, 1 / 32), orc.fixed_budget(8192, 1 / 8), orc.fixed_budget(32768, 1 / 32)] == [256, 1024, 1024]
    assert [orc.fixed_budget(100, 1 / 32), orc.fixed_budget(50, 0.5), orc.fixed_budget(4, 1.0)] == [3, 0, 0]
    lay = orc.selection_layout(100)
    assert (lay.fixed_count, lay.candidates, lay.lo, lay.hi) == (68, 32, 4, 36)
    assert lay.fixed_positions() == list(range(4)) + list(range(36, 100))
    assert (orc.selection_layout(50).fixed_count, orc.selection_layout(50).candidates) == (50, 0)
    assert (orc.selection_layout(3).fixed_count, orc.selection_layout(3).prefix) == (3, 3)
    assert (orc.legal_length(5, 10), orc.legal_length(20, 10)) == (6, 10)
    for bad in ((-1, 10), (3, 0)):
        with pytest.raises(ValueError):
            orc.legal_length(*bad)
    with pytest.raises(ValueError):
        orc.selection_layout(0)
    plan = orc.make_plan(1, 2, 128, legal=100, rho=1 / 32, n0=8192)
    assert (plan.k0, plan.k, plan.selected_count) == (256, 32, 100)
    only_f = orc.make_plan(1, 2, 128, legal=128, rho=0.0)
    assert (only_f.k, only_f.selected_count) == (0, 68)
    short = orc.make_plan(1, 2, 128, legal=60, rho=1 / 8)
    assert (short.k, short.selected_count) == (0, 60)
    at128 = orc.make_plan(1, 2, 128, legal=128, rho=1 / 8)
    assert (at128.layout.fixed_count, at128.k, at128.selected_count) == (68, 16, 84)
    at256 = orc.make_plan(1, 2, 256, legal=256, rho=1 / 8)
    assert (at256.lo, at256.hi, at256.k) == (4, 192, 32)
    assert orc.fixed_budget(101, 1 / 8) == 13                       # test_qwen_wrapper.py:387-399
    assert orc.fixed_budget(8193, 1 / 32) == 256                    # config C2's k0


def test_known_answers_ledger():
    """Known answers of the reference's ledger tests (tests/test_roofline.py:14-37)."""
    m4b = orc.LEDGER_MODELS["Qwen3-4B"]
    assert orc.ledger(orc.LEDGER_MODELS["Qwen3-0.6B"], 8192)["index_parameter_count"] == 2752512
    assert orc.ledger(m4b, 8192)["index_parameter_count"] == 5898240
    x = orc.ledger(m4b, 512, rho=0)
    assert (x["k"], x["selected_count"]) == (0, 68)
    assert orc.ledger(m4b, 512, rho=1)["selected_count"] == 512
    x = orc.ledger(m4b, 4)
    assert (x["fixed_count"], x["candidate_count"], x["k"]) == (4, 0, 0)
    x = orc.ledger(m4b, 8192)
    assert x["d_s2_bytes"] - x["d_s1_bytes"] == 2 * x["selected_kv_bytes"]
    x = orc.ledger(m4b, 32768, scan_scope="all")
    assert x["index_read_bytes"] / x["dense_kv_bytes"] == 0.125
    bw = 716.8e9
    assert round((x["dense_kv_bytes"] - x["d_s1_bytes"]) / bw * 1000, 2) == 5.67
    assert round((x["dense_kv_bytes"] - x["d_s2_bytes"]) / bw * 1000, 2) == 5.22
    for kw in ({"rho": -1}, {"rho": float("nan")}, {"rho": 1.1}, {"r": 0}, {"element_bytes": 0}):
        with pytest.raises(ValueError):
            orc.ledger(m4b, 8192, **kw)
    # per-(layer, request) terms used by the bench: config C3 at zb = 2 (21.2 MB) and zb = 4 (37.96 MB)
    c3 = orc.layer_request_bytes(G=8, d=128, r=32, M=32768 - 68, S=68 + 1024, zb=2, eb=2)
    assert c3["score_bytes"] == 8 * 32 * 32700 * 2 and c3["attend_bytes"] == 1092 * 8 * 128 * 2 * 2
    assert abs(c3["d_s1_bytes"] / 1e6 - 21.2) < 0.05
    assert abs(orc.layer_request_bytes(G=8, d=128, r=32, M=32700, S=1092, zb=4, eb=2)["d_s1_bytes"] / 1e6 - 37.96) < 0.05


def test_topk_tie_rule_and_nan():
    s = np.array([[1.0, 3.0, 3.0, np.nan, 2.0, 3.0]])
    assert orc.topk_indices(s, 3).tolist() == [[3, 1, 2]]
    assert orc.topk_indices(s, 4).tolist() == [[3, 1, 2, 5]]
    assert orc.topk_indices(s, 0).shape == (1, 0)
    # NaN ranks above +inf (torch.topk's order), equal NaNs and equal infinities by position
    s = np.array([[np.inf, 1.0, np.nan, np.inf, np.nan, -np.inf]])
    assert orc.topk_indices(s, 6).tolist() == [[2, 4, 0, 3, 1, 5]]


def test_context_split_protocol_equals_single_device():
    """Local top-k per shard, a global k-th key from the union, a keep mask and an LSE merge reproduce the
    single-device top-k set and attention exactly (the C4 protocol, checked on the oracle)."""
    rng = np.random.default_rng(0)
    M, k, P, h, d = 4000, 300, 4, 4, 128
    s = rng.standard_normal(M).astype(np.float32).astype(np.float64)
    s[100:110] = s[5]          # ties across shards
    pos = np.arange(M)
    want = set(orc.topk_indices(s[None], k)[0].tolist())
    shards = np.array_split(pos, P)
    loc = [orc.local_topk(s[sh], sh, k) for sh in shards]
    tau_s, tau_p = orc.global_threshold(np.concatenate([a for a, _ in loc]), np.concatenate([b for _, b in loc]), k)
    got = set()
    for sh in shards:
        got |= set(sh[orc.keep_mask(s[sh], sh, tau_s, tau_p)].tolist())
    assert got == want
    q = rng.standard_normal((h, d))
    K = rng.standard_normal((M, d))
    V = rng.standard_normal((M, d))
    sel = np.array(sorted(want))
    parts = [orc.partial_attention(q, K[np.intersect1d(sh, sel)], V[np.intersect1d(sh, sel)], 1 / math.sqrt(d))
             for sh in shards]
    merged = orc.lse_merge([p[0] for p in parts], [p[1] for p in parts], [p[2] for p in parts])
    full = orc.subset_attention(q[None, None, :, None, :], K[sel][None, None], V[sel][None, None], 1 / math.sqrt(d))
    assert np.abs(merged - full[0, 0, :, 0, :]).max() < 1e-12


def test_selectors_b_and_c_known_answers():
    """B takes the k newest candidates after F (decode.py:94-107); C draws a uniform k-subset per (batch, group) from
    the caller's generator, so the same seed gives the same rows (decode.py:110-127)."""
    fixed = np.array([[[0, 1, 2, 3, 90, 91]]], dtype=np.int64)
    off_lo = np.array([[[4]]], dtype=np.int64)
    rows = orc.select_rows_recent(fixed, off_lo, 4, 90, 5)
    assert rows.tolist() == [0, 1, 2, 3, 90, 91, 85, 86, 87, 88, 89]
    a = orc.select_rows_uniform(fixed, off_lo, 4, 90, 7, rng=np.random.default_rng(11))
    b = orc.select_rows_uniform(fixed, off_lo, 4, 90, 7, rng=np.random.default_rng(11))
    assert np.array_equal(a, b) and len(set(a[6:].tolist())) == 7 and all(4 <= r < 90 for r in a[6:])
    with pytest.raises(ValueError):
        orc.select_rows_recent(fixed, off_lo, 4, 90, 87)


@pytest.mark.parametrize("name", NAMES)
def test_torch_restatement_reproduces_the_reference(name):
    """oracle/torch_ref.py (the reference arm of bench.py) runs the reference's own torch operators in the reference's
    dtypes: on the golden inputs it must give the reference's rows, z column and output."""
    from oracle import torch_ref as tr
    case, g = cs.CASES[name], load(name)
    t = cs.build(case)
    c = cs.step_constants(case)
    zT = t["zT"].clone()
    with torch.inference_mode():
        out, rows = tr.sparse_decode_step_kernel(t["q"], t["q_pre"], t["k"], t["v"], zT, t["wq_t"], t["wk"],
                                                 torch.from_numpy(c["fixed_rows"]), torch.from_numpy(c["off_lo"]),
                                                 c["lo"], c["hi"], c["k"], c["S"], k_pre_new=t["k_pre_new"],
                                                 write_col=c["write_col"], scale=1 / math.sqrt(case.d),
                                                 canonical_order=case.canonical)
    assert np.array_equal(zT[..., c["write_col"]].to(torch.float32).numpy(), g["zcol"])
    assert np.array_equal(rows.numpy(), g["rows"])
    assert np.abs(out.to(torch.float32).numpy() - g["out"]).max() <= 1e-6
