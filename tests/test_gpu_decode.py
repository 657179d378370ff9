"""GPU parity of the sm_100a sparse-decode path against the reference's golden outputs and the float64 oracle.

Ports the reference's hot-path contracts (tests/test_attention_contracts.py, tests/test_metal_score.py,
tests/test_metal_attend.py) to the CUDA kernels, calling through the C ABI. Tolerances: tests/parity.py.
"""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

import cases as cs
from oracle import oracle as orc
from parity import check_out, check_scores, check_topk_sets

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
NAMES = sorted(cs.CASES)


def _al():
    import attention_lab_b200 as al
    from attention_lab_b200 import _lib
    return al, _lib


def gpu(t):
    return {k: (v.to(DEV) if torch.is_tensor(v) else v) for k, v in t.items()}


def golden(name):
    from pathlib import Path
    return np.load(Path(cs.__file__).parent / f"{name}.npz")


def run_step(case, *, cluster=0, k_override=None, poison=None, t=None):
    al, lib = _al()
    t = cs.build(case) if t is None else t
    c = cs.step_constants(case)
    g = gpu(t)
    if poison is not None:
        poison(g)
    zT = g["zT"].clone()
    M = max(c["hi"] - c["lo"], 0)
    scores = torch.full((case.B * case.G * M,), float("nan"), dtype=torch.float32, device=DEV)
    out, rows = al.sparse_decode_step_kernel(
        g["q"], g["q_pre"], g["k"], g["v"], zT, g["wq_t"], g["wk"], torch.from_numpy(c["fixed_rows"]).to(DEV),
        torch.from_numpy(c["off_lo"]).to(DEV), c["lo"], c["hi"], c["k"], c["S"], k_pre_new=g["k_pre_new"],
        write_col=c["write_col"], scale=1 / math.sqrt(case.d), return_rows=True, canonical_order=case.canonical,
        cluster=cluster, scores_out=scores)
    torch.cuda.synchronize()
    assert lib.device_status() == 0
    return t, c, g, out.float().cpu().numpy(), rows.cpu().numpy(), zT, scores.cpu().numpy().reshape(case.B, case.G, M)


def oracle_scores(t, c):
    n = cs.to_np
    u = orc.project_queries(n(t["q_pre"]), n(t["wq_t"]))
    return orc.candidate_scores(u, n(t["zT"]), c["lo"], c["hi"])[:, :, 0, :]


@pytest.mark.parametrize("name", NAMES)
def test_fused_step_matches_reference(name):
    case, gd = cs.CASES[name], golden(name)
    t, c, g, out, rows, zT, scores = run_step(case)
    B, G, S, F = case.B, case.G, c["S"], c["fixed_count"]
    # z column: written once, within one ulp of the reference's value; every other column untouched
    zc = zT[..., c["write_col"]].float().cpu().numpy()
    if case.idx_dtype == "bfloat16":
        assert (np.abs(zc - gd["zcol"]) <= 2.0 ** -8 * np.abs(gd["zcol"]) + 1e-6).all()
        assert (zc == gd["zcol"]).mean() >= 0.9
    else:
        assert np.abs(zc - gd["zcol"]).max() <= 1e-6
    keep = torch.ones(case.C, dtype=torch.bool)
    keep[c["write_col"]] = False
    a, b = zT.cpu()[..., keep], t["zT"][..., keep]
    assert torch.equal(a.view(torch.int16) if a.dtype == torch.bfloat16 else a.view(torch.int32),
                       b.view(torch.int16) if b.dtype == torch.bfloat16 else b.view(torch.int32))
    # scores and top-k set
    s64 = oracle_scores(t, c)
    if s64.size:
        check_scores(scores, s64)
    check_topk_sets(rows, gd["rows"], s64, case, c)
    rows3 = rows.reshape(B, G, S)
    if case.canonical:
        assert (np.diff(rows3, axis=-1) > 0).all(), "canonical order must sort every group's rows"
    else:
        assert (rows3[..., :F] == c["fixed_rows"]).all(), "F must come first"
        assert (np.diff(rows3[..., F:], axis=-1) > 0).all(), "chosen candidates follow in ascending position order"
    # attention over our rows against the float64 oracle, and against the reference's output when sets agree
    n = cs.to_np
    want = orc.gathered_decode_step(n(t["q"]), n(t["k"]), n(t["v"]), rows, S, 1 / math.sqrt(case.d))
    check_out(out, want, case.kv_dtype)
    if all(set(x) == set(y) for x, y in zip(rows3.reshape(B * G, S), gd["rows"].reshape(B * G, S))):
        check_out(out, gd["out_f32"], case.kv_dtype, "out vs reference")


@pytest.mark.parametrize("name", ["c1", "batch2_h4", "capacity_gt_legal"])
def test_every_cluster_size_gives_the_same_rows_and_output(name):
    case = cs.CASES[name]
    base = None
    for cl in (1, 2, 4, 8, 16):
        _, c, _, out, rows, _, scores = run_step(case, cluster=cl)
        if base is None:
            base = (out, rows, scores)
            continue
        assert np.array_equal(rows, base[1]), f"cluster {cl}: rows differ"
        assert np.array_equal(scores, base[2]), f"cluster {cl}: scores differ"
        assert np.abs(out - base[0]).max() <= 1e-5, f"cluster {cl}: output differs"


def test_unselected_rows_are_never_read():
    case = cs.CASES["c1"]
    _, c, _, clean, rows, _, _ = run_step(case)
    sel = np.zeros(case.B * case.G * case.C, dtype=bool)
    sel[rows] = True
    sel_t = torch.from_numpy(sel).to(DEV).view(case.B, case.G, case.C)

    def poison(g):
        g["k"][~sel_t] = float("nan")
        g["v"][~sel_t] = float("nan")
    _, _, _, dirty, rows2, _, _ = run_step(case, poison=poison)
    assert np.array_equal(rows, rows2)
    assert np.isfinite(dirty).all(), "NaN leaked from a row that must not be read"
    assert np.array_equal(dirty, clean)


def test_index_columns_outside_the_scan_may_be_garbage():
    case = cs.CASES["c1_bf16kv"]
    _, c, _, clean, rows, _, scores = run_step(case)

    def poison(g):
        g["zT"][..., :c["lo"]] = float("nan")
        g["zT"][..., c["hi"]:] = float("nan")
    _, _, _, dirty, rows2, zT2, scores2 = run_step(case, poison=poison)
    assert np.array_equal(rows, rows2) and np.array_equal(scores, scores2) and np.array_equal(clean, dirty)
    assert torch.isfinite(zT2[..., c["write_col"]].float()).all(), "write_col must hold the new z"


@pytest.mark.parametrize("name", NAMES)
def test_dense_decode_matches_reference(name):
    al, lib = _al()
    case, gd = cs.CASES[name], golden(name)
    g = gpu(cs.build(case))
    for cl in (0, 1, 4):
        out = al.dense_decode_step(g["q"], g["k"], g["v"], case.L, scale=1 / math.sqrt(case.d), cluster=cl)
        torch.cuda.synchronize()
        assert lib.device_status() == 0
        n = cs.to_np
        want = orc.dense_decode_step(n(g["q"].cpu()), n(g["k"].cpu()), n(g["v"].cpu()), case.L, 1 / math.sqrt(case.d))
        check_out(out.float().cpu().numpy(), want, case.kv_dtype, f"dense cluster {cl}")
        ref_kind = "float32" if case.kv_dtype == "float32" else "bfloat16_vs_bfloat16"
        check_out(out.float().cpu().numpy(), gd["dense"], ref_kind, "dense vs reference")


def test_full_selection_equals_dense():
    al, _ = _al()
    case = cs.CASES["full_selection"]
    _, c, g, out, rows, _, _ = run_step(case)
    assert c["S"] == case.L
    dense = al.dense_decode_step(g["q"], g["k"], g["v"], case.L, scale=1 / math.sqrt(case.d))
    assert np.abs(out - dense.float().cpu().numpy()).max() <= 5e-6
    assert sorted(rows.reshape(case.G, -1)[0] % case.C) == list(range(case.L))


def _attend(al, g, rows, S, cl, d=128):
    out = al.gathered_decode_step_kernel(g["q"], g["k"], g["v"], rows, S, scale=1 / math.sqrt(d), cluster=cl)
    torch.cuda.synchronize()
    return out.float().cpu().numpy()


def test_gathered_attend_boundary_sizes_and_every_cluster():
    al, lib = _al()
    case = cs.Case("attend_sizes", C=600, L=600, kv_dtype="bfloat16", seed=11)
    t = cs.build(case)
    g = gpu(t)
    n = cs.to_np
    for S in (1, 5, 31, 32, 33, 64, 65, 255, 257, 600):
        pos = np.stack([np.random.default_rng(S + gg).permutation(600)[:S] for gg in range(case.G)])
        rows = (pos + np.arange(case.G)[:, None] * case.C).reshape(-1).astype(np.int64)
        want = orc.gathered_decode_step(n(t["q"]), n(t["k"]), n(t["v"]), rows, S, 1 / math.sqrt(case.d))
        for cl in (1, 2, 4, 8, 16):
            out = _attend(al, g, torch.from_numpy(rows).to(DEV), S, cl)
            check_out(out, want, case.kv_dtype, f"S={S} cluster={cl}")
    assert lib.device_status() == 0


def test_gathered_rows_are_original_positions_and_order_does_not_matter():
    al, _ = _al()
    case = cs.CASES["canonical"]
    t, c, g, out, rows, _, _ = run_step(case)
    S = c["S"]
    rows3 = rows.reshape(case.G, S)
    perm = np.stack([np.random.default_rng(i).permutation(S) for i in range(case.G)])
    shuffled = np.take_along_axis(rows3, perm, axis=1).reshape(-1)
    a = _attend(al, g, torch.from_numpy(rows).to(DEV), S, 4)
    b = _attend(al, g, torch.from_numpy(shuffled).to(DEV), S, 4)
    assert np.abs(a - b).max() <= 5e-5
    two = (np.array([2, 9])[None, :] + np.arange(case.G)[:, None] * case.C).reshape(-1)
    zero_one = (np.array([0, 1])[None, :] + np.arange(case.G)[:, None] * case.C).reshape(-1)
    n = cs.to_np
    got = _attend(al, g, torch.from_numpy(two).to(DEV), 2, 1)
    want = orc.gathered_decode_step(n(t["q"]), n(t["k"]), n(t["v"]), two, 2, 1 / math.sqrt(case.d))
    wrong = orc.gathered_decode_step(n(t["q"]), n(t["k"]), n(t["v"]), zero_one, 2, 1 / math.sqrt(case.d))
    check_out(got, want, case.kv_dtype)
    assert np.abs(got - wrong).max() > 1e-2
    assert np.abs(a[:, :, 0] - a[:, :, 1]).max() > 1e-2, "the heads of a group share rows, not answers"


@pytest.mark.parametrize("selector", ["B_recent", "C_uniform"])
def test_selectors_b_and_c_attend_through_the_gathered_kernel(selector):
    """The reference's B and C selectors (decode.py:94-127) build their row lists on the host and attend through
    gathered_decode_step_kernel; here that kernel is the CUDA one. Same F, same budget, the same rows as the oracle's
    restatement of each selector, outputs within the tolerance of tests/parity.py."""
    al, lib = _al()
    for name in ("c1_bf16kv", "canonical"):
        case = cs.CASES[name]
        t = cs.build(case)
        c = cs.step_constants(case)
        g = gpu(t)
        n = cs.to_np
        if selector == "B_recent":
            rows = orc.select_rows_recent(c["fixed_rows"], c["off_lo"], c["lo"], c["hi"], c["k"])
        else:
            rows = orc.select_rows_uniform(c["fixed_rows"], c["off_lo"], c["lo"], c["hi"], c["k"],
                                           rng=np.random.default_rng(1234))
        want = orc.gathered_decode_step(n(t["q"]), n(t["k"]), n(t["v"]), rows, c["S"], 1 / math.sqrt(case.d))
        out = al.gathered_decode_step_kernel(g["q"], g["k"], g["v"], torch.from_numpy(rows).to(DEV), c["S"],
                                             scale=1 / math.sqrt(case.d))
        check_out(out.float().cpu().numpy(), want, case.kv_dtype, f"{selector} {name}")
    assert lib.device_status() == 0


def test_select_rows_and_indexer_ops_match_the_oracle():
    al, lib = _al()
    case, gd = cs.CASES["batch2_h4"], golden("batch2_h4")
    t = cs.build(case)
    c = cs.step_constants(case)
    g = gpu(t)
    n = cs.to_np
    u = al.project_queries(g["q_pre"], g["wq_t"])
    u64 = orc.project_queries(n(t["q_pre"]), n(t["wq_t"]))
    assert np.abs(u.cpu().numpy() - u64).max() <= 1e-6
    zT = g["zT"].clone()
    zT[..., c["write_col"]] = al.project_keys(g["k_pre_new"], g["wk"])[..., 0]
    s = al.candidate_scores(u, zT, c["lo"], c["hi"])
    s64 = orc.candidate_scores(u64, n(t["zT"]), c["lo"], c["hi"])
    check_scores(s.cpu().numpy(), s64)
    rows = al.select_rows_kernel(u, zT, torch.from_numpy(c["fixed_rows"]).to(DEV),
                                 torch.from_numpy(c["off_lo"]).to(DEV), c["lo"], c["hi"], c["k"])
    torch.cuda.synchronize()
    assert lib.device_status() == 0
    check_topk_sets(rows.cpu().numpy(), gd["rows"], s64[:, :, 0, :], case, c)
    z = al.project_keys(g["k_pre"][:, :, :case.L - 1].contiguous(), g["wk"])
    z64 = orc.project_keys(n(t["k_pre"][:, :, :case.L - 1]), n(t["wk"]))
    assert np.abs(z.cpu().numpy() - z64).max() <= 1e-6
    k0 = al.select_rows_kernel(u, zT, torch.from_numpy(c["fixed_rows"]).to(DEV),
                               torch.from_numpy(c["off_lo"]).to(DEV), c["lo"], c["hi"], 0)
    assert torch.equal(k0.cpu(), torch.from_numpy(c["fixed_rows"]).reshape(-1))


def test_append_writes_rows_and_index_columns_chunked_equals_one_shot():
    al, lib = _al()
    B, G, C, d, r = 2, 4, 300, 128, 32
    gen = torch.Generator().manual_seed(3)
    k_new = torch.randn(B, 50, G, d, generator=gen).transpose(1, 2)          # strided like the model's k_main
    v_new = torch.randn(B, G, 50, d, generator=gen)
    k_pre = torch.randn(B, 50, G, d, generator=gen).transpose(1, 2)
    wk = torch.randn(G, r, d, generator=gen) * 0.02
    outs = []
    for bounds in ((0, 50), (0, 7, 30, 50)):
        K = torch.full((B, G, C, d), float("nan"), device=DEV, dtype=torch.bfloat16)
        V = torch.full_like(K, float("nan"))
        Z = torch.full((B, G, r, C), float("nan"), device=DEV)
        for a, b in zip(bounds, bounds[1:]):
            al.append_kvz(K, V, Z, 10 + a, k_new[:, :, a:b].to(DEV), v_new[:, :, a:b].to(DEV),
                          k_pre=k_pre[:, :, a:b].to(DEV), wk=wk.to(DEV))
        torch.cuda.synchronize()
        outs.append((K.cpu(), V.cpu(), Z.cpu()))
        assert torch.equal(K[:, :, 10:60].cpu(), k_new.to(torch.bfloat16))
        assert torch.equal(V[:, :, 10:60].cpu(), v_new.to(torch.bfloat16))
        assert torch.isnan(K[:, :, :10].float()).all() and torch.isnan(K[:, :, 60:].float()).all()
        z64 = orc.project_keys(k_pre.double().numpy(), wk.double().numpy())
        assert np.abs(Z[..., 10:60].cpu().numpy() - z64).max() <= 1e-5
    assert torch.equal(outs[0][2][..., 10:60], outs[1][2][..., 10:60]), "chunked index build differs from one-shot"
    with pytest.raises(RuntimeError, match="capacity"):
        al.append_kvz(K, V, Z, 290, k_new[:, :, :20].to(DEV), v_new[:, :, :20].to(DEV))
    assert lib.device_status() == 0


def test_validation_raises_value_error():
    al, _ = _al()
    case = cs.CASES["c1"]
    t = cs.build(case)
    c = cs.step_constants(case)
    g = gpu(t)
    fr, ol = torch.from_numpy(c["fixed_rows"]).to(DEV), torch.from_numpy(c["off_lo"]).to(DEV)
    base = dict(k_pre_new=g["k_pre_new"], write_col=c["write_col"])

    def call(**kw):
        args = dict(q_main=g["q"], q_pre=g["q_pre"], k_cache=g["k"], v_cache=g["v"], zT=g["zT"].clone(),
                    wq_t_scaled=g["wq_t"], wk=g["wk"])
        args.update({k: v for k, v in kw.items() if k in args})
        extra = {**base, **{k: v for k, v in kw.items() if k not in args}}
        return al.sparse_decode_step_kernel(args["q_main"], args["q_pre"], args["k_cache"], args["v_cache"],
                                            args["zT"], args["wq_t_scaled"], args["wk"], fr, ol, c["lo"], c["hi"],
                                            c["k"], c["S"], **extra)
    with pytest.raises(ValueError):
        call(write_col=(c["lo"] + c["hi"]) // 2)                         # write inside the scanned range
    with pytest.raises(ValueError):
        call(q_main=g["q"].double(), k_cache=g["k"].double(), v_cache=g["v"].double())
    with pytest.raises(ValueError):
        call(k_cache=g["k"].transpose(2, 3).contiguous().transpose(2, 3))  # not contiguous
    with pytest.raises(ValueError):
        call(q_main=torch.cat([g["q"], g["q"]], dim=3))                    # T = 2
    with pytest.raises(ValueError):
        call(backend="flash")
    with pytest.raises(ValueError):
        al.gathered_decode_step_kernel(g["q"], g["k"], g["v"], torch.zeros(8 * 4, dtype=torch.int32, device=DEV), 4)
    with pytest.raises(ValueError):
        q64 = g["q"][..., :64].contiguous()
        al.dense_decode_step(q64, g["k"][..., :64].contiguous(), g["v"][..., :64].contiguous(), 100)


@pytest.mark.parametrize("pattern", ["all_equal", "three_values"])
def test_ties_go_to_the_smaller_position_for_every_cluster_size(pattern):
    """Heavy ties: index columns repeat one (or three) z vectors, so scores tie exactly. The chosen set must be the
    oracle's (score desc, position asc) top-k for every cluster size; all-equal scores also overflow the candidate
    list and exercise the full-array fallback."""
    case = cs.CASES["c1"]
    t = cs.build(case)
    c = cs.step_constants(case)
    zt = t["zT"]
    if pattern == "all_equal":
        zt[..., :case.L - 1] = zt[..., 100:101]
    else:
        idx = torch.arange(case.L - 1) % 3
        zt[..., :case.L - 1] = zt[..., 100:103][..., idx]
    n = cs.to_np
    s64 = oracle_scores(t, c)
    want = orc.topk_indices(s64, c["k"]) + c["lo"]
    for cl in (1, 2, 4, 8, 16):
        _, _, _, _, rows, _, _ = run_step(case, cluster=cl, t=t)
        got = rows.reshape(case.B, case.G, -1)[..., c["fixed_count"]:] - c["off_lo"] + c["lo"]
        assert np.array_equal(np.sort(got, axis=-1), np.sort(want, axis=-1)), f"cluster {cl}"


@pytest.mark.parametrize("pattern", ["all_equal", "half_equal", "three_values"])
def test_ties_with_candidate_list_overflow(pattern):
    """60000 candidates with heavy ties: a CTA whose filtered candidate list overflows rescans the index columns
    (clusters 1 and 2: one CTA holds more tied keys than its list), and in half_equal only the CTA over the tied
    half overflows, so the cluster must agree on the rescan. The chosen set must still be the oracle's
    (score desc, position asc) top-k."""
    case = cs.Case("ties_large", G=2, h=2, C=60000, L=60000, kv_dtype="bfloat16", seed=21)
    t = cs.build(case)
    c = cs.step_constants(case)
    zt = t["zT"]
    n_cand = case.L - 1
    if pattern == "all_equal":
        zt[..., :n_cand] = zt[..., 100:101]
    elif pattern == "half_equal":
        zt[..., : n_cand // 2] = zt[..., 100:101]
    else:
        idx = torch.arange(n_cand) % 3
        zt[..., :n_cand] = zt[..., 100:103][..., idx]
    s64 = oracle_scores(t, c)
    for cl in (1, 2, 4):
        _, _, _, out, rows, _, scores = run_step(case, cluster=cl, t=t)
        check_scores(scores, s64)
        # exact top-k of the kernel's own fp32 scores under (score desc, position asc)
        want = orc.topk_indices(scores.astype(np.float64), c["k"]) + c["lo"]
        got = rows.reshape(case.B, case.G, -1)[..., c["fixed_count"]:] - c["off_lo"] + c["lo"]
        assert np.array_equal(np.sort(got, axis=-1), np.sort(want, axis=-1)), f"cluster {cl}"
        assert np.all(np.diff(got, axis=-1) > 0), "chosen candidates in ascending position order"
