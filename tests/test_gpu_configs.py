"""GPU parity of the fused step at the configurations the bench numbers are quoted on, against the float64 oracle.

- C3: B = 32, G = 8, h = 4, L = C = 32768, rho = 1/32 (k = 1024, S = 1092), bf16 K/V, bf16 index keys (the bench's
  launch: 256 segments, one CTA each, the one-CTA fast selection) and the same shape with fp32 index keys;
- C4: B = 1, L = C = 131072, k = 4096, automatic cluster (8 CTAs per segment, distributed-shared-memory select).

Inputs are the bench's synthetic distributions (K/V ~ N(0,1); index keys ~ N(0, 0.23^2); wq_t ~ N(0, (0.02/sqrt r)^2),
wk ~ N(0, 0.02^2)), drawn on the device. Checks, per segment (tolerances of tests/parity.py):
- the z column of the newest key is within one index-dtype rounding of the float64 Wk . k_pre_new;
- the kernel's fp32 scores are within the fp32 bound of the float64 scores;
- the chosen set is exactly the top-k of the kernel's own fp32 scores under (score desc, position asc) -- the
  reference's top-k on identical fp32 scores (decode.py:92) -- and it equals the float64 oracle's top-k except for
  candidates whose float64 score lies within TIE_TOL of the k-th (the north-star rule);
- the attention output is within the bf16 tolerance of the float64 oracle over the same rows, and over the oracle's
  own rows whenever the two sets agree;
- the bench path (no score output) chooses exactly the rows of the instrumented path.
"""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from oracle import oracle as orc
from parity import check_out, check_scores, check_topk_float64

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
D, R = 128, 32


def _inputs(B, G, h, C, idx_dtype, seed):
    gen = torch.Generator(device=DEV).manual_seed(seed)
    bf = torch.bfloat16

    def rnd(*shape, dtype=bf, std=1.0):
        return torch.empty(shape, dtype=dtype, device=DEV).normal_(0.0, std, generator=gen)
    t = dict(q=rnd(B, G, h, 1, D), k=rnd(B, G, C, D), v=rnd(B, G, C, D),
             q_pre=rnd(B, G, h, 1, D, dtype=idx_dtype), zT=rnd(B, G, R, C, dtype=idx_dtype, std=0.23),
             wq_t=rnd(G, h * D, R, dtype=idx_dtype, std=0.02 / math.sqrt(R)), wk=rnd(G, R, D, dtype=idx_dtype, std=0.02),
             k_pre_new=rnd(B, G, 1, D, dtype=idx_dtype))
    return t


def _run(t, plan, cluster, scores):
    import attention_lab_b200 as al
    zT = t["zT"].clone()
    B, G = t["q"].shape[:2]
    so = torch.full((B * G * (plan.hi - plan.lo),), float("nan"), device=DEV) if scores else None
    out, rows = al.sparse_decode_step_kernel(t["q"], t["q_pre"], t["k"], t["v"], zT, t["wq_t"], t["wk"],
                                             plan.fixed_rows, plan.off_lo, plan.lo, plan.hi, plan.k,
                                             plan.selected_count, k_pre_new=t["k_pre_new"], write_col=plan.write_col,
                                             return_rows=True, cluster=cluster, scores_out=so)
    torch.cuda.synchronize()
    return out, rows, zT, so


def _np(x):
    return x.detach().to(torch.float64).cpu().numpy()


def _check_config(B, G, h, L, idx_dtype, cluster, seed):
    from attention_lab_b200 import _lib
    from attention_lab_b200.selection import build_step_plan, fixed_budget
    C = L
    t = _inputs(B, G, h, C, idx_dtype, seed)
    plan = build_step_plan(B, G, C, L, fixed_budget(L, 1 / 32), DEV)
    k, S, F, M = plan.k, plan.selected_count, plan.fixed_count, plan.hi - plan.lo
    out, rows, zT, so = _run(t, plan, cluster, scores=True)
    out_b, rows_b, zT_b, _ = _run(t, plan, cluster, scores=False)       # the bench's path: no score output
    assert _lib.device_status() == 0
    assert torch.equal(rows, rows_b), "the bench path chose other rows than the instrumented path"
    assert torch.equal(out.view(torch.int16), out_b.view(torch.int16))

    # z column of the newest key
    z64 = orc.project_keys(_np(t["k_pre_new"]), _np(t["wk"]))[..., 0]         # [B,G,r]
    zc = _np(zT[..., plan.write_col])
    if idx_dtype == torch.bfloat16:
        assert (np.abs(zc - z64) <= 2.0 ** -8 * np.abs(z64) + 1e-7).all()
    else:
        assert np.abs(zc - z64).max() <= 1e-6
    keep = torch.ones(C, dtype=torch.bool, device=DEV)
    keep[plan.write_col] = False
    assert torch.equal(zT[..., keep], t["zT"][..., keep]), "only the write column may change"

    # scores
    u64 = orc.project_queries(_np(t["q_pre"]), _np(t["wq_t"]))                   # [B,G,1,r]
    s64 = orc.candidate_scores(u64, _np(t["zT"]), plan.lo, plan.hi)[:, :, 0, :]  # [B,G,M]
    s32 = so.view(B, G, M).cpu().numpy()
    check_scores(s32, s64)

    # the chosen set
    pos = (rows.view(B, G, S) - plan.off_lo + plan.lo).cpu().numpy()            # candidate positions; F first
    chosen = pos[..., F:] - plan.lo                                              # candidate indices in [0, M)
    assert (np.diff(chosen, axis=-1) > 0).all(), "chosen candidates follow F in ascending position order"
    own = orc.topk_indices(s32.astype(np.float64), k)                            # exact top-k of the fp32 scores
    assert np.array_equal(np.sort(own, axis=-1), chosen), "not the top-k of the kernel's own fp32 scores"
    n_tie = check_topk_float64(chosen, s64, k, "C-config top-k")
    want = orc.topk_indices(s64, k)
    assert (rows.view(B, G, S)[..., :F] == plan.fixed_rows).all(), "F comes first"

    # attention over the chosen rows (and over the oracle's rows where the sets agree)
    flat_k, flat_v = t["k"].view(-1, D), t["v"].view(-1, D)
    rsel = rows.view(B, G, S)
    ksub, vsub = _np(flat_k[rsel.reshape(-1)].view(B, G, S, D)), _np(flat_v[rsel.reshape(-1)].view(B, G, S, D))
    want_out = orc.subset_attention(_np(t["q"]), ksub, vsub, 1 / math.sqrt(D))
    check_out(_np(out), want_out, "bfloat16", "output over the chosen rows")
    if n_tie == 0:
        orows = torch.from_numpy(np.concatenate([plan.fixed_rows.cpu().numpy(), want + plan.off_lo.cpu().numpy()],
                                                axis=-1)).to(DEV)
        ks2, vs2 = _np(flat_k[orows.reshape(-1)].view(B, G, S, D)), _np(flat_v[orows.reshape(-1)].view(B, G, S, D))
        check_out(_np(out), orc.subset_attention(_np(t["q"]), ks2, vs2, 1 / math.sqrt(D)), "bfloat16",
                  "output over the oracle's rows")
    return rows


@pytest.mark.parametrize("idx_dtype", [torch.bfloat16, torch.float32], ids=["bf16_index", "f32_index"])
def test_c3_fused_step_matches_the_oracle(idx_dtype):
    """The C3 launch: 256 segments, one CTA each (the automatic choice at this batch), one-CTA fast selection."""
    rows1 = _check_config(32, 8, 4, 32768, idx_dtype, cluster=1, seed=31)
    rows0 = _check_config(32, 8, 4, 32768, idx_dtype, cluster=0, seed=31)
    assert torch.equal(rows0, rows1)


def test_c3_segments_with_clusters_agree():
    """Fewer requests than SMs: the automatic cluster splits each C3 segment over several CTAs; the rows must be
    those of a one-CTA segment and of the oracle."""
    rows_auto = _check_config(2, 8, 4, 32768, torch.bfloat16, cluster=0, seed=32)
    rows_one = _check_config(2, 8, 4, 32768, torch.bfloat16, cluster=1, seed=32)
    assert torch.equal(rows_auto, rows_one)


def test_c4_fused_step_matches_the_oracle():
    """C4: one request, 131072 positions, k = 4096, automatic cluster (8 CTAs per segment)."""
    _check_config(1, 8, 4, 131072, torch.bfloat16, cluster=0, seed=41)
