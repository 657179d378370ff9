"""CPU oracle for the sparse-decode hot path -- TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the algorithm of attention-lab's sparse decode step so that the CUDA path can be
checked against it. It is the checker, never the product: only `tests/`, `__graft_entry__.smoke()` and the
`cpu_baseline` / `--impl reference` legs of `bench.py` may import it. The product path (`attention_lab_b200`) never
imports anything from here and fails loudly when its CUDA library is missing.

Parity of this restatement is pinned against golden vectors produced by the reference itself (the generating script
is `tests/golden/make_golden.py`; the fixtures are `tests/golden/*.npz`, checked by `tests/test_oracle_golden.py`).

Every function cites the reference file:line it restates (paths relative to the attention-lab project root).
Arithmetic is float64 unless a `dtype` argument says otherwise; the reference's own brute-force check
(`src/attention_lab/indexer.py:57-64`) is float64 too.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

FIXED_PREFIX = 4      # src/attention_lab/selection.py:17
FIXED_RECENT = 64     # src/attention_lab/selection.py:18


# ---------------------------------------------------------------------------------------------------------------------
# selection rules (src/attention_lab/selection.py)
# ---------------------------------------------------------------------------------------------------------------------
def legal_length(query_position: int, valid_length: int) -> int:
    """Legal key range is [0, n): selection.py:21-30."""
    qp, vl = int(query_position), int(valid_length)
    if qp < 0 or vl < 0:
        raise ValueError("negative query position or valid length")
    n = min(vl, qp + 1)
    if n <= 0:
        raise ValueError("no legal key position")
    return n


@dataclass(frozen=True)
class Layout:
    """F = [0, prefix) U [recent_start, legal); candidates [prefix, recent_start): selection.py:33-68."""

    legal: int
    prefix: int
    recent_start: int

    @property
    def lo(self) -> int:
        return self.prefix

    @property
    def hi(self) -> int:
        return self.recent_start

    @property
    def candidates(self) -> int:
        return self.recent_start - self.prefix

    @property
    def fixed_count(self) -> int:
        return self.prefix + (self.legal - self.recent_start)

    def fixed_positions(self) -> list[int]:
        return list(range(self.prefix)) + list(range(self.recent_start, self.legal))

    def clamp_k(self, k: int) -> int:
        if k < 0:
            raise ValueError("k must be non-negative")
        return min(int(k), self.candidates)


def selection_layout(legal: int, fixed_prefix: int = FIXED_PREFIX, fixed_recent: int = FIXED_RECENT) -> Layout:
    """selection.py:71-79."""
    legal = int(legal)
    if legal <= 0:
        raise ValueError("legal length must be positive")
    prefix = min(fixed_prefix, legal)
    return Layout(legal, prefix, max(prefix, legal - fixed_recent))


def fixed_budget(n0: int, rho: float) -> int:
    """k0 = min(round(rho * n0), candidates(n0)), Python round (ties to even): selection.py:80-86."""
    rho = float(rho)
    if math.isnan(rho) or not 0.0 <= rho <= 1.0:
        raise ValueError("rho must be in [0, 1]")
    return min(round(rho * int(n0)), selection_layout(n0).candidates)


def row_offsets(B: int, G: int, C: int) -> np.ndarray:
    """[B,G,1] int64 flat-row offsets (b*G+g)*C: sparse.py:14-16."""
    return (np.arange(B * G, dtype=np.int64) * C).reshape(B, G, 1)


@dataclass
class Plan:
    """Per-step constants of one decode step: decode.py:27-83 (DecodeRequest) / qwen_wrap.py:145-181 (StepPlan)."""

    layout: Layout
    k0: int
    k: int
    fixed_rows: np.ndarray      # [B,G,F] int64 flat rows
    off_lo: np.ndarray          # [B,G,1] int64

    @property
    def lo(self):
        return self.layout.lo

    @property
    def hi(self):
        return self.layout.hi

    @property
    def selected_count(self) -> int:
        return self.layout.fixed_count + self.k

    @property
    def write_col(self) -> int:
        return self.layout.legal - 1


def make_plan(B: int, G: int, C: int, *, legal: int, rho: float, n0=None) -> Plan:
    """prepare_request (decode.py:61-83) for a query at the end of the legal range."""
    if legal > C:
        raise ValueError("legal length exceeds capacity")
    n0 = legal if n0 is None else int(n0)
    k0 = fixed_budget(n0, rho)
    lay = selection_layout(legal)
    off = row_offsets(B, G, C)
    fixed = np.asarray(lay.fixed_positions(), dtype=np.int64).reshape(1, 1, -1)
    return Plan(lay, k0, lay.clamp_k(k0), (fixed + off).copy(), (off + lay.lo).copy())


# ---------------------------------------------------------------------------------------------------------------------
# indexer (src/attention_lab/indexer.py)
# ---------------------------------------------------------------------------------------------------------------------
def project_keys(k_pre: np.ndarray, wk: np.ndarray, dtype=np.float64) -> np.ndarray:
    """zT[b,g,j,c] = sum_e wk[g,j,e] * k_pre[b,g,c,e]: indexer.py:15-17. k_pre [B,G,C,d], wk [G,r,d]."""
    return np.einsum("gje,bgce->bgjc", wk.astype(dtype), k_pre.astype(dtype))


def project_queries(q_pre: np.ndarray, wq_t_scaled: np.ndarray, dtype=np.float64) -> np.ndarray:
    """u[b,g,t,j] = sum_f qcat[b,g,t,f] * wq_t[g,f,j], f = head*d + dim: indexer.py:20-24. q_pre [B,G,h,T,d]."""
    B, G, h, T, d = q_pre.shape
    qcat = np.transpose(q_pre, (0, 1, 3, 2, 4)).reshape(B, G, T, h * d)
    return np.einsum("bgtf,gfj->bgtj", qcat.astype(dtype), wq_t_scaled.astype(dtype))


def candidate_scores(u: np.ndarray, zT: np.ndarray, lo: int, hi: int, dtype=np.float64) -> np.ndarray:
    """s[b,g,t,m] = sum_j u[b,g,t,j] * zT[b,g,j,lo+m]: indexer.py:27-29. Only columns [lo, hi) are touched."""
    return np.einsum("bgtj,bgjm->bgtm", u.astype(dtype), zT[..., lo:hi].astype(dtype))


def indexer_weights(G: int, h: int, d: int, r: int = 32, seed: int = 0, init_std: float = 0.02):
    """GroupedIndexer init (indexer.py:35-45): wq then wk drawn N(0,1) in float64 from torch.Generator(seed), scaled by
    init_std; wq_t_scaled = (wq / sqrt(r))^T. Returns float64 arrays (wq [G,r,h*d], wk [G,r,d], wq_t_scaled [G,h*d,r]).

    The draw uses torch's CPU generator because the reference's weights are defined by that generator's stream.
    """
    import torch
    gen = torch.Generator().manual_seed(int(seed))
    wq = torch.randn(G, r, h * d, generator=gen, dtype=torch.float64) * init_std
    wk = torch.randn(G, r, d, generator=gen, dtype=torch.float64) * init_std
    wq_t = (wq / math.sqrt(r)).transpose(1, 2).contiguous()
    return wq.numpy(), wk.numpy(), wq_t.numpy()


def reference_scores(q_pre, k_pre, wq, wk, r: int, lo: int, hi: int) -> np.ndarray:
    """float64 brute force (Wq.qcat).(Wk.k)/sqrt(r) over [lo, hi): indexer.py:57-64."""
    B, G, h, T, d = q_pre.shape
    qcat = np.transpose(q_pre, (0, 1, 3, 2, 4)).reshape(B, G, T, h * d).astype(np.float64)
    u = np.einsum("bgtf,gjf->bgtj", qcat, wq.astype(np.float64))
    z = np.einsum("gje,bgce->bgcj", wk.astype(np.float64), k_pre.astype(np.float64))
    return np.einsum("bgtj,bgcj->bgtc", u, z)[..., lo:hi] / math.sqrt(r)


# ---------------------------------------------------------------------------------------------------------------------
# top-k and row lists (src/attention_lab/decode.py)
# ---------------------------------------------------------------------------------------------------------------------
def topk_indices(scores: np.ndarray, k: int) -> np.ndarray:
    """Indices of the k largest values along the last axis, ordered (value desc, index asc).

    Restates the single torch.topk of decode.py:92. torch leaves the order of equal values unspecified; this oracle
    (and the CUDA kernels) break ties by the smaller index. NaN ranks above every number, as in torch.topk.
    """
    if k <= 0:
        return np.zeros(scores.shape[:-1] + (0,), dtype=np.int64)
    s = np.asarray(scores, dtype=np.float64)
    nan = np.isnan(s)
    s = np.where(nan, 0.0, s)
    idx = np.broadcast_to(np.arange(s.shape[-1]), s.shape)
    # last key is primary: NaN first (above +inf), then -s ascending, then index ascending
    order = np.lexsort((idx, -s, ~nan), axis=-1)
    return order[..., :k].astype(np.int64)


def select_rows(u, zT, fixed_rows, off_lo, lo: int, hi: int, k: int) -> np.ndarray:
    """F first, then the k best candidates as flat rows: decode.py:86-93. Returns int64 [B*G*S]."""
    B, G = fixed_rows.shape[:2]
    if k <= 0:
        return fixed_rows.reshape(-1).copy()
    s = candidate_scores(u, zT, lo, hi)[:, :, 0, :]            # [B,G,M]
    top = topk_indices(s, k)                                      # [B,G,k]
    return np.concatenate([fixed_rows, top + off_lo], axis=-1).reshape(-1)


def prefill_topk(u: np.ndarray, zT: np.ndarray, q_pos0: int, k: int, kcap=None, scores=None) -> np.ndarray:
    """Batched prefill scorer (config C5): for every query row t (position q_pos0 + t) of every head, the candidates
    of a decode step at legal length q_pos0 + t + 1 (selection.py:71-79) ranked by decode.py:86-93's single top-k
    (ties to the smaller position, topk_indices above), chosen positions in ascending order then -1 up to kcap.

    u [H,T,r], zT [H,r,C]. Scores are float64 u.zT unless `scores` ([H,T,C], e.g. a kernel's own fp32 scores) is
    given, in which case the selection is restated on exactly those values."""
    H, T, _ = u.shape
    kcap = int(k) if kcap is None else int(kcap)
    out = np.full((H, T, kcap), -1, dtype=np.int32)
    for t in range(T):
        lay = selection_layout(q_pos0 + t + 1)
        kk = lay.clamp_k(k)
        if kk == 0:
            continue
        if scores is None:
            s = np.einsum("hj,hjc->hc", u[:, t].astype(np.float64), zT[:, :, lay.lo:lay.hi].astype(np.float64))
        else:
            s = np.asarray(scores[:, t, lay.lo:lay.hi], dtype=np.float64)
        out[:, t, :kk] = np.sort(topk_indices(s, kk) + lay.lo, axis=-1)
    return out


def select_rows_recent(fixed_rows, off_lo, lo: int, hi: int, k: int) -> np.ndarray:
    """Selector B: F, then the k most recent candidates [hi - k, hi) as flat rows: decode.py:94-107."""
    B, G = fixed_rows.shape[:2]
    if k <= 0:
        return fixed_rows.reshape(-1).copy()
    M = hi - lo
    if k > M:
        raise ValueError(f"k={k} exceeds the candidate count {M}")
    rel = np.broadcast_to(np.arange(M - k, M, dtype=np.int64), (B, G, k))
    return np.concatenate([fixed_rows, rel + off_lo], axis=-1).reshape(-1)


def select_rows_uniform(fixed_rows, off_lo, lo: int, hi: int, k: int, *, rng) -> np.ndarray:
    """Selector C: F, then k candidates drawn uniformly without replacement per (batch, group), as the top-k of
    i.i.d. float64 uniforms from the numpy Generator `rng` (drawn [B,G,M] in one call): decode.py:110-127."""
    B, G = fixed_rows.shape[:2]
    if k <= 0:
        return fixed_rows.reshape(-1).copy()
    M = hi - lo
    if k > M:
        raise ValueError(f"k={k} exceeds the candidate count {M}")
    u = rng.random((B, G, M), dtype=np.float64)
    rel = topk_indices(u, k)
    return np.concatenate([fixed_rows, rel + off_lo], axis=-1).reshape(-1)


def subset_attention(q: np.ndarray, k_sub: np.ndarray, v_sub: np.ndarray, scale=None) -> np.ndarray:
    """softmax(q.k_sub^T * scale) @ v_sub with the h query heads sharing the subset: sparse.py:40-60.

    q [B,G,h,T,d], k_sub/v_sub [B,G,S,d] -> [B,G,h,T,d], float64.
    """
    d = q.shape[-1]
    sc = 1.0 / math.sqrt(d) if scale is None else float(scale)
    s = np.einsum("bghtd,bgsd->bghts", q.astype(np.float64), k_sub.astype(np.float64)) * sc
    s = s - s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(axis=-1, keepdims=True)
    return np.einsum("bghts,bgsd->bghtd", p, v_sub.astype(np.float64))


def gathered_decode_step(q_main, k_cache, v_cache, rows, selected_count: int, scale=None) -> np.ndarray:
    """Read exactly the listed flat rows of K and V, then attend: decode.py:131-142."""
    B, G, h, T, d = q_main.shape
    if T != 1:
        raise ValueError("a decode step takes exactly one new query position")
    kf = k_cache.reshape(-1, d)
    vf = v_cache.reshape(-1, d)
    k_sub = kf[rows].reshape(B, G, selected_count, d)
    v_sub = vf[rows].reshape(B, G, selected_count, d)
    return subset_attention(q_main, k_sub, v_sub, scale)


def sparse_decode_step(q_main, q_pre, k_cache, v_cache, zT, wq_t_scaled, wk, fixed_rows, off_lo, lo, hi, k,
                       selected_count, *, k_pre_new=None, write_col=-1, scale=None, canonical_order=False,
                       z_dtype=None):
    """One layer's D read: decode.py:145-163. Writes z of the newest key into zT[..., write_col] (in place, rounded to
    `z_dtype`, default zT's dtype), then u, scores, one top-k, merge with F, optional ascending sort, attend.
    Returns (out [B,G,h,1,d] float64, rows int64 [B*G*S])."""
    B, G, h, T, d = q_main.shape
    if T != 1:
        raise ValueError("a decode step takes exactly one new query position")
    if k_pre_new is not None:
        z = project_keys(k_pre_new, wk)                                   # [B,G,r,1]
        zT[..., write_col:write_col + 1] = z.astype(z_dtype or zT.dtype)
    u = project_queries(q_pre, wq_t_scaled)
    rows = select_rows(u, zT, fixed_rows, off_lo, lo, hi, k)
    if canonical_order:
        rows = np.sort(rows.reshape(B, G, selected_count), axis=-1).reshape(-1)
    out = gathered_decode_step(q_main, k_cache, v_cache, rows, selected_count, scale)
    return out, rows


def dense_decode_step(q_main, k_cache, v_cache, valid_length: int, scale=None) -> np.ndarray:
    """A read for T == 1 at the end of the legal range: every position [0, valid_length), no mask (full.py:17-45)."""
    L = int(valid_length)
    if not 0 < L <= k_cache.shape[2]:
        raise ValueError("valid_length must be in (0, capacity]")
    return subset_attention(q_main, k_cache[:, :, :L], v_cache[:, :, :L], scale)


def dense_mask_reference(q, k, v, selected, valid_length=None, scale=None) -> np.ndarray:
    """Attention restricted to a position subset [B,G,S] (duplicates counted once): reference.py:80-97."""
    B, G, h, T, d = q.shape
    L = k.shape[2] if valid_length is None else int(valid_length)
    sel = np.asarray(selected, dtype=np.int64)
    if sel.size and (sel.min() < 0 or sel.max() >= L):
        raise ValueError("selected positions must lie in [0, legal)")
    keep = np.zeros((B, G, L), dtype=bool)
    for b in range(B):
        for g in range(G):
            keep[b, g, sel[b, g]] = True
    if not keep.any(axis=-1).all():
        raise ValueError("empty selection")
    sc = 1.0 / math.sqrt(d) if scale is None else float(scale)
    s = np.einsum("bghtd,bgld->bghtl", q.astype(np.float64), k[:, :, :L].astype(np.float64)) * sc
    s = np.where(keep[:, :, None, None, :], s, -np.inf)
    s = s - s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(axis=-1, keepdims=True)
    return np.einsum("bghtl,bgld->bghtd", p, v[:, :, :L].astype(np.float64))


# ---------------------------------------------------------------------------------------------------------------------
# cache append (src/attention_lab/qwen_wrap.py:90-106)
# ---------------------------------------------------------------------------------------------------------------------
def append(k_cache, v_cache, z_cache, start: int, k_new, v_new, z_new=None) -> None:
    """Write T new rows at [start, start+T) of K/V [B,G,C,d] and (optionally) z columns of zT [B,G,r,C]."""
    T = k_new.shape[2]
    if start + T > k_cache.shape[2]:
        raise RuntimeError("cache capacity exceeded")
    k_cache[:, :, start:start + T] = k_new
    v_cache[:, :, start:start + T] = v_new
    if z_new is not None:
        z_cache[..., start:start + T] = z_new


# ---------------------------------------------------------------------------------------------------------------------
# context split across ranks (new in the B200 build; the merge is the math of metal_attend.py:147-169)
# ---------------------------------------------------------------------------------------------------------------------
def local_topk(scores: np.ndarray, positions: np.ndarray, k: int):
    """Best min(k, n) (score desc, position asc) of one rank's candidate slice -> (scores, positions)."""
    n = scores.shape[-1]
    kk = min(k, n)
    order = np.lexsort((positions, -np.where(np.isnan(scores), np.inf, scores)))[:kk]
    return scores[order], positions[order]


def global_threshold(all_scores: np.ndarray, all_pos: np.ndarray, k: int):
    """The k-th best (score, position) pair of the union of every rank's local top-k."""
    order = np.lexsort((all_pos, -np.where(np.isnan(all_scores), np.inf, all_scores)))
    j = order[k - 1]
    return float(all_scores[j]), int(all_pos[j])


def keep_mask(scores: np.ndarray, positions: np.ndarray, tau_score: float, tau_pos: int) -> np.ndarray:
    """Candidate is in the global top-k iff (score, -pos) >= (tau_score, -tau_pos) lexicographically."""
    return (scores > tau_score) | ((scores == tau_score) & (positions <= tau_pos))


def partial_attention(q: np.ndarray, k_rows: np.ndarray, v_rows: np.ndarray, scale: float):
    """Unnormalised partial (m, l, acc) of one shard: q [h,d], rows [n,d] -> m [h], l [h], acc [h,d] (float64)."""
    s = (q.astype(np.float64) @ k_rows.astype(np.float64).T) * scale          # [h, n]
    if s.shape[1] == 0:
        return np.full(q.shape[0], -np.inf), np.zeros(q.shape[0]), np.zeros_like(q, dtype=np.float64)
    m = s.max(axis=1)
    p = np.exp(s - m[:, None])
    return m, p.sum(axis=1), p @ v_rows.astype(np.float64)


def lse_merge(ms, ls, accs) -> np.ndarray:
    """Merge P partials: w_p = exp(m_p - m*) where l_p > 0; out = sum w_p acc_p / sum w_p l_p (metal_attend.py:147-169)."""
    ms, ls, accs = np.asarray(ms), np.asarray(ls), np.asarray(accs)          # [P,h], [P,h], [P,h,d]
    mstar = ms.max(axis=0)
    w = np.where(ls > 0, np.exp(ms - mstar[None]), 0.0)
    return (w[..., None] * accs).sum(axis=0) / (w * ls).sum(axis=0)[:, None]


# ---------------------------------------------------------------------------------------------------------------------
# byte ledger (scripts/roofline.py:30-100, scan_scope="candidates")
# ---------------------------------------------------------------------------------------------------------------------
@dataclass(frozen=True)
class ModelShape:
    layers: int
    q_heads: int
    kv_heads: int
    head_dim: int
    parameters: int


LEDGER_MODELS = {  # scripts/roofline.py:24-28
    "Qwen3-0.6B": ModelShape(28, 16, 8, 128, 596_049_920),
    "Qwen3-1.7B": ModelShape(28, 16, 8, 128, 1_720_574_976),
    "Qwen3-4B": ModelShape(36, 32, 8, 128, 4_022_468_096),
}


def ledger(model: ModelShape, n: int, *, rho: float = 1 / 32, r: int = 32, fixed: int = 68, element_bytes: int = 2,
           index_bytes=None, scan_scope: str = "candidates") -> dict:
    """Per-decode-step traffic scenario of one batch-1 request over every layer: roofline.py:30-100."""
    ib = element_bytes if index_bytes is None else index_bytes
    if not isinstance(n, int) or n < 1:
        raise ValueError("n must be a positive integer")
    if not (math.isfinite(rho) and 0 <= rho <= 1):
        raise ValueError("rho must be finite and in [0, 1]")
    if r < 1 or element_bytes < 1 or ib < 1 or fixed < 0:
        raise ValueError("bad ledger parameter")
    if scan_scope not in ("all", "candidates"):
        raise ValueError("scan_scope must be 'all' or 'candidates'")
    fixed_count = min(fixed, n)
    cand = n - fixed_count
    k = min(round(rho * n), cand)
    selected = fixed_count + k
    per_pos = 2 * model.layers * model.kv_heads * model.head_dim * element_bytes
    dense_kv = per_pos * n
    scanned = n if scan_scope == "all" else cand
    idx_per_pos = model.layers * model.kv_heads * r * ib
    index_read = scanned * idx_per_pos
    selected_kv = selected * per_pos
    return {"n": n, "k": k, "fixed_count": fixed_count, "candidate_count": cand, "selected_count": selected,
            "weights_bytes": model.parameters * element_bytes, "dense_kv_bytes": dense_kv,
            "index_stored_bytes": n * idx_per_pos, "index_read_bytes": index_read, "selected_kv_bytes": selected_kv,
            "d_s1_bytes": index_read + selected_kv, "d_s2_bytes": index_read + 3 * selected_kv,
            "index_parameter_count": model.layers * model.kv_heads * r * ((model.q_heads // model.kv_heads + 1) * model.head_dim)}


def layer_request_bytes(*, G: int, d: int, r: int, M: int, S: int, zb: int, eb: int) -> dict:
    """Algorithmic bytes of one (layer, request) decode step, the same ledger terms per layer:
    score = G*r*M*zb (roofline.py:69-72), attend = S*G*d*2*eb (roofline.py:66,73), d_s1 = score + attend (:74)."""
    score = G * r * M * zb
    attend = S * G * d * 2 * eb
    return {"score_bytes": score, "attend_bytes": attend, "d_s1_bytes": score + attend}


# ---------------------------------------------------------------------------------------------------------------------
# float32 CPU decode step for timing (the reference's own device-agnostic torch path, decode.py:145-163, runs the
# same arithmetic on CPU in float32); used only as the measured CPU baseline
# ---------------------------------------------------------------------------------------------------------------------
def cpu_sparse_request(q, q_pre, K, V, zT, wq_t, wk, k_new, lo: int, hi: int, k: int, L: int, scale: float):
    """One (layer, request) step in float32 on CPU. q, q_pre [G,h,d]; K, V [G,C,d]; zT [G,r,C]; wq_t [G,h*d,r];
    wk [G,r,d]; k_new [G,d]. Writes z of the newest key into zT[:, :, L-1]; returns out [G,h,d]."""
    G, h, d = q.shape
    zT[:, :, L - 1] = np.einsum("gjd,gd->gj", wk, k_new)                              # decode.py:156-157
    u = np.einsum("gf,gfj->gj", q_pre.reshape(G, h * d), wq_t)                         # indexer.py:20-24
    out = np.empty((G, h, d), dtype=np.float32)
    fixed = np.r_[0:lo, hi:L]
    for g in range(G):
        s = u[g] @ zT[g, :, lo:hi]                                                      # indexer.py:27-29
        top = np.argpartition(-s, k - 1)[:k] + lo if 0 < k < s.shape[0] else np.arange(lo, lo + k)   # decode.py:92
        rows = np.concatenate([fixed, top])
        ks, vs = K[g, rows], V[g, rows]                                                 # decode.py:140-141
        sc = (q[g] @ ks.T) * scale                                                      # sparse.py:40-60
        sc -= sc.max(axis=1, keepdims=True)
        p = np.exp(sc)
        p /= p.sum(axis=1, keepdims=True)
        out[g] = p @ vs
    return out


def cpu_prefill_rows(u: np.ndarray, zT: np.ndarray, q_pos0: int, t0: int, t1: int, k: int) -> np.ndarray:
    """float32 timing restatement of prefill_topk for query rows [t0, t1) of one head (u [T,r], zT [r,C]): one
    matmul for the block, then a partial sort per row (np.argpartition; ties are not ordered here, this is the CPU
    baseline's cost model, not a parity oracle). Returns int32 [t1-t0, k]."""
    hi_max = max(0, q_pos0 + t1 - 64)
    s_all = u[t0:t1] @ zT[:, :hi_max]
    out = np.full((t1 - t0, k), -1, dtype=np.int32)
    for i in range(t1 - t0):
        L = q_pos0 + t0 + i + 1
        lo = min(4, L)
        hi = max(lo, L - 64)
        kk = min(k, hi - lo)
        if kk == 0:
            continue
        s = s_all[i, lo:hi]
        part = np.argpartition(-s, kk - 1)[:kk] if kk < hi - lo else np.arange(hi - lo)
        out[i, :kk] = np.sort(part) + lo
    return out
