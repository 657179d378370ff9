"""Drop-in operators for attention-lab's sparse-decode path, backed by the sm_100a C-ABI library.

Names, argument order, argument meaning, return values and exception types follow the reference's operators:

    sparse_decode_step_kernel   decode.py:145-163      fused: z column, u, scores, top-k, F merge, attend
    select_rows_kernel          decode.py:86-93        scores + top-k + F merge -> flat int64 rows [B*G*S]
    gathered_decode_step_kernel decode.py:131-142      attention over listed flat rows, read in place
    dense_decode_step           decode.py:174-176      dense read of [0, valid_length) for one query
    candidate_scores            indexer.py:27-29
    project_keys                indexer.py:15-17
    project_queries             indexer.py:20-24
    append_kvz                  qwen_wrap.py:90-106    the K/V (+ index column) write of LabCache.append

Every tensor must live on a CUDA device; float32 and bfloat16 are supported, head_dim must be 128 and the index
width at most 32. The work is enqueued on the current CUDA stream of the tensors' device and nothing synchronises.
Differences from the reference that do not change results: top-k ties go to the smaller position (torch.topk leaves
them unspecified), and the chosen candidates follow F in ascending position order rather than in descending score
order (the set, and every attention output, is the same; with canonical_order both paths sort every list).
"""
from __future__ import annotations

import math

import ctypes

import torch

from . import _lib

_DTYPES = {torch.float32: _lib.AL_F32, torch.bfloat16: _lib.AL_BF16}
SUBSET_BACKENDS = ("sdpa", "explicit")
FULL_BACKENDS = ("sdpa_fold", "sdpa_gqa", "sdpa_repeat", "explicit")


def _code(t: torch.Tensor, what: str) -> int:
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise ValueError(f"{what} must be float32 or bfloat16 on the CUDA path, got {t.dtype}") from None


def _cuda(*ts):
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("every tensor must live on a CUDA device (the CUDA path has no CPU fallback)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError("all inputs must live on the same device")
    return dev


def _stream(dev) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _ptr(t):
    return None if t is None else t.data_ptr()


def _scale(d: int, scale) -> float:
    return 1.0 / math.sqrt(d) if scale is None else float(scale)


def _check_cache(x: torch.Tensor, what: str):
    if x.dim() != 4:
        raise ValueError(f"{what} must be [B,G,C,d], got {tuple(x.shape)}")
    if not x.is_contiguous():
        raise ValueError(f"{what} must be contiguous so the flattened view is free")


def _q_strides(q: torch.Tensor, what: str):
    if q.dim() != 5:
        raise ValueError(f"{what} must be [B,G,h,T,d], got {tuple(q.shape)}")
    if q.shape[3] != 1:
        raise ValueError("a decode step takes exactly one new query position")
    if q.stride(4) != 1:
        q = q.contiguous()
    return q, q.stride(0), q.stride(1), q.stride(2)


def _check_backend(backend: str, allowed):
    if backend not in allowed:
        raise ValueError(f"unknown backend {backend!r}; choose from {allowed}")


def sparse_decode_step_kernel(q_main, q_pre, k_cache, v_cache, zT, wq_t_scaled, wk, fixed_rows, off_lo, lo: int,
                              hi: int, k: int, selected_count: int, *, k_pre_new=None, write_col: int = -1,
                              scale=None, backend="sdpa", return_rows: bool = False, canonical_order: bool = False,
                              cluster: int = 0, scores_out=None):
    """One layer's D read for one new query (T == 1), as one kernel launch. Writes z of the newest key into
    zT[..., write_col] when k_pre_new is given. Returns out [B,G,h,1,d] (and flat int64 rows [B*G*S] with
    return_rows). `cluster` (CTAs per (batch, group), 0 = automatic) and `scores_out` (fp32 [B,G,hi-lo] scores)
    are extensions for tuning and diagnostics."""
    _check_backend(backend, SUBSET_BACKENDS)
    dev = _cuda(q_main, q_pre, k_cache, v_cache, zT, wq_t_scaled, wk, fixed_rows, off_lo, k_pre_new)
    q_main, qsb, qsg, qsh = _q_strides(q_main, "q_main")
    q_pre, psb, psg, psh = _q_strides(q_pre, "q_pre")
    B, G, h, _, d = q_main.shape
    _check_cache(k_cache, "k_cache")
    _check_cache(v_cache, "v_cache")
    if k_cache.shape != v_cache.shape or k_cache.shape[0] != B or k_cache.shape[1] != G or k_cache.shape[3] != d:
        raise ValueError(f"shape mismatch: q {tuple(q_main.shape)} k {tuple(k_cache.shape)} v {tuple(v_cache.shape)}")
    kv = _code(q_main, "q_main")
    if k_cache.dtype != q_main.dtype or v_cache.dtype != q_main.dtype:
        raise ValueError("q_main, k_cache and v_cache must share one dtype")
    C = k_cache.shape[2]
    if zT.dim() != 4 or zT.shape[0] != B or zT.shape[1] != G or zT.shape[3] != C or not zT.is_contiguous():
        raise ValueError("zT must be a contiguous [B,G,r,C] tensor matching the cache")
    r = zT.shape[2]
    idx = _code(zT, "zT")
    for t, what in ((q_pre, "q_pre"), (wq_t_scaled, "wq_t_scaled"), (wk, "wk"), (k_pre_new, "k_pre_new")):
        if t is not None and t.dtype != zT.dtype:
            raise ValueError(f"{what} must have the index dtype {zT.dtype}, got {t.dtype}")
    if tuple(q_pre.shape) != (B, G, h, 1, d):
        raise ValueError("q_pre must match q_main's shape")
    if tuple(wq_t_scaled.shape) != (G, h * d, r) or tuple(wk.shape) != (G, r, d):
        raise ValueError("wq_t_scaled must be [G,h*d,r] and wk [G,r,d]")
    wq_t_scaled, wk = wq_t_scaled.contiguous(), wk.contiguous()
    F = int(fixed_rows.shape[-1])
    if tuple(fixed_rows.shape) != (B, G, F) or fixed_rows.dtype != torch.int64:
        raise ValueError("fixed_rows must be int64 [B,G,F]")
    if off_lo.numel() != B * G or off_lo.dtype != torch.int64:
        raise ValueError("off_lo must be int64 [B,G,1]")
    fixed_rows, off_lo = fixed_rows.contiguous(), off_lo.contiguous()
    kn_sb = kn_sg = 0
    if k_pre_new is not None:
        if tuple(k_pre_new.shape) != (B, G, 1, d):
            raise ValueError("k_pre_new must be [B,G,1,d]")
        if k_pre_new.stride(3) != 1:
            k_pre_new = k_pre_new.contiguous()
        kn_sb, kn_sg = k_pre_new.stride(0), k_pre_new.stride(1)
    out = torch.empty((B, G, h, 1, d), dtype=q_main.dtype, device=dev)
    rows = torch.empty(B * G * selected_count, dtype=torch.int64, device=dev) if return_rows else None
    if scores_out is not None and (scores_out.dtype != torch.float32 or not scores_out.is_contiguous()
                                   or scores_out.numel() != B * G * max(hi - lo, 0)):
        raise ValueError("scores_out must be a contiguous float32 tensor of B*G*(hi-lo) elements")
    lib = _lib.load()
    with torch.cuda.device(dev):
        _lib.check(lib.al_sparse_decode_step(
            q_main.data_ptr(), qsb, qsg, qsh, q_pre.data_ptr(), psb, psg, psh,
            k_cache.data_ptr(), v_cache.data_ptr(), kv, zT.data_ptr(), wq_t_scaled.data_ptr(), wk.data_ptr(), idx,
            _ptr(k_pre_new), kn_sb, kn_sg, fixed_rows.data_ptr(), off_lo.data_ptr(),
            B, G, h, d, r, C, int(lo), int(hi), int(k), int(selected_count), F, int(write_col),
            _scale(d, scale), int(bool(canonical_order)), out.data_ptr(), _ptr(rows), _ptr(scores_out),
            int(cluster), _stream(dev)))
    return (out, rows) if return_rows else out


def select_rows_kernel(u, zT, fixed_rows, off_lo, lo: int, hi: int, k: int, *, canonical_order: bool = False,
                       cluster: int = 0) -> torch.Tensor:
    """D0 selection: one scan of the candidate columns, one top-k, merge with the fixed rows -> flat rows
    [B*G*S] (decode.py:86-93)."""
    B, G = fixed_rows.shape[:2]
    if k <= 0:
        return fixed_rows.reshape(-1)
    dev = _cuda(u, zT, fixed_rows, off_lo)
    if u.dim() != 4 or u.shape[2] != 1:
        raise ValueError("u must be [B,G,1,r]")
    if zT.dim() != 4 or not zT.is_contiguous() or u.dtype != zT.dtype:
        raise ValueError("zT must be a contiguous [B,G,r,C] tensor of u's dtype")
    idx = _code(zT, "zT")
    r, C = zT.shape[2], zT.shape[3]
    F = int(fixed_rows.shape[-1])
    if fixed_rows.dtype != torch.int64 or off_lo.dtype != torch.int64:
        raise ValueError("fixed_rows and off_lo must be int64")
    u, fixed_rows, off_lo = u.contiguous(), fixed_rows.contiguous(), off_lo.contiguous()
    S = F + int(k)
    rows = torch.empty(B * G * S, dtype=torch.int64, device=dev)
    with torch.cuda.device(dev):
        _lib.check(_lib.load().al_select_rows(
            u.data_ptr(), G * r, r, zT.data_ptr(), idx, fixed_rows.data_ptr(), off_lo.data_ptr(),
            B, G, r, C, int(lo), int(hi), int(k), S, F, int(bool(canonical_order)), rows.data_ptr(), None,
            int(cluster), _stream(dev)))
    return rows


def gathered_decode_step_kernel(q_main, k_cache, v_cache, rows, selected_count: int, *, scale=None, backend="sdpa",
                                cluster: int = 0):
    """Read exactly the listed flat rows of K and V in place and attend over them (decode.py:131-142)."""
    _check_backend(backend, SUBSET_BACKENDS)
    dev = _cuda(q_main, k_cache, v_cache, rows)
    q_main, qsb, qsg, qsh = _q_strides(q_main, "q_main")
    B, G, h, _, d = q_main.shape
    _check_cache(k_cache, "k_cache")
    _check_cache(v_cache, "v_cache")
    if k_cache.dtype != q_main.dtype or v_cache.dtype != q_main.dtype or k_cache.shape != v_cache.shape:
        raise ValueError("q_main, k_cache and v_cache must share one dtype and K/V one shape")
    if rows.dtype != torch.int64 or rows.numel() != B * G * selected_count:
        raise ValueError("rows must be int64 flat row ids [B*G*selected_count]")
    kv = _code(q_main, "q_main")
    rows = rows.contiguous()
    out = torch.empty((B, G, h, 1, d), dtype=q_main.dtype, device=dev)
    with torch.cuda.device(dev):
        _lib.check(_lib.load().al_gathered_attend(
            q_main.data_ptr(), qsb, qsg, qsh, k_cache.data_ptr(), v_cache.data_ptr(), kv, rows.data_ptr(),
            B, G, h, d, k_cache.shape[2], int(selected_count), _scale(d, scale), out.data_ptr(), int(cluster),
            _stream(dev)))
    return out


def dense_decode_step(q_main, k_cache, v_cache, valid_length: int, *, backend="sdpa_fold", scale=None,
                      cluster: int = 0):
    """A read for one new query at the end of the legal range: every position [0, valid_length) (decode.py:174-176,
    full.py:17-45). Every reference backend computes the same function; the CUDA path has one kernel."""
    _check_backend(backend, FULL_BACKENDS)
    dev = _cuda(q_main, k_cache, v_cache)
    q_main, qsb, qsg, qsh = _q_strides(q_main, "q_main")
    B, G, h, _, d = q_main.shape
    _check_cache(k_cache, "k_cache")
    _check_cache(v_cache, "v_cache")
    if k_cache.dtype != q_main.dtype or v_cache.dtype != q_main.dtype or k_cache.shape != v_cache.shape:
        raise ValueError("q_main, k_cache and v_cache must share one dtype and K/V one shape")
    kv = _code(q_main, "q_main")
    out = torch.empty((B, G, h, 1, d), dtype=q_main.dtype, device=dev)
    with torch.cuda.device(dev):
        _lib.check(_lib.load().al_dense_decode(
            q_main.data_ptr(), qsb, qsg, qsh, k_cache.data_ptr(), v_cache.data_ptr(), kv,
            B, G, h, d, k_cache.shape[2], int(valid_length), _scale(d, scale), out.data_ptr(), int(cluster),
            _stream(dev)))
    return out


def project_keys(k_pre: torch.Tensor, wk: torch.Tensor) -> torch.Tensor:
    """k_pre [B,G,C,d], wk [G,r,d] -> zT [B,G,r,C] (indexer.py:15-17), in k_pre's dtype."""
    dev = _cuda(k_pre, wk)
    if k_pre.dim() != 4 or wk.dim() != 3 or k_pre.dtype != wk.dtype:
        raise ValueError("k_pre must be [B,G,C,d] and wk [G,r,d] of one dtype")
    B, G, T, d = k_pre.shape
    r = wk.shape[1]
    idx = _code(k_pre, "k_pre")
    wk = wk.contiguous()
    z = torch.empty((B, G, r, T), dtype=k_pre.dtype, device=dev)
    with torch.cuda.device(dev):
        _lib.check(_lib.load().al_project_keys(k_pre.data_ptr(), _lib.strides(k_pre, 4), wk.data_ptr(), idx,
                                               B, G, T, d, r, z.data_ptr(), T, 0, _stream(dev)))
    return z


def project_queries(q_pre: torch.Tensor, wq_t_scaled: torch.Tensor) -> torch.Tensor:
    """q_pre [B,G,h,T,d], wq_t_scaled [G,h*d,r] -> u [B,G,T,r] (indexer.py:20-24), in q_pre's dtype."""
    dev = _cuda(q_pre, wq_t_scaled)
    if q_pre.dim() != 5 or wq_t_scaled.dim() != 3 or q_pre.dtype != wq_t_scaled.dtype:
        raise ValueError("q_pre must be [B,G,h,T,d] and wq_t_scaled [G,h*d,r] of one dtype")
    B, G, h, T, d = q_pre.shape
    r = wq_t_scaled.shape[2]
    idx = _code(q_pre, "q_pre")
    wq = wq_t_scaled.contiguous()
    u = torch.empty((B, G, T, r), dtype=q_pre.dtype, device=dev)
    with torch.cuda.device(dev):
        _lib.check(_lib.load().al_project_queries(q_pre.data_ptr(), _lib.strides(q_pre, 5), wq.data_ptr(), idx,
                                                  B, G, h, T, d, r, u.data_ptr(), 0, _stream(dev)))
    return u


def candidate_scores(u: torch.Tensor, zT: torch.Tensor, lo: int, hi: int, *, out_dtype=None) -> torch.Tensor:
    """u [B,G,T,r] against the candidate columns only -> [B,G,T,hi-lo] (indexer.py:27-29). Accumulates in fp32;
    the result has u's dtype (as torch.matmul's) unless out_dtype=torch.float32."""
    dev = _cuda(u, zT)
    if u.dim() != 4 or zT.dim() != 4 or not zT.is_contiguous() or u.dtype != zT.dtype:
        raise ValueError("u must be [B,G,T,r] and zT a contiguous [B,G,r,C] tensor of the same dtype")
    B, G, T, r = u.shape
    C = zT.shape[3]
    idx = _code(zT, "zT")
    f32 = out_dtype == torch.float32
    out = torch.empty((B, G, T, max(hi - lo, 0)), dtype=torch.float32 if f32 else u.dtype, device=dev)
    with torch.cuda.device(dev):
        _lib.check(_lib.load().al_candidate_scores(u.data_ptr(), _lib.strides(u, 4), zT.data_ptr(), idx,
                                                   B, G, T, r, C, int(lo), int(hi), out.data_ptr(), int(f32),
                                                   _stream(dev)))
    return out


def append_kvz(k_cache, v_cache, zT, start: int, k_new, v_new, z_new=None, *, k_pre=None, wk=None) -> None:
    """Write T new rows at positions [start, start+T) of K/V [B,G,C,d] and, when given, index columns of zT
    [B,G,r,C]: either the values z_new [B,G,r,T] or Wk . k_pre computed in the same launch sequence (the prefill
    index build). The K/V part of LabCache.append (qwen_wrap.py:90-106)."""
    dev = _cuda(k_cache, v_cache, zT, k_new, v_new, z_new, k_pre, wk)
    _check_cache(k_cache, "k_cache")
    _check_cache(v_cache, "v_cache")
    B, G, C, d = k_cache.shape
    if k_new.dim() != 4 or tuple(k_new.shape[:2]) != (B, G) or k_new.shape[3] != d or v_new.shape != k_new.shape:
        raise ValueError("k_new and v_new must be [B,G,T,d] matching the cache")
    if v_new.dtype != k_new.dtype:
        raise ValueError("k_new and v_new must share one dtype")
    T = k_new.shape[2]
    kv, nd = _code(k_cache, "k_cache"), _code(k_new, "k_new")
    idx, r = 0, 0
    zs = kps = None
    if z_new is not None or k_pre is not None:
        if zT is None:
            raise RuntimeError("this cache was created without an index table")
        idx, r = _code(zT, "zT"), zT.shape[2]
        if z_new is not None:
            if tuple(z_new.shape) != (B, G, r, T) or z_new.dtype != zT.dtype:
                raise ValueError("z_new must be [B,G,r,T] in the index dtype")
            zs = _lib.strides(z_new, 4)
        else:
            if wk is None or k_pre.dtype != zT.dtype or wk.dtype != zT.dtype:
                raise ValueError("k_pre and wk must be given in the index dtype")
            if tuple(k_pre.shape) != (B, G, T, d):
                raise ValueError("k_pre must be [B,G,T,d]")
            wk = wk.contiguous()
            kps = _lib.strides(k_pre, 4)
    with torch.cuda.device(dev):
        _lib.check(_lib.load().al_append_kvz(
            k_cache.data_ptr(), v_cache.data_ptr(), kv, k_new.data_ptr(), _lib.strides(k_new, 4), v_new.data_ptr(),
            _lib.strides(v_new, 4), nd, _ptr(zT), idx, _ptr(z_new), zs, _ptr(k_pre), kps, _ptr(wk),
            B, G, C, d, r, int(start), T, _stream(dev)))


# ---------------------------------------------------------------------------------------------------------------------
# context split across ranks (config C4): the device steps driven by attention_lab_b200.context_split
# ---------------------------------------------------------------------------------------------------------------------
def context_local_topk(q_pre, zT, wq_t_scaled, wk, fixed_rows, off_lo, lo: int, hi: int, k: int, *, key_pos: int,
                       key_stride: int, k_pre_new=None, write_col: int = -1, cluster: int = 0, keys_out=None):
    """Local top-k of one shard's candidates [lo, hi): returns (rows [B,G,F+k] int64: F then the chosen candidates in
    ascending position order, as flat ids of the shard's cache; keys [B,G,key_stride] int64 holding the chosen
    candidates' 64-bit keys (score order key << 32 | 2^32-1 - (key_pos + column)), zero past k). Writes z of the
    newest key into zT[..., write_col] when k_pre_new is given. `keys_out` (int64 [B,G,key_stride], contiguous, e.g. a
    view of a peer-exchange region) receives the keys instead of a new tensor."""
    dev = _cuda(q_pre, zT, wq_t_scaled, wk, fixed_rows, off_lo, k_pre_new)
    q_pre, psb, psg, psh = _q_strides(q_pre, "q_pre")
    B, G, h, _, d = q_pre.shape
    if zT.dim() != 4 or zT.shape[0] != B or zT.shape[1] != G or not zT.is_contiguous():
        raise ValueError("zT must be a contiguous [B,G,r,C] tensor")
    r, C = zT.shape[2], zT.shape[3]
    idx = _code(zT, "zT")
    for t, what in ((q_pre, "q_pre"), (wq_t_scaled, "wq_t_scaled"), (wk, "wk"), (k_pre_new, "k_pre_new")):
        if t is not None and t.dtype != zT.dtype:
            raise ValueError(f"{what} must have the index dtype {zT.dtype}, got {t.dtype}")
    if tuple(wq_t_scaled.shape) != (G, h * d, r) or tuple(wk.shape) != (G, r, d):
        raise ValueError("wq_t_scaled must be [G,h*d,r] and wk [G,r,d]")
    wq_t_scaled, wk = wq_t_scaled.contiguous(), wk.contiguous()
    F = int(fixed_rows.shape[-1])
    if tuple(fixed_rows.shape) != (B, G, F) or fixed_rows.dtype != torch.int64:
        raise ValueError("fixed_rows must be int64 [B,G,F]")
    if off_lo.numel() != B * G or off_lo.dtype != torch.int64:
        raise ValueError("off_lo must be int64 [B,G,1]")
    fixed_rows, off_lo = fixed_rows.contiguous(), off_lo.contiguous()
    kn_sb = kn_sg = 0
    if k_pre_new is not None:
        if tuple(k_pre_new.shape) != (B, G, 1, d):
            raise ValueError("k_pre_new must be [B,G,1,d]")
        if k_pre_new.stride(3) != 1:
            k_pre_new = k_pre_new.contiguous()
        kn_sb, kn_sg = k_pre_new.stride(0), k_pre_new.stride(1)
    rows = torch.empty((B, G, F + k), dtype=torch.int64, device=dev)
    if keys_out is None:
        keys = torch.empty((B, G, key_stride), dtype=torch.int64, device=dev)
    else:
        if tuple(keys_out.shape) != (B, G, key_stride) or keys_out.dtype != torch.int64 or not keys_out.is_contiguous():
            raise ValueError("keys_out must be a contiguous int64 [B,G,key_stride] tensor")
        keys = keys_out
    lib = _lib.load()
    with torch.cuda.device(dev):
        _lib.check(lib.al_context_local_topk(
            q_pre.data_ptr(), psb, psg, psh, zT.data_ptr(), wq_t_scaled.data_ptr(), wk.data_ptr(), idx,
            _ptr(k_pre_new), kn_sb, kn_sg, fixed_rows.data_ptr(), off_lo.data_ptr(),
            B, G, h, r, C, int(lo), int(hi), int(k), F, int(write_col), int(key_pos), int(key_stride),
            rows.data_ptr(), keys.data_ptr(), int(cluster), _stream(dev)))
    return rows, keys


def context_threshold(all_keys, rows, rank: int, k: int, fixed_count: int, k_local: int):
    """rows [B,G,F+k_local] of rank with -1 in place of every candidate below the global k-th key of all_keys
    [world,B,G,key_stride] (every rank's keys from context_local_topk)."""
    dev = _cuda(all_keys, rows)
    if all_keys.dim() != 4 or all_keys.dtype != torch.int64 or not all_keys.is_contiguous():
        raise ValueError("all_keys must be a contiguous int64 [world,B,G,key_stride] tensor")
    world, B, G, kst = all_keys.shape
    if tuple(rows.shape) != (B, G, fixed_count + k_local) or rows.dtype != torch.int64:
        raise ValueError("rows must be int64 [B,G,fixed_count+k_local]")
    rows = rows.contiguous()
    out = torch.empty_like(rows)
    lib = _lib.load()
    with torch.cuda.device(dev):
        _lib.check(lib.al_context_threshold(all_keys.data_ptr(), world, int(rank), B, G, kst, int(k),
                                            int(fixed_count), int(k_local), rows.data_ptr(), out.data_ptr(),
                                            _stream(dev)))
    return out


def gathered_attend_partial(q_main, k_cache, v_cache, rows, *, scale=None, cluster: int = 0, part_out=None):
    """Unnormalised attention partial over rows [B,G,n] (flat ids of the cache, -1 = not read): returns float32
    [B,G,h,130] = (m in the log2 domain, l, acc[128]) per head, for lse_merge (into `part_out` when given)."""
    dev = _cuda(q_main, k_cache, v_cache, rows)
    q_main, qsb, qsg, qsh = _q_strides(q_main, "q_main")
    B, G, h, _, d = q_main.shape
    _check_cache(k_cache, "k_cache")
    _check_cache(v_cache, "v_cache")
    if k_cache.shape != v_cache.shape or k_cache.shape[0] != B or k_cache.shape[1] != G or k_cache.shape[3] != d:
        raise ValueError(f"shape mismatch: q {tuple(q_main.shape)} k {tuple(k_cache.shape)} v {tuple(v_cache.shape)}")
    kv = _code(q_main, "q_main")
    if k_cache.dtype != q_main.dtype or v_cache.dtype != q_main.dtype:
        raise ValueError("q_main, k_cache and v_cache must share one dtype")
    if rows.dtype != torch.int64 or rows.numel() % (B * G) != 0:
        raise ValueError("rows must be int64 with B*G*n elements")
    n = rows.numel() // (B * G)
    rows = rows.contiguous()
    if part_out is None:
        part = torch.empty((B, G, h, d + 2), dtype=torch.float32, device=dev)
    else:
        if tuple(part_out.shape) != (B, G, h, d + 2) or part_out.dtype != torch.float32 or not part_out.is_contiguous():
            raise ValueError("part_out must be a contiguous float32 [B,G,h,d+2] tensor")
        part = part_out
    lib = _lib.load()
    with torch.cuda.device(dev):
        _lib.check(lib.al_gathered_attend_partial(
            q_main.data_ptr(), qsb, qsg, qsh, k_cache.data_ptr(), v_cache.data_ptr(), kv, rows.data_ptr(),
            B, G, h, d, k_cache.shape[2], n, _scale(d, scale), part.data_ptr(), int(cluster), _stream(dev)))
    return part


def lse_merge(all_parts, dtype=torch.bfloat16):
    """Merge partials [world,B,G,h,130] by log-sum-exp into out [B,G,h,1,d] of dtype."""
    dev = _cuda(all_parts)
    if all_parts.dim() != 5 or all_parts.dtype != torch.float32 or not all_parts.is_contiguous():
        raise ValueError("all_parts must be a contiguous float32 [world,B,G,h,d+2] tensor")
    world, B, G, h, d2 = all_parts.shape
    out = torch.empty((B, G, h, 1, d2 - 2), dtype=dtype, device=dev)
    code = _DTYPES.get(dtype)
    if code is None:
        raise ValueError(f"dtype must be float32 or bfloat16, got {dtype}")
    lib = _lib.load()
    with torch.cuda.device(dev):
        _lib.check(lib.al_lse_merge(all_parts.data_ptr(), world, B, G, h, d2 - 2, out.data_ptr(), code, _stream(dev)))
    return out


class _DeviceArray:
    """A raw device pointer seen as an array (`__cuda_array_interface__`), for torch.as_tensor views."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(int(x) for x in shape), "typestr": typestr,
                                         "data": (int(ptr), False), "version": 3, "strides": None}


def device_view(ptr: int, shape, dtype, device) -> torch.Tensor:
    """A tensor over device memory the library allocated (no copy; the memory must outlive the tensor)."""
    typestr = {torch.int64: "<i8", torch.float32: "<f4", torch.int32: "<i4"}[dtype]
    with torch.cuda.device(device):
        return torch.as_tensor(_DeviceArray(ptr, shape, typestr), device=device)


def xchg_create(nbytes: int, device) -> tuple:
    """A zero-filled exchange region of nbytes on `device` (al_xchg_create): (address, 64-byte CUDA IPC handle)."""
    lib = _lib.load()
    region, handle = ctypes.c_void_p(), (ctypes.c_char * 64)()
    with torch.cuda.device(device):
        _lib.check(lib.al_xchg_create(int(nbytes), ctypes.byref(region), handle))
    return int(region.value), bytes(handle)


def xchg_open(handle: bytes, device) -> int:
    """Map a peer's exchange region from its handle (al_xchg_open); returns its address in this process."""
    if len(handle) != 64:
        raise ValueError("an exchange handle is 64 bytes")
    lib = _lib.load()
    ptr = ctypes.c_void_p()
    with torch.cuda.device(device):
        _lib.check(lib.al_xchg_open(ctypes.create_string_buffer(handle, 64), ctypes.byref(ptr)))
    return int(ptr.value)


def xchg_close(ptr: int, device) -> None:
    with torch.cuda.device(device):
        _lib.check(_lib.load().al_xchg_close(ctypes.c_void_p(ptr)))


def xchg_destroy(ptr: int, device) -> None:
    with torch.cuda.device(device):
        _lib.check(_lib.load().al_xchg_destroy(ctypes.c_void_p(ptr)))


def xchg_push(src: torch.Tensor, dst, rank: int, done: int, counter: int, peer_flags) -> None:
    """Copy src (contiguous, a multiple of 16 bytes) into slot `rank` of every rank's gather area (dst: int64 device
    tensor of the ranks' gather-area addresses), then publish this rank's next epoch of the channel to every peer
    (al_xchg_push)."""
    dev = _cuda(src, dst, peer_flags)
    if not src.is_contiguous():
        raise ValueError("the pushed tensor must be contiguous")
    with torch.cuda.device(dev):
        _lib.check(_lib.load().al_xchg_push(src.data_ptr(), src.numel() * src.element_size(), dst.data_ptr(),
                                            dst.numel(), int(rank), ctypes.c_void_p(done), ctypes.c_void_p(counter),
                                            peer_flags.data_ptr(), _stream(dev)))


def context_threshold_peer(gather, flags: int, counter: int, rows, rank: int, k: int, fixed_count: int, k_local: int,
                           *, spin: int = 1 << 22):
    """context_threshold over this rank's gather area of keys [world,B,G,key_stride] (filled by the ranks' xchg_push)
    once every peer's flag has reached this rank's epoch (bounded wait)."""
    dev = _cuda(gather, rows)
    if gather.dim() != 4 or gather.dtype != torch.int64 or not gather.is_contiguous():
        raise ValueError("gather must be a contiguous int64 [world,B,G,key_stride] tensor")
    world, B, G, kst = gather.shape
    if tuple(rows.shape) != (B, G, fixed_count + k_local) or rows.dtype != torch.int64:
        raise ValueError("rows must be int64 [B,G,fixed_count+k_local]")
    rows = rows.contiguous()
    out = torch.empty_like(rows)
    with torch.cuda.device(dev):
        _lib.check(_lib.load().al_context_threshold_peer(
            gather.data_ptr(), ctypes.c_void_p(flags), ctypes.c_void_p(counter), int(spin), world, int(rank), B, G,
            kst, int(k), int(fixed_count), int(k_local), rows.data_ptr(), out.data_ptr(), _stream(dev)))
    return out


def lse_merge_peer(gather, flags: int, counter: int, rank: int, dtype=torch.bfloat16, *, spin: int = 1 << 22):
    """lse_merge over this rank's gather area of partials [world,B,G,h,d+2] once every peer's flag has reached this
    rank's epoch (bounded wait). Returns [B,G,h,1,d] of dtype."""
    dev = _cuda(gather)
    if gather.dim() != 5 or gather.dtype != torch.float32 or not gather.is_contiguous():
        raise ValueError("gather must be a contiguous float32 [world,B,G,h,d+2] tensor")
    world, B, G, h, d2 = gather.shape
    code = _DTYPES.get(dtype)
    if code is None:
        raise ValueError(f"dtype must be float32 or bfloat16, got {dtype}")
    out = torch.empty((B, G, h, 1, d2 - 2), dtype=dtype, device=dev)
    with torch.cuda.device(dev):
        _lib.check(_lib.load().al_lse_merge_peer(
            gather.data_ptr(), ctypes.c_void_p(flags), ctypes.c_void_p(counter), int(spin), world, int(rank), B, G, h,
            d2 - 2, out.data_ptr(), code, _stream(dev)))
    return out


def prefill_score_topk(u: torch.Tensor, zT: torch.Tensor, k: int = 256, *, q_pos0: int = 0, kcap=None,
                       scores_out=None) -> torch.Tensor:
    """Batched prefill scorer (config C5): for every query row t of a prefill chunk (position q_pos0 + t) and every
    KV head, the top min(k, M) candidates of a decode step at legal length q_pos0 + t + 1 (selection.py:71-79,
    decode.py:86-93, ties to the smaller position) under the scores u[h, t] . zT[h, :, c].

    u [H,T,r] bf16 and zT [H,r,C] bf16 (last dims contiguous; r = 32). Returns int32 [H,T,kcap] (kcap defaults to
    k): the chosen positions in ascending order, then -1. `scores_out` (fp32 [H,T,C], contiguous) receives the
    scores of the candidate columns, for diagnostics."""
    dev = _cuda(u, zT, scores_out)
    if u.dim() != 3 or zT.dim() != 3 or u.dtype != torch.bfloat16 or zT.dtype != torch.bfloat16:
        raise ValueError("u must be bf16 [H,T,r] and zT bf16 [H,r,C]")
    if u.stride(2) != 1 or zT.stride(2) != 1:
        raise ValueError("u and zT need a contiguous last dimension")
    H, T, r = u.shape
    if zT.shape[0] != H or zT.shape[1] != r:
        raise ValueError(f"zT {tuple(zT.shape)} does not match u {tuple(u.shape)}")
    C = zT.shape[2]
    kcap = int(k) if kcap is None else int(kcap)
    if scores_out is not None and (scores_out.shape != (H, T, C) or scores_out.dtype != torch.float32
                                   or not scores_out.is_contiguous()):
        raise ValueError("scores_out must be a contiguous float32 [H,T,C] tensor")
    out = torch.empty((H, T, kcap), dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        _lib.check(_lib.load().al_prefill_score_topk(u.data_ptr(), u.stride(0), u.stride(1), zT.data_ptr(), zT.stride(0),
                                                     zT.stride(1), H, T, C, r, int(q_pos0), int(k), kcap,
                                                     out.data_ptr(), _ptr(scores_out), _stream(dev)))
    return out
