"""Qwen3 decode driver on the B200 kernels: attention-lab's Qwen3 wrapper (src/attention_lab/qwen_wrap.py) rebuilt
on this library's C ABI, with the reference's interface.

A wrapped model keeps every module of the installed transformers Qwen3 (embeddings, q/k/v/o projections, q_norm and
k_norm, the model's own RoPE, MLPs, norms, lm_head); only each layer's attention read changes, as in the reference:

    hidden -> q/k/v proj -> q_norm/k_norm -> (q_pre, k_pre: index features, before RoPE) -> RoPE -> (q_main, k_main)
           -> append k_main, v (and z = Wk . k_pre) once -> read -> o_proj

What runs where:

    append              al_append_kvz: K/V rows at [valid_length, +T); with an index table and k_pre also the index
                        columns z = Wk . k_pre, computed on the device in the same call (prefill and full decode)
    sparse decode (D0)  al_sparse_decode_step: the newest key's z column, u, candidate scores, top-k, F merge and the
                        gather-free attention, one launch per layer
    selectors B / C     their row lists (selection rules of decode.py:94-127), then al_gathered_attend
    full decode (A)     al_dense_decode over [0, legal length) (or torch SDPA, decode_backend="sdpa_fold")
    prefill read        torch scaled_dot_product_attention over [0, L0 + T) with the legality mask (a dense,
                        compute-bound read outside the decode hot path; full.py:17-45 sdpa_fold semantics)

Positions are original: a token's slot is its absolute position, rows are read in place and never renumbered, z is
built from the pre-RoPE k. The legal range grows by one per decode step; after a rollback the old suffix stays in
memory but lies outside the legal range. The caches and the model must live on a CUDA device: the kernels have no
CPU path.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import nn

from . import ops
from .selection import FIXED_PREFIX, FIXED_RECENT, fixed_budget, row_offsets, selection_layout

try:  # transformers is needed by the wrapper only; the operators import without it
    from transformers.models.qwen3.modeling_qwen3 import apply_rotary_pos_emb
except ImportError as _e:  # pragma: no cover
    apply_rotary_pos_emb = None
    _TRANSFORMERS_IMPORT_ERROR = _e

# Qwen3Model.forward skips its causal-mask construction when the mask argument is already a dict (the read here
# applies its own legality rules).
MASK_BYPASS = {"full_attention": None}
SELECTORS = ("index", "recent", "uniform")   # D0 / B / C
# full-mode decode read: this library's dense kernel, or torch SDPA with the heads folded (the reference's A path,
# full.py:31-34), kept as the same-box dense baseline
DECODE_BACKENDS = ("kernel", "sdpa_fold")


# ---------------------------------------------------------------------------------------------------------------------
# static cache
# ---------------------------------------------------------------------------------------------------------------------
class LabCache:
    """Preallocated per-layer K/V [B,G,C,d] and (optionally) index tables zT [B,G,r,C] on the device; one legal
    length for all layers (qwen_wrap.py:46-143). Unwritten slots hold whatever the allocator left there: no read or
    selection ever touches a slot at or beyond valid_length."""

    def __init__(self, *, layers: int, batch: int, groups: int, capacity: int, head_dim: int, index_dim=None, device,
                 dtype=torch.bfloat16, index_dtype=None):
        if int(capacity) <= 0 or int(layers) <= 0:
            raise ValueError("capacity and layers must be positive")
        self.layers, self.batch, self.groups = int(layers), int(batch), int(groups)
        self.capacity, self.head_dim = int(capacity), int(head_dim)
        self.index_dim = None if index_dim is None else int(index_dim)
        self.device, self.dtype = torch.device(device), dtype
        self.index_dtype = dtype if index_dtype is None else index_dtype
        shape = (self.batch, self.groups, self.capacity, self.head_dim)
        self.k = [torch.empty(shape, device=self.device, dtype=dtype) for _ in range(self.layers)]
        self.v = [torch.empty(shape, device=self.device, dtype=dtype) for _ in range(self.layers)]
        self.z = None if self.index_dim is None else [
            torch.empty((self.batch, self.groups, self.index_dim, self.capacity), device=self.device,
                        dtype=self.index_dtype) for _ in range(self.layers)]
        self.valid_length = 0
        self.offsets = row_offsets(self.batch, self.groups, self.capacity, self.device)            # [B,G,1]
        self.prefix_rows = (torch.arange(FIXED_PREFIX, device=self.device).view(1, 1, -1) + self.offsets).contiguous()
        self.recent_base = (torch.arange(-FIXED_RECENT, 0, device=self.device).view(1, 1, -1)
                            + self.offsets).contiguous()
        self.off_lo = (self.offsets + FIXED_PREFIX).contiguous()
        self.writes = [0] * self.layers
        self.last_write = [None] * self.layers
        self._pending = None

    @property
    def has_index(self) -> bool:
        return self.z is not None

    def append(self, layer: int, k_main: torch.Tensor, v: torch.Tensor, z=None, *, k_pre=None, wk=None) -> None:
        """Write this layer's new rows at [valid_length, valid_length + T): K/V, and the index columns either from z
        ([B,G,r,T]) or built on the device from k_pre ([B,G,T,d]) and wk. Exactly once per layer per forward."""
        start, T = self.valid_length, int(k_main.shape[2])
        if start + T > self.capacity:
            raise RuntimeError(f"cache capacity {self.capacity} exceeded: valid {start} + new {T}")
        if self._pending is None:
            self._pending = T
        elif self._pending != T:
            raise RuntimeError("layers appended different lengths within one forward")
        wants_z = z is not None or k_pre is not None
        if wants_z and self.z is None:
            ops.append_kvz(self.k[layer], self.v[layer], None, start, k_main, v)
            raise RuntimeError("this cache was created without an index table")
        zt = self.z[layer] if wants_z else None
        ops.append_kvz(self.k[layer], self.v[layer], zt, start, k_main, v,
                       None if z is None else z.to(zt.dtype),
                       k_pre=None if k_pre is None else k_pre.to(zt.dtype),
                       wk=None if k_pre is None else wk)
        self.writes[layer] += 1
        self.last_write[layer] = (start, T)

    def advance(self, T: int) -> None:
        """Commit a forward of T tokens after every layer appended exactly once."""
        if self._pending != int(T):
            raise RuntimeError(f"advance({T}) does not match the appended length {self._pending}")
        if any(w != self.writes[0] for w in self.writes):
            raise RuntimeError(f"unequal append counts across layers: {self.writes}")
        self.valid_length += int(T)
        self._pending = None

    def rollback(self, length: int) -> None:
        """Shrink the legal range; the old suffix stays in memory and can neither be read nor selected."""
        if not 0 <= int(length) <= self.valid_length:
            raise ValueError(f"rollback to {length} outside [0, {self.valid_length}]")
        if self._pending is not None:
            raise RuntimeError("rollback during a forward")
        self.valid_length = int(length)

    def clone(self) -> "LabCache":
        """An independent copy (a request branch): device copies of every buffer, no shared storage."""
        new = LabCache.__new__(LabCache)
        new.__dict__.update({k: v for k, v in self.__dict__.items() if k not in ("k", "v", "z", "writes", "last_write")})
        new.k = [t.clone() for t in self.k]
        new.v = [t.clone() for t in self.v]
        new.z = None if self.z is None else [t.clone() for t in self.z]
        new.writes, new.last_write = list(self.writes), list(self.last_write)
        return new

    def bytes(self) -> dict:
        es = self.k[0].element_size()
        kv = self.layers * 2 * self.batch * self.groups * self.capacity * self.head_dim * es
        z = 0 if self.z is None else (self.layers * self.batch * self.groups * self.index_dim * self.capacity
                                      * self.z[0].element_size())
        return {"kv_bytes": kv, "index_bytes": z, "total_bytes": kv + z}


# ---------------------------------------------------------------------------------------------------------------------
# per-step plan
# ---------------------------------------------------------------------------------------------------------------------
@dataclass
class StepPlan:
    """One decode step's selection constants, shared by every layer (qwen_wrap.py:145-163)."""

    legal_length: int
    k0: int
    k: int
    lo: int
    hi: int
    fixed_count: int
    selected_count: int
    fixed_rows: torch.Tensor      # [B,G,F] flat rows
    off_lo: torch.Tensor          # [B,G,1]
    step_index: int = 0
    shared_rows: torch.Tensor | None = None   # selector B: one row list for every layer of the step
    uniform_rng: object | None = None         # selector C: this step's generator

    @property
    def write_col(self) -> int:
        return self.legal_length - 1

    @property
    def candidate_count(self) -> int:
        return self.hi - self.lo


def build_step_plan(cache: LabCache, legal_length: int, k0: int) -> StepPlan:
    """F and the candidate domain for a step whose legal range is [0, legal_length); from legal length 68 on, F's
    rows are derived from the cache's preallocated row tensors on the device (no host-to-device copy)."""
    lay = selection_layout(legal_length)
    k = lay.clamp_k(k0)
    if lay.fixed_prefix == FIXED_PREFIX and lay.recent_start == legal_length - FIXED_RECENT:
        fixed_rows = torch.cat([cache.prefix_rows, cache.recent_base + legal_length], dim=-1)
        off_lo = cache.off_lo
    else:
        pos = torch.tensor(lay.fixed_positions(), dtype=torch.long, device=cache.device).view(1, 1, -1)
        fixed_rows = (pos + cache.offsets).contiguous()
        off_lo = (cache.offsets + lay.candidate_lo).contiguous()
    return StepPlan(legal_length=int(legal_length), k0=int(k0), k=int(k), lo=lay.candidate_lo, hi=lay.candidate_hi,
                    fixed_count=lay.fixed_count, selected_count=lay.fixed_count + k, fixed_rows=fixed_rows,
                    off_lo=off_lo)


def select_rows_recent(fixed_rows, off_lo, lo: int, hi: int, k: int) -> torch.Tensor:
    """Selector B: F, then the k most recent candidates [hi - k, hi) as flat rows (decode.py:96-107)."""
    B, G = fixed_rows.shape[:2]
    if k <= 0:
        return fixed_rows.reshape(-1)
    M = hi - lo
    if k > M:
        raise ValueError(f"k={k} exceeds the candidate count {M}")
    rel = torch.arange(M - k, M, device=fixed_rows.device, dtype=torch.long).view(1, 1, k).expand(B, G, k)
    return torch.cat([fixed_rows, rel + off_lo], dim=-1).reshape(-1)


def select_rows_uniform(fixed_rows, off_lo, lo: int, hi: int, k: int, *, rng) -> torch.Tensor:
    """Selector C: F, then k candidates drawn uniformly without replacement per (batch, group): the top-k of i.i.d.
    float64 uniforms drawn [B,G,M] in one call from the numpy generator `rng` (decode.py:110-127)."""
    import numpy as np
    B, G = fixed_rows.shape[:2]
    if k <= 0:
        return fixed_rows.reshape(-1)
    M = hi - lo
    if k > M:
        raise ValueError(f"k={k} exceeds the candidate count {M}")
    u = torch.from_numpy(rng.random((B, G, M), dtype=np.float64))
    rel = torch.topk(u, k, dim=-1).indices.to(fixed_rows.device)
    return torch.cat([fixed_rows, rel + off_lo], dim=-1).reshape(-1)


# ---------------------------------------------------------------------------------------------------------------------
# indexers and state
# ---------------------------------------------------------------------------------------------------------------------
class Indexer:
    """One layer's untrained grouped indexer (indexer.py:30-45): wq [G,r,h*d] and wk [G,r,d] drawn N(0, init_std^2)
    in float64 on the CPU from torch.Generator(seed), then cast once; wq_t_scaled = (wq / sqrt(r))^T."""

    def __init__(self, groups: int, heads_per_group: int, head_dim: int, r: int = 32, *, device, dtype,
                 seed: int = 0, init_std: float = 0.02):
        gen = torch.Generator().manual_seed(int(seed))
        wq = torch.randn(groups, r, heads_per_group * head_dim, generator=gen, dtype=torch.float64) * init_std
        wk = torch.randn(groups, r, head_dim, generator=gen, dtype=torch.float64) * init_std
        self.r = int(r)
        self.wq = wq.to(device=device, dtype=dtype)
        self.wk = wk.to(device=device, dtype=dtype)
        self.wq_t_scaled = (wq / math.sqrt(r)).transpose(1, 2).contiguous().to(device=device, dtype=dtype)


class LabState:
    """One read configuration: the cache, optional indexers, the mode (full | sparse), the sparse selector
    (index = D0, recent = B, uniform = C) and the plan of the step in flight (qwen_wrap.py:189-240)."""

    def __init__(self, cache: LabCache, indexers=None, *, mode: str = "full", selector: str = "index",
                 uniform_seed: int = 0, sparse_layers=None, cache_guard=None, canonical_order=False,
                 decode_backend: str = "kernel"):
        if mode not in ("full", "sparse"):
            raise ValueError("mode must be 'full' or 'sparse'")
        if decode_backend not in DECODE_BACKENDS:
            raise ValueError(f"decode_backend must be one of {DECODE_BACKENDS}")
        self.decode_backend = decode_backend
        if selector not in SELECTORS:
            raise ValueError(f"selector must be one of {SELECTORS}")
        if mode == "sparse" and selector == "index" and (indexers is None or not cache.has_index):
            raise ValueError("the index selector (D0) needs indexers and a cache with an index table")
        if indexers is not None and len(indexers) != cache.layers:
            raise ValueError("one indexer per layer")
        self.cache, self.indexers, self.mode, self.selector = cache, indexers, mode, selector
        self.sparse_layers = None if sparse_layers is None else frozenset(sparse_layers)
        if self.sparse_layers is not None and not self.sparse_layers.issubset(range(cache.layers)):
            raise ValueError("sparse layer index outside model")
        self.cache_guard = cache_guard
        self.canonical_order = bool(canonical_order)
        self.uniform_seed = int(uniform_seed)
        self.request_counter = 0
        self.record_selection = False
        self.last_rows: list = [None] * cache.layers
        self.plan: StepPlan | None = None
        self.phase: str | None = None
        self.rho = None
        self.k0 = None
        self.request_start_length = None

    def uniform_rng(self, step_index: int):
        """Selector C's generator for one step: numpy default_rng([uniform_seed, request_counter, step_index])."""
        import numpy as np
        return np.random.default_rng([self.uniform_seed, self.request_counter, int(step_index)])

    def begin_request(self, rho, *, k0=None) -> int:
        """Fix k0 from the legal length of the first decode step (the prefilled tokens plus the new one); `k0`
        overrides the rho rule (k is still clamped to the candidate count at every step)."""
        self.rho = None if rho is None else float(rho)
        self.request_start_length = self.cache.valid_length + 1
        self.k0 = fixed_budget(self.request_start_length, self.rho) if k0 is None else int(k0)
        self.request_counter += 1
        return self.k0


class StateHolder:
    """Mutable pointer so one wrapped model can alternate between read configurations."""

    def __init__(self, state: LabState | None = None):
        self.state = state


# ---------------------------------------------------------------------------------------------------------------------
# the attention module
# ---------------------------------------------------------------------------------------------------------------------
def prefill_attention(q5: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, start: int, scale: float):
    """Queries at positions start .. start + T - 1 over keys [0, start + T) with key j legal for query p when
    j <= p; the h heads of a group folded into the query axis (full.py:31-34). q5 [B,G,h,T,d] -> [B,G,h,T,d]."""
    B, G, h, T, d = q5.shape
    n = start + T
    qpos = torch.arange(start, n, device=q5.device)
    legal = torch.arange(n, device=q5.device).view(1, n) <= qpos.view(T, 1)                 # [T, n]
    mask = legal.repeat(h, 1).view(1, 1, h * T, n)
    out = F.scaled_dot_product_attention(q5.reshape(B, G, h * T, d), k_cache[:, :, :n], v_cache[:, :, :n],
                                         attn_mask=mask, scale=scale)
    return out.reshape(B, G, h, T, d)


class LabAttention(nn.Module):
    """Replacement for one Qwen3Attention (qwen_wrap.py:243-326): the original module's projections, norms and RoPE
    are reused as they are; only the read differs. `inner` is the original module object."""

    def __init__(self, inner: nn.Module, holder: StateHolder, layer_idx: int):
        super().__init__()
        if apply_rotary_pos_emb is None:  # pragma: no cover
            raise _TRANSFORMERS_IMPORT_ERROR
        self.inner, self.holder, self.layer_idx = inner, holder, int(layer_idx)
        cfg = inner.config
        self.num_heads = int(cfg.num_attention_heads)
        self.num_groups = int(cfg.num_key_value_heads)
        self.head_dim = int(inner.head_dim)
        if self.num_heads % self.num_groups:
            raise ValueError("query heads must be a multiple of KV heads")
        self.heads_per_group = self.num_heads // self.num_groups
        self.scaling = float(inner.scaling)
        self.is_causal = True

    def forward(self, hidden_states, position_embeddings, attention_mask=None, past_key_values=None, **kwargs):
        inner, st = self.inner, self.holder.state
        if st is None:
            raise RuntimeError("no LabState set on the wrapped model")
        B, T, _ = hidden_states.shape
        d, G, h = self.head_dim, self.num_groups, self.heads_per_group
        shape = (B, T, -1, d)
        q_pre = inner.q_norm(inner.q_proj(hidden_states).view(shape)).transpose(1, 2)   # [B,H,T,d], before RoPE
        k_pre = inner.k_norm(inner.k_proj(hidden_states).view(shape)).transpose(1, 2)   # [B,G,T,d], before RoPE
        v = inner.v_proj(hidden_states).view(shape).transpose(1, 2)
        cos, sin = position_embeddings
        q_main, k_main = apply_rotary_pos_emb(q_pre, k_pre, cos, sin)
        cache, l = st.cache, self.layer_idx
        L0 = cache.valid_length
        q5 = q_main.view(B, G, h, T, d)                          # query head g*h + i reads group g
        idx = st.indexers[l] if st.indexers is not None else None
        build_z = cache.has_index and idx is not None
        if st.phase not in ("prefill", "decode"):
            raise RuntimeError("LabState.phase must be 'prefill' or 'decode' (set by LabRunner.prefill / "
                               "LabRunner.step); the phase is never inferred from the input length")
        if st.phase == "decode":
            if T != 1:
                raise RuntimeError("a decode step takes exactly one new token")
            if st.mode == "sparse" and (st.sparse_layers is None or l in st.sparse_layers):
                plan = st.plan
                if plan is None or plan.legal_length != L0 + 1:
                    raise RuntimeError("sparse decode needs a StepPlan built for this step's legal length")
                cache.append(l, k_main, v)          # K/V; the newest key's z column is written by the fused kernel
                if st.selector == "index":
                    zd = cache.z[l].dtype
                    out, rows = ops.sparse_decode_step_kernel(
                        q5, q_pre.view(B, G, h, 1, d).to(zd), cache.k[l], cache.v[l], cache.z[l], idx.wq_t_scaled,
                        idx.wk, plan.fixed_rows, plan.off_lo, plan.lo, plan.hi, plan.k, plan.selected_count,
                        k_pre_new=k_pre.to(zd), write_col=plan.write_col, scale=self.scaling,
                        return_rows=True, canonical_order=st.canonical_order)
                else:
                    if st.selector == "recent":
                        rows = plan.shared_rows
                    else:
                        rows = select_rows_uniform(plan.fixed_rows, plan.off_lo, plan.lo, plan.hi, plan.k,
                                                   rng=plan.uniform_rng)
                    if st.canonical_order:
                        rows = rows.view(B, G, plan.selected_count).sort(dim=-1).values.reshape(-1)
                    out = ops.gathered_decode_step_kernel(q5, cache.k[l], cache.v[l], rows, plan.selected_count,
                                                          scale=self.scaling)
                if st.record_selection:
                    st.last_rows[l] = rows
            else:
                cache.append(l, k_main, v, k_pre=k_pre if build_z else None, wk=idx.wk if build_z else None)
                if st.decode_backend == "kernel":
                    out = ops.dense_decode_step(q5, cache.k[l], cache.v[l], L0 + 1, scale=self.scaling)
                else:
                    out = F.scaled_dot_product_attention(q5.reshape(B, G, h, d), cache.k[l][:, :, :L0 + 1],
                                                         cache.v[l][:, :, :L0 + 1], scale=self.scaling)
        else:   # prefill: every legal position is read whatever the chunk size; the index table is filled on the way
            cache.append(l, k_main, v, k_pre=k_pre if build_z else None, wk=idx.wk if build_z else None)
            out = prefill_attention(q5, cache.k[l], cache.v[l], L0, self.scaling)
        attn = out.reshape(B, self.num_heads, T, d).transpose(1, 2).reshape(B, T, self.num_heads * d)
        return inner.o_proj(attn), None


# ---------------------------------------------------------------------------------------------------------------------
# geometry, construction, wrap / unwrap
# ---------------------------------------------------------------------------------------------------------------------
@dataclass(frozen=True)
class ModelGeometry:
    layers: int
    hidden: int
    heads: int
    groups: int
    head_dim: int
    vocab: int
    max_positions: int

    @property
    def heads_per_group(self) -> int:
        return self.heads // self.groups


def _attention_module(layer):
    return layer.self_attn.inner if isinstance(layer.self_attn, LabAttention) else layer.self_attn


def geometry_of(model) -> ModelGeometry:
    """The geometry from the config, checked against the parameter shapes."""
    cfg = model.config
    attn = _attention_module(model.model.layers[0])
    heads, groups = int(cfg.num_attention_heads), int(cfg.num_key_value_heads)
    head_dim, hidden = int(attn.head_dim), int(cfg.hidden_size)
    expect = {"q_proj": (heads * head_dim, hidden), "k_proj": (groups * head_dim, hidden),
              "v_proj": (groups * head_dim, hidden), "o_proj": (hidden, heads * head_dim)}
    for name, want in expect.items():
        got = tuple(getattr(attn, name).weight.shape)
        if got != want:
            raise ValueError(f"{name} weight shape {got} != {want} implied by the config")
    return ModelGeometry(layers=len(model.model.layers), hidden=hidden, heads=heads, groups=groups, head_dim=head_dim,
                         vocab=int(cfg.vocab_size), max_positions=int(cfg.max_position_embeddings))


def make_cache(model, capacity: int, *, with_index: bool, index_dim: int = 32, batch: int = 1, dtype=None,
               device=None, index_dtype=None) -> LabCache:
    geo = geometry_of(model)
    p = next(model.parameters())
    return LabCache(layers=geo.layers, batch=batch, groups=geo.groups, capacity=capacity, head_dim=geo.head_dim,
                    index_dim=index_dim if with_index else None, device=p.device if device is None else device,
                    dtype=p.dtype if dtype is None else dtype, index_dtype=index_dtype)


def make_indexers(model, *, r: int = 32, seed: int = 0, dtype=None, device=None) -> list[Indexer]:
    """One untrained grouped indexer per layer, seeded seed * 1000 + layer (qwen_wrap.py:376-381)."""
    geo = geometry_of(model)
    p = next(model.parameters())
    return [Indexer(geo.groups, geo.heads_per_group, geo.head_dim, r, device=p.device if device is None else device,
                    dtype=p.dtype if dtype is None else dtype, seed=seed * 1000 + i) for i in range(geo.layers)]


def make_state(model, capacity: int, mode: str, *, selector: str = "index", r: int = 32, seed: int = 0,
               batch: int = 1, index_dtype=None, **kw) -> LabState:
    """A: mode "full". D0: mode "sparse" (index table + indexers). B / C: mode "sparse" with selector "recent" /
    "uniform" (no index table)."""
    with_index = mode == "sparse" and selector == "index"
    cache = make_cache(model, capacity, with_index=with_index, index_dim=r, batch=batch, index_dtype=index_dtype)
    idx = make_indexers(model, r=r, seed=seed, dtype=cache.index_dtype) if with_index else None
    return LabState(cache, idx, mode=mode, selector=selector, **kw)


def wrap_model(model, holder: StateHolder | None = None) -> StateHolder:
    """Replace every layer's self_attn with LabAttention around the original module; returns the shared holder."""
    holder = StateHolder() if holder is None else holder
    for i, layer in enumerate(model.model.layers):
        if isinstance(layer.self_attn, LabAttention):
            raise RuntimeError("model is already wrapped")
        layer.self_attn = LabAttention(layer.self_attn, holder, i)
    return holder


def unwrap_model(model) -> None:
    for layer in model.model.layers:
        if isinstance(layer.self_attn, LabAttention):
            layer.self_attn = layer.self_attn.inner


def is_wrapped(model) -> bool:
    return isinstance(model.model.layers[0].self_attn, LabAttention)


# ---------------------------------------------------------------------------------------------------------------------
# the driver
# ---------------------------------------------------------------------------------------------------------------------
class LabRunner:
    """Prefill / decode driver for a wrapped model and one LabState (qwen_wrap.py:410-486). Every forward goes through
    the model's own entry (embeddings -> layers -> norm -> lm_head); position ids are views of one preallocated
    device arange."""

    def __init__(self, model, holder: StateHolder, state: LabState):
        if not is_wrapped(model):
            raise RuntimeError("wrap_model first")
        self.model, self.holder, self.state = model, holder, state
        self.positions = torch.arange(state.cache.capacity, device=state.cache.device)

    @property
    def cache(self) -> LabCache:
        return self.state.cache

    def forward(self, input_ids: torch.Tensor, *, phase: str, logits_to_keep: int = 1) -> torch.Tensor:
        """One model forward. `phase` is explicit: "prefill" reads every legal position and fills the index table
        (any chunk size, one token included); "decode" is one new token read by the state's mode."""
        if phase not in ("prefill", "decode"):
            raise ValueError("phase must be 'prefill' or 'decode'")
        st, cache = self.state, self.state.cache
        if st.cache_guard is not None:
            st.cache_guard(st)
        B, T = input_ids.shape
        if B != cache.batch:
            raise ValueError("batch size differs from the cache")
        start = cache.valid_length
        st.phase = phase
        st.plan = None
        if phase == "decode":
            if T != 1:
                raise ValueError("a decode step takes exactly one token per sequence")
            if st.mode == "sparse":
                if st.k0 is None:
                    raise RuntimeError("call state.begin_request(rho) before the first sparse decode step")
                st.plan = build_step_plan(cache, start + 1, st.k0)
                st.plan.step_index = start + 1 - st.request_start_length
                if st.selector == "recent":
                    st.plan.shared_rows = select_rows_recent(st.plan.fixed_rows, st.plan.off_lo, st.plan.lo,
                                                             st.plan.hi, st.plan.k)
                elif st.selector == "uniform":
                    st.plan.uniform_rng = st.uniform_rng(st.plan.step_index)
        self.holder.state = st
        out = self.model(input_ids=input_ids, position_ids=self.positions[start:start + T].unsqueeze(0),
                         attention_mask=MASK_BYPASS, use_cache=False, logits_to_keep=logits_to_keep)
        cache.advance(T)
        return out.logits

    def prefill(self, input_ids: torch.Tensor, chunk: int, *, keep_logits: bool = False):
        """Dense prefill in chunks; the index table is filled chunk by chunk when the cache has one."""
        T = input_ids.shape[1]
        if chunk <= 0:
            raise ValueError("chunk must be positive")
        outs, logits = [], None
        for a in range(0, T, chunk):
            logits = self.forward(input_ids[:, a:a + chunk], phase="prefill", logits_to_keep=0 if keep_logits else 1)
            if keep_logits:
                outs.append(logits)
        return torch.cat(outs, dim=1) if keep_logits else logits

    def step(self, token_ids: torch.Tensor) -> torch.Tensor:
        """One decode step: token ids [B,1] -> next-token scores [B,1,V]."""
        if token_ids.shape[1] != 1:
            raise ValueError("a decode step takes one token per sequence")
        return self.forward(token_ids, phase="decode", logits_to_keep=1)

    def rollback(self, length: int) -> None:
        self.state.cache.rollback(length)


# ---------------------------------------------------------------------------------------------------------------------
# model construction for tests and benchmarks (no checkpoint download)
# ---------------------------------------------------------------------------------------------------------------------
QWEN3_SHAPES = {
    # the public Qwen3 configurations the reference names (configs/mac_gate1b.json for 0.6B; 8B as the bench shape)
    "0.6b": dict(num_hidden_layers=28, hidden_size=1024, intermediate_size=3072, num_attention_heads=16,
                 num_key_value_heads=8, head_dim=128, vocab_size=151936, max_position_embeddings=40960,
                 rope_theta=1000000.0, tie_word_embeddings=True),
    "8b": dict(num_hidden_layers=36, hidden_size=4096, intermediate_size=12288, num_attention_heads=32,
               num_key_value_heads=8, head_dim=128, vocab_size=151936, max_position_embeddings=40960,
               rope_theta=1000000.0, tie_word_embeddings=False),
}


def qwen3_config(shape: str, **overrides):
    from transformers import Qwen3Config
    kw = dict(QWEN3_SHAPES[shape])
    kw.update(overrides)
    rope = kw.pop("rope_theta")
    cfg = Qwen3Config(attn_implementation="sdpa", **kw)
    if isinstance(getattr(cfg, "rope_parameters", None), dict):
        cfg.rope_parameters["rope_theta"] = rope
    else:
        cfg.rope_theta = rope
    return cfg


def _reset_rope(model, device) -> None:
    """Recompute the rotary inverse frequencies in float32 (a dtype cast of the whole model must not round them)."""
    rot = model.model.rotary_emb
    inv, scaling = rot.compute_default_rope_parameters(rot.config, device)
    rot.inv_freq = inv
    rot.original_inv_freq = inv.clone()
    rot.attention_scaling = scaling


def random_qwen3(cfg, *, device, dtype=torch.bfloat16, seed: int = 0):
    """A randomly initialised Qwen3 built directly on the device: parameters allocated without initialisation
    (meta device), then drawn N(0, initializer_range^2) from a seeded device generator, norm weights 1 (the
    transformers init rule for this architecture). Frozen, eval mode."""
    from transformers import Qwen3ForCausalLM
    with torch.device("meta"):
        model = Qwen3ForCausalLM(cfg)
    model = model.to_empty(device=device).to(dtype)
    gen = torch.Generator(device=device).manual_seed(int(seed))
    std = float(getattr(cfg, "initializer_range", 0.02))
    with torch.no_grad():
        for name, p in model.named_parameters():
            if name.endswith("norm.weight"):
                p.fill_(1.0)
            else:
                p.normal_(0.0, std, generator=gen)
    if cfg.tie_word_embeddings:
        model.tie_weights()
    _reset_rope(model, device)
    model.eval()
    for p in model.parameters():
        p.requires_grad_(False)
    return model


def tiny_qwen3(*, seed: int = 0, layers: int = 2, hidden: int = 256, heads: int = 4, groups: int = 2,
               head_dim: int = 128, intermediate: int = 512, vocab: int = 256, max_positions: int = 4096,
               dtype=torch.float32, device="cpu"):
    """A small randomly initialised Qwen3 with the real module code and this library's head_dim (128), built on the
    CPU from torch.manual_seed(seed) (so the same weights come out wherever the same torch runs), then moved."""
    from transformers import Qwen3Config, Qwen3ForCausalLM
    cfg = Qwen3Config(vocab_size=vocab, hidden_size=hidden, intermediate_size=intermediate, num_hidden_layers=layers,
                      num_attention_heads=heads, num_key_value_heads=groups, head_dim=head_dim,
                      max_position_embeddings=max_positions, tie_word_embeddings=False, attn_implementation="sdpa")
    torch.manual_seed(int(seed))
    model = Qwen3ForCausalLM(cfg).to(dtype).eval()
    _reset_rope(model, "cpu")
    model = model.to(device)
    for p in model.parameters():
        p.requires_grad_(False)
    return model
