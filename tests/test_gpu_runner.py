"""The Qwen3 decode driver (attention_lab_b200.runner) on CUDA: the reference wrapper's contracts
(tests/test_qwen_wrapper.py of attention-lab) ported to this library's kernels, on a tiny randomly initialised Qwen3
with the kernels' head dimension (128), float32 and bfloat16, plus the reference's own outputs on the same model
(tests/golden/model_tiny.npz, made by tests/golden/make_model_golden.py with the reference's LabRunner).

Tolerances are the reference's preset ones for this tiny model (float32: max |diff| 1e-4, relative norm 1e-5;
bfloat16: 5e-2 / 2e-2), never loosened to pass; exact comparisons stay exact.
"""
from __future__ import annotations

import hashlib
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
TOL = {"float32": {"atol": 1e-4, "rel_norm": 1e-5}, "bfloat16": {"atol": 5e-2, "rel_norm": 2e-2}}
EXACT = {"atol": 0.0, "rel_norm": 0.0}
GOLDEN = Path(__file__).resolve().parent / "golden" / "model_tiny.npz"


def rn():
    from attention_lab_b200 import runner
    return runner


def tiny(dtype="float32"):
    return rn().tiny_qwen3(dtype=getattr(torch, dtype), device=DEV)


def ids(n, seed=1, vocab=256):
    return torch.randint(0, vocab, (1, n), generator=torch.Generator().manual_seed(seed)).to(DEV)


def close(a, b, tol, what):
    a, b = a.detach().double().cpu(), b.detach().double().cpu()
    assert torch.isfinite(a).all(), f"{what}: non-finite output"
    diff = float((a - b).abs().max())
    rel = float((a - b).norm() / (b.norm() + 1e-30))
    assert diff <= tol["atol"], f"{what}: max abs diff {diff:.3e} > {tol['atol']}"
    assert rel <= tol["rel_norm"], f"{what}: rel norm diff {rel:.3e} > {tol['rel_norm']}"


def poison_unwritten(cache):
    """NaN into every slot at or beyond valid_length (K, V and z): a correct path never reads them."""
    L = cache.valid_length
    for l in range(cache.layers):
        cache.k[l][:, :, L:] = float("nan")
        cache.v[l][:, :, L:] = float("nan")
        if cache.z is not None:
            cache.z[l][..., L:] = float("nan")


def weights_sha256(model) -> str:
    h = hashlib.sha256()
    for name, p in sorted(model.state_dict().items()):
        h.update(name.encode())
        h.update(p.detach().to(torch.float32).contiguous().cpu().numpy().tobytes())
    return h.hexdigest()


def test_matches_the_reference_wrapper_outputs():
    """The reference's LabRunner (CPU, float32) and this runner (CUDA kernels, float32) on the same model, prompt and
    continuation. Full mode: the same logits at every step. Sparse mode: every layer's row list equals the
    reference's as a set (the reference lists the chosen candidates by score, this library by position), except for
    candidates whose float64 score lies within TIE_TOL of the k-th (the two sides sum the same fp32 products in a
    different order); the logits agree at every step until the first such tie changes a row, after which the
    states differ (later layers' K/V depend on the earlier layers' reads)."""
    from parity import check_topk_float64
    g = np.load(GOLDEN)
    r = rn()
    with torch.inference_mode():
        m = r.tiny_qwen3(seed=0, vocab=1024, device="cpu")
        assert weights_sha256(m) == str(g["weights_sha256"]), "the tiny model's weights differ from the fixture's"
        m = m.to(DEV)
        holder = r.wrap_model(m)
        q_pre = {}
        hooks = [layer.self_attn.inner.q_norm.register_forward_hook(
            lambda mod, inp, out, l=l: q_pre.__setitem__(l, out.detach().clone()))
            for l, layer in enumerate(m.model.layers)]
        prompt = torch.from_numpy(g["prompt"]).to(DEV)
        cont = torch.from_numpy(g["cont"]).to(DEV)
        steps = cont.shape[1]
        for mode in ("sparse", "full"):
            st = r.make_state(m, 320, mode, seed=0)
            run = r.LabRunner(m, holder, st)
            run.prefill(prompt, 128)
            if mode == "sparse":
                assert st.begin_request(1 / 8) == int(g["k0"])
                st.record_selection = True
            diverged = False
            for i in range(steps):
                logits = run.step(cont[:, i:i + 1])[0, 0]
                if mode == "sparse" and not diverged:
                    p, G = st.plan, st.cache.groups
                    S, F = p.selected_count, p.fixed_count
                    for l in range(st.cache.layers):
                        mine = st.last_rows[l].view(G, S).cpu().numpy()
                        ref = g["rows_sparse"][i, l].reshape(G, S)
                        if all(set(mine[x].tolist()) == set(ref[x].tolist()) for x in range(G)):
                            continue
                        # a difference: both choices must be top-k sets of the float64 scores up to ties
                        qp = q_pre[l].transpose(1, 2).reshape(1, G, -1).double()            # [1,G,h*d] pre-RoPE
                        u = torch.einsum("bgf,gfj->bgj", qp, st.indexers[l].wq_t_scaled.double())
                        s64 = torch.einsum("bgj,bgjm->bgm", u, st.cache.z[l][..., p.lo:p.hi].double())[0].cpu().numpy()
                        for side, rows in (("this runner", mine), ("reference", ref)):
                            offs = np.arange(G)[:, None] * st.cache.capacity
                            chosen = np.sort(rows - offs, axis=-1)
                            chosen = np.array([[c for c in row if p.lo <= c < p.hi] for row in chosen]) - p.lo
                            check_topk_float64(chosen, s64, p.k, f"step {i} layer {l} {side}")
                        diverged = True
                        break
                if not diverged:
                    close(logits, torch.from_numpy(g[f"logits_{mode}"][i]), TOL["float32"], f"{mode} step {i} logits")
            if mode == "full":
                assert not diverged
            else:   # the fixture's prompt has no repeated token, so no exact tie: the two sides agree at every step
                assert not diverged, "a near-tie changed a row (allowed by the rule, but not expected on this fixture)"
        for h in hooks:
            h.remove()
        r.unwrap_model(m)


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_wrapped_full_path_matches_the_unmodified_model(dtype):
    r, tol = rn(), TOL[dtype]
    from transformers import DynamicCache
    for L in (32, 128, 300):
        with torch.inference_mode():
            m = tiny(dtype)
            x = ids(L)
            ref = m(x).logits
            dc = DynamicCache(config=m.config)
            m(x, past_key_values=dc, use_cache=True)
            holder = r.wrap_model(m)
            assert r.is_wrapped(m)
            st = r.make_state(m, L + 40, "full")
            run = r.LabRunner(m, holder, st)
            poison_unwritten(st.cache)
            close(run.prefill(x, L, keep_logits=True), ref, tol, "wrapped one-shot vs unmodified logits")
            for l in range(st.cache.layers):
                lay = dc.layers[l]
                close(st.cache.k[l][:, :, :L], lay.keys, tol, f"layer {l} K vs transformers cache")
                close(st.cache.v[l][:, :, :L], lay.values, tol, f"layer {l} V vs transformers cache")
            st2 = r.make_state(m, L + 40, "full")
            run2 = r.LabRunner(m, holder, st2)
            poison_unwritten(st2.cache)
            head = run2.prefill(x[:, :L - 8], 37, keep_logits=True)
            tail = torch.cat([run2.step(x[:, i:i + 1]) for i in range(L - 8, L)], dim=1)
            close(torch.cat([head, tail], 1), ref, tol, "wrapped incremental vs unmodified logits")
            assert st2.cache.valid_length == L
            assert st2.cache.writes == [-(-(L - 8) // 37) + 8] * st2.cache.layers, "one append per layer per forward"
            r.unwrap_model(m)
            assert not r.is_wrapped(m)
            close(m(x).logits, ref, EXACT, "unwrapped model is the original object graph")


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_full_selection_matches_full_path_and_poison_proves_the_subset_is_read(dtype):
    r, tol = rn(), TOL[dtype]
    with torch.inference_mode():
        m = tiny(dtype)
        L = 160
        x = ids(L, seed=2)
        ref = m(x).logits
        holder = r.wrap_model(m)
        stA = r.make_state(m, L + 16, "full")
        runA = r.LabRunner(m, holder, stA)
        runA.prefill(x[:, :L - 6], 50)
        stD = r.make_state(m, L + 16, "sparse")
        runD = r.LabRunner(m, holder, stD)
        runD.prefill(x[:, :L - 6], 50)
        stD.begin_request(None, k0=stD.cache.capacity)           # every candidate on every step
        outA, outD = [], []
        for i in range(L - 6, L):
            outA.append(runA.step(x[:, i:i + 1]))
            outD.append(runD.step(x[:, i:i + 1]))
            assert stD.plan.selected_count == stD.plan.legal_length
        outA, outD = torch.cat(outA, 1), torch.cat(outD, 1)
        close(outA, ref[:, L - 6:], tol, "wrapped full decode vs unmodified")
        close(outD, outA, tol, "sparse path with every position selected vs the full path")
        # a partial read: record the rows each layer chose, poison every other row -> D unchanged, A broken
        runD.rollback(L - 6)
        runA.rollback(L - 6)
        stD.begin_request(1 / 8)
        stD.record_selection = True
        clean = runD.step(x[:, L - 6:L - 5])
        plan = stD.plan
        assert plan.selected_count < plan.legal_length
        C = stD.cache.capacity
        for l in range(stD.cache.layers):
            keep = torch.zeros(stD.cache.batch * stD.cache.groups * C, dtype=torch.bool, device=DEV)
            keep[stD.last_rows[l]] = True
            keep = keep.view(stD.cache.batch, stD.cache.groups, C)
            for cache in (stD.cache, stA.cache):
                cache.k[l][~keep] = float("nan")
                cache.v[l][~keep] = float("nan")
        runD.rollback(L - 6)
        poisoned = runD.step(x[:, L - 6:L - 5])
        assert torch.isfinite(poisoned).all(), "the sparse path read a row it did not select"
        close(poisoned, clean, EXACT, "sparse step with its unselected rows poisoned")
        assert not torch.isfinite(runA.step(x[:, L - 6:L - 5])).all(), "the full path must see the poison"
        r.unwrap_model(m)


def test_unwritten_slots_and_future_positions_never_change_a_step():
    r = rn()
    with torch.inference_mode():
        m = tiny()
        L = 120
        x = ids(L, seed=3)
        holder = r.wrap_model(m)
        for mode in ("full", "sparse"):
            st = r.make_state(m, L + 64, mode)
            run = r.LabRunner(m, holder, st)
            run.prefill(x[:, :L - 5], 40)
            if mode == "sparse":
                st.begin_request(1 / 8)
            clean = torch.cat([run.step(x[:, i:i + 1]) for i in range(L - 5, L)], 1)
            run.rollback(L - 5)
            for l in range(st.cache.layers):                     # garbage and a huge finite value in future slots
                st.cache.k[l][:, :, L - 5:L - 2] = float("nan")
                st.cache.k[l][:, :, L - 2:] = 1e6
                st.cache.v[l][:, :, L - 5:] = float("nan")
                if st.cache.z is not None:
                    st.cache.z[l][..., L - 5:] = float("nan")
            again = torch.cat([run.step(x[:, i:i + 1]) for i in range(L - 5, L)], 1)
            assert torch.isfinite(again).all(), f"{mode}: an unwritten or future slot leaked"
            close(again, clean, EXACT, f"{mode}: poisoned future slots")
        r.unwrap_model(m)


def test_rollback_branches_and_the_old_suffix_is_unreadable():
    r = rn()
    with torch.inference_mode():
        m = tiny()
        x, alt = ids(140, seed=4), ids(140, seed=5)
        holder = r.wrap_model(m)
        for mode in ("full", "sparse"):
            st = r.make_state(m, 160, mode)
            run = r.LabRunner(m, holder, st)
            run.prefill(x[:, :100], 37)
            if mode == "sparse":
                st.begin_request(1 / 8)
            first = torch.cat([run.step(x[:, i:i + 1]) for i in range(100, 105)], 1)
            assert st.cache.valid_length == 105
            run.rollback(100)
            poison_unwritten(st.cache)                           # the rolled-back suffix must be invisible
            second = torch.cat([run.step(x[:, i:i + 1]) for i in range(100, 105)], 1)
            close(second, first, EXACT, f"{mode}: same tokens after rollback")
            run.rollback(100)
            branch = torch.cat([run.step(alt[:, i:i + 1]) for i in range(100, 105)], 1)
            fresh = r.make_state(m, 160, mode)
            runf = r.LabRunner(m, holder, fresh)
            runf.prefill(x[:, :100], 100)
            if mode == "sparse":
                fresh.begin_request(1 / 8)
            fresh_out = torch.cat([runf.step(alt[:, i:i + 1]) for i in range(100, 105)], 1)
            close(branch, fresh_out, TOL["float32"], f"{mode}: overwritten suffix vs fresh cache")
            with pytest.raises(ValueError):
                run.rollback(200)
        # cloned caches (request branches) share no storage and do not alias
        st = r.make_state(m, 128, "sparse")
        run = r.LabRunner(m, holder, st)
        run.prefill(x[:, :100], 100)
        st.begin_request(1 / 8)
        st2 = r.LabState(st.cache.clone(), st.indexers, mode="sparse")
        st2.begin_request(1 / 8)
        run2 = r.LabRunner(m, holder, st2)
        ptrs = {t.data_ptr() for t in st.cache.k + st.cache.v + st.cache.z}
        assert ptrs.isdisjoint({t.data_ptr() for t in st2.cache.k + st2.cache.v + st2.cache.z})
        out1 = run.step(x[:, 100:101])
        out2 = run2.step(alt[:, 100:101])
        assert not torch.equal(st.cache.k[0][:, :, 100], st2.cache.k[0][:, :, 100])
        assert torch.equal(st.cache.k[0][:, :, :100], st2.cache.k[0][:, :, :100])
        run.rollback(100)
        close(run.step(x[:, 100:101]), out1, EXACT, "branch 1 unaffected by branch 2")
        run2.rollback(100)
        close(run2.step(alt[:, 100:101]), out2, EXACT, "branch 2 unaffected by branch 1")
        r.unwrap_model(m)


def test_chunked_prefill_matches_one_shot_for_kv_and_index_table():
    r, tol = rn(), TOL["float32"]
    with torch.inference_mode():
        m = tiny()
        L = 100
        x = ids(L, seed=6)
        holder = r.wrap_model(m)
        one = r.make_state(m, L + 8, "sparse")
        r.LabRunner(m, holder, one).prefill(x, L)
        for bounds in ((0, 5, 50, 100), (0, 1, 2, 100)):
            chunked = r.make_state(m, L + 8, "sparse")
            runc = r.LabRunner(m, holder, chunked)
            for a, b in zip(bounds, bounds[1:]):
                runc.forward(x[:, a:b], phase="prefill", logits_to_keep=1)
            assert chunked.cache.valid_length == L and chunked.plan is None
            for l in range(one.cache.layers):
                close(chunked.cache.k[l][:, :, :L], one.cache.k[l][:, :, :L], tol, f"layer {l} K chunked vs one-shot")
                close(chunked.cache.v[l][:, :, :L], one.cache.v[l][:, :, :L], tol, f"layer {l} V chunked vs one-shot")
                close(chunked.cache.z[l][..., :L], one.cache.z[l][..., :L], tol, f"layer {l} z chunked vs one-shot")
        r.unwrap_model(m)


def test_index_features_are_pre_rope_and_each_z_column_is_written_once():
    r, tol = rn(), TOL["float32"]
    with torch.inference_mode():
        m = tiny()
        L = 90
        x = ids(L + 3, seed=7)
        holder = r.wrap_model(m)
        st = r.make_state(m, L + 16, "sparse")
        run = r.LabRunner(m, holder, st)
        captured = {}
        hooks = [layer.self_attn.inner.k_norm.register_forward_hook(
            lambda mod, inp, out, l=l: captured.__setitem__(l, out.detach().clone()))
            for l, layer in enumerate(m.model.layers)]
        run.prefill(x[:, :L], L)
        wkz = lambda k_pre, wk: torch.matmul(wk.unsqueeze(0), k_pre.transpose(-1, -2))   # indexer.py:15-17
        for l in range(st.cache.layers):
            k_pre = captured[l].transpose(1, 2)                  # [B,G,T,d] after k_norm, before RoPE
            close(st.cache.z[l][..., :L], wkz(k_pre, st.indexers[l].wk), tol, f"layer {l} z = Wk . k_pre")
            rotated = wkz(st.cache.k[l][:, :, :L].float(), st.indexers[l].wk)
            rel = float((st.cache.z[l][..., :L] - rotated).norm() / rotated.norm())
            assert rel > 0.1, "z must not come from the rotated keys in the cache"
        st.begin_request(1 / 8)
        snapshot = [st.cache.z[l][..., :L].clone() for l in range(st.cache.layers)]
        for i in range(L, L + 3):
            run.step(x[:, i:i + 1])
            for l in range(st.cache.layers):
                close(st.cache.z[l][..., i:i + 1], wkz(captured[l].transpose(1, 2), st.indexers[l].wk), tol,
                      f"step {i} layer {l} new z column")
                assert torch.equal(st.cache.z[l][..., :L], snapshot[l]), "older z columns were rewritten"
                assert st.cache.last_write[l] == (i, 1)
        assert st.cache.writes == [1 + 3] * st.cache.layers
        for h in hooks:
            h.remove()
        r.unwrap_model(m)


def test_a_sparse_step_selects_on_the_device_one_row_list_per_layer(monkeypatch):
    """The reference's sparse step calls torch.topk once per layer; here the top-k runs inside the fused kernel, so a
    sparse step calls neither torch.topk nor torch.gather, and every layer leaves exactly one row list."""
    r = rn()
    with torch.inference_mode():
        m = tiny()
        x = ids(130, seed=8)
        holder = r.wrap_model(m)
        st = r.make_state(m, 160, "sparse")
        run = r.LabRunner(m, holder, st)
        run.prefill(x[:, :129], 129)
        st.begin_request(1 / 8)
        st.record_selection = True

        def forbidden(*a, **k):
            raise AssertionError("a torch top-k or gather ran in a sparse step")
        monkeypatch.setattr(torch, "topk", forbidden)
        monkeypatch.setattr(torch, "gather", forbidden)
        run.step(x[:, 129:130])
        monkeypatch.undo()
        S = st.plan.selected_count
        assert all(rows is not None and rows.numel() == st.cache.groups * S for rows in st.last_rows)
        r.unwrap_model(m)


def test_k_rule_fixed_per_request_and_short_history_degenerates_to_full():
    r = rn()
    with torch.inference_mode():
        m = tiny()
        x = ids(130, seed=11)
        ref = m(x).logits
        holder = r.wrap_model(m)
        st = r.make_state(m, 160, "sparse")
        run = r.LabRunner(m, holder, st)
        run.prefill(x[:, :100], 100)
        k0 = st.begin_request(1 / 8)
        assert (st.request_start_length, k0) == (101, 13)
        for i in range(100, 110):
            run.step(x[:, i:i + 1])
            p = st.plan
            assert (p.k, p.k0, p.legal_length, p.selected_count, p.candidate_count, p.write_col) == \
                (13, 13, i + 1, 68 + 13, i + 1 - 68, i)
        short = r.make_state(m, 160, "sparse")
        runs = r.LabRunner(m, holder, short)
        runs.prefill(x[:, :20], 20)
        assert short.begin_request(1 / 8) == 0
        out = torch.cat([runs.step(x[:, i:i + 1]) for i in range(20, 30)], 1)
        assert (short.plan.k, short.plan.selected_count) == (0, 30)
        close(out, ref[:, 20:30], TOL["float32"], "legal length <= 68 reads everything")
        with pytest.raises(RuntimeError):
            fresh = r.make_state(m, 160, "sparse")
            r.LabRunner(m, holder, fresh).step(x[:, :1])        # sparse decode without begin_request
        r.unwrap_model(m)


def test_phase_is_explicit_and_a_one_token_prefill_chunk_never_selects():
    r, tol = rn(), TOL["float32"]
    with torch.inference_mode():
        m = tiny()
        x = ids(140, seed=21)
        ref = m(x).logits
        holder = r.wrap_model(m)
        st = r.make_state(m, 64, "sparse")
        run = r.LabRunner(m, holder, st)
        close(run.prefill(x[:, :1], 2048, keep_logits=True), ref[:, :1], tol, "one-token prompt")
        assert st.plan is None and st.cache.valid_length == 1
        st2 = r.make_state(m, 160, "sparse")
        run2 = r.LabRunner(m, holder, st2)
        st2.begin_request(1 / 8)
        close(run2.prefill(x[:, :101], 50, keep_logits=True), ref[:, :101], tol, "prefill ending in a one-token chunk")
        assert st2.plan is None, "a one-token prefill chunk built a selection plan"
        with pytest.raises(TypeError):
            run2.forward(x[:, 101:102])
        with pytest.raises(ValueError):
            run2.forward(x[:, 101:103], phase="decode")
        with pytest.raises(ValueError):
            run2.forward(x[:, 101:102], phase="generate")
        r.unwrap_model(m)


@pytest.mark.parametrize("selector", ["recent", "uniform"])
def test_selectors_b_and_c_read_exactly_their_rows(selector):
    """B and C (decode.py:96-127): the same F and budget as D0, their own row lists, attended by the gathered kernel;
    the output equals the full path's read restricted to those rows (a dense masked read with the model's own SDPA)."""
    r = rn()
    with torch.inference_mode():
        m = tiny()
        x = ids(200, seed=13)
        holder = r.wrap_model(m)
        st = r.make_state(m, 220, "sparse", selector=selector, uniform_seed=5)
        run = r.LabRunner(m, holder, st)
        run.prefill(x[:, :180], 64)
        st.begin_request(1 / 8)
        st.record_selection = True
        run.step(x[:, 180:181])
        plan = st.plan
        rows = st.last_rows[0].view(st.cache.groups, plan.selected_count)
        pos = (rows - torch.arange(st.cache.groups, device=DEV).view(-1, 1) * st.cache.capacity).cpu()
        F = plan.fixed_count
        assert torch.equal(pos[:, :F], torch.tensor(list(range(4)) + list(range(plan.hi, plan.legal_length))).expand(
            st.cache.groups, F))
        cand = pos[:, F:]
        assert ((cand >= plan.lo) & (cand < plan.hi)).all() and cand.shape[1] == plan.k
        assert all(len(set(c.tolist())) == plan.k for c in cand)
        if selector == "recent":
            assert torch.equal(cand.sort(dim=-1).values, torch.arange(plan.hi - plan.k, plan.hi).expand_as(cand))
        r.unwrap_model(m)
