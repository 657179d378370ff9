"""The product's host-side selection rules (attention_lab_b200.selection, used by the bench, the context split and
the model runner) against the known answers of the reference's own contract tests
(tests/test_attention_contracts.py:309-335 and tests/test_qwen_wrapper.py:387-399 of attention-lab), and the
device-free parts of the step plan. CPU only."""
from __future__ import annotations

import pytest
import torch

from attention_lab_b200 import selection as sel


def test_fixed_budget_known_answers():
    assert [sel.fixed_budget(8192, 1 / 32), sel.fixed_budget(8192, 1 / 8), sel.fixed_budget(32768, 1 / 32)] == \
        [256, 1024, 1024]
    assert [sel.fixed_budget(100, 1 / 32), sel.fixed_budget(50, 0.5), sel.fixed_budget(4, 1.0)] == [3, 0, 0]
    assert sel.fixed_budget(101, 1 / 8) == 13
    assert sel.fixed_budget(8193, 1 / 32) == 256              # config C2's k0
    assert sel.fixed_budget(131072, 1 / 32) == 4096           # config C4's k
    assert sel.fixed_budget(2048, 1 / 32) == 64               # config C1's k
    for bad in (-0.1, 1.5, float("nan")):
        with pytest.raises(ValueError):
            sel.fixed_budget(100, bad)


def test_round_is_ties_to_even():
    # rho * N0 = 2.5 and 3.5 exactly (rho = 1/64): Python's round goes to the even neighbour, as in the reference
    assert sel.fixed_budget(160, 1 / 64) == 2
    assert sel.fixed_budget(224, 1 / 64) == 4


def test_selection_layout_known_answers():
    lay = sel.selection_layout(100)
    assert (lay.fixed_count, lay.candidate_count, lay.candidate_lo, lay.candidate_hi) == (68, 32, 4, 36)
    assert lay.fixed_positions() == list(range(4)) + list(range(36, 100))
    assert (sel.selection_layout(50).fixed_count, sel.selection_layout(50).candidate_count) == (50, 0)
    assert (sel.selection_layout(3).fixed_count, sel.selection_layout(3).fixed_prefix) == (3, 3)
    with pytest.raises(ValueError):
        sel.selection_layout(0)
    assert sel.selection_layout(100).clamp_k(1000) == 32
    with pytest.raises(ValueError):
        sel.selection_layout(100).clamp_k(-1)


def test_legal_length_known_answers():
    assert (sel.legal_length(5, 10), sel.legal_length(20, 10)) == (6, 10)
    for bad in ((-1, 10), (3, 0)):
        with pytest.raises(ValueError):
            sel.legal_length(*bad)


def test_step_plan_rows():
    """k0 fixed by N0 and clamped now (prepare_request at legal length 100 with n0 = 8192: k0 256, k 32, S 100);
    rho = 0 reads exactly F; a legal length <= 68 selects nothing beyond F."""
    p = sel.build_step_plan(2, 3, 128, 100, sel.fixed_budget(8192, 1 / 32), "cpu")
    assert (p.k0, p.k, p.selected_count, p.write_col) == (256, 32, 100, 99)
    off = torch.arange(6).view(2, 3, 1) * 128
    assert torch.equal(p.fixed_rows, torch.tensor(list(range(4)) + list(range(36, 100))).view(1, 1, -1) + off)
    assert torch.equal(p.off_lo, off + 4)
    only_f = sel.build_step_plan(1, 2, 128, 128, 0, "cpu")
    assert (only_f.k, only_f.selected_count) == (0, 68)
    short = sel.build_step_plan(1, 2, 128, 60, sel.fixed_budget(60, 1 / 8), "cpu")
    assert (short.k, short.selected_count) == (0, 60)
    with pytest.raises(ValueError):
        sel.build_step_plan(1, 2, 128, 129, 4, "cpu")
