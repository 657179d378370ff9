"""The C-ABI library loads without a GPU and exports every entry point include/attention_lab_b200.h declares;
the Python operators refuse non-CUDA tensors instead of falling back to a CPU path. CPU only."""
from __future__ import annotations

import re
from pathlib import Path

import pytest
import torch

from attention_lab_b200 import _lib, ops

HEADER = Path(__file__).resolve().parents[1] / "include" / "attention_lab_b200.h"


def declared_names():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+char\s*\*|int)\s+(al_\w+)\s*\(", text, flags=re.M)))


REQUIRED = {"al_sparse_decode_step", "al_select_rows", "al_gathered_attend", "al_dense_decode", "al_append_kvz",
            "al_project_keys", "al_project_queries", "al_candidate_scores", "al_context_local_topk",
            "al_context_threshold", "al_gathered_attend_partial", "al_lse_merge", "al_xchg_create", "al_xchg_open",
            "al_xchg_close", "al_xchg_destroy", "al_xchg_push", "al_context_threshold_peer", "al_lse_merge_peer",
            "al_context_threshold_noalloc", "al_prefill_score_topk", "al_last_error", "al_version", "al_device_status"}


def test_header_declares_the_bound_entry_points():
    names = declared_names()
    assert REQUIRED <= set(names), f"missing from the header: {sorted(REQUIRED - set(names))}"
    assert names == sorted(_lib.SIGNATURES), "ctypes signatures and the header disagree"


def test_library_loads_and_exports_every_symbol():
    lib = _lib.load()
    for name in declared_names():
        assert hasattr(lib, name), f"{name} is not exported"
    assert lib.al_version() == 1
    assert lib.al_last_error() == b""


def test_operators_refuse_cpu_tensors():
    q = torch.zeros(1, 2, 2, 1, 128)
    k = torch.zeros(1, 2, 64, 128)
    with pytest.raises(ValueError, match="CUDA"):
        ops.gathered_decode_step_kernel(q, k, k, torch.zeros(2 * 4, dtype=torch.long), 4)
    with pytest.raises(ValueError, match="CUDA"):
        ops.dense_decode_step(q, k, k, 64)
    with pytest.raises(ValueError, match="backend"):
        ops.dense_decode_step(q, k, k, 64, backend="nope")


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", tmp_path / "absent.so")
    with pytest.raises(RuntimeError, match="not built"):
        _lib.load()
