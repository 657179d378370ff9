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


def test_header_declares_the_bound_entry_points():
    names = declared_names()
    assert len(names) >= 10
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
