"""install() rebinds exactly the wrapper names the reference's decode path calls, keeps LabCache's bookkeeping and
errors, and uninstall() restores the originals. CPU only: a stand-in module with the reference's attribute names."""
from __future__ import annotations

import types

import pytest
import torch

from attention_lab_b200 import install as inst
from attention_lab_b200 import ops


class FakeCache:
    def __init__(self, capacity=8):
        self.capacity, self.valid_length, self._pending = capacity, 0, None
        self.k = [torch.zeros(1, 2, capacity, 128)]
        self.v = [torch.zeros(1, 2, capacity, 128)]
        self.z = None
        self.writes, self.last_write = [0], [None]

    def append(self, layer, k_main, v, z=None):  # the original
        return "original"


def fake_wrapper():
    m = types.SimpleNamespace()
    m.sparse_decode_step_kernel = lambda *a, **k: "ref-sparse"
    m.gathered_decode_step_kernel = lambda *a, **k: "ref-gathered"
    m.LabCache = FakeCache
    return m


def test_install_rebinds_and_uninstall_restores():
    m = fake_wrapper()
    orig = (m.sparse_decode_step_kernel, m.gathered_decode_step_kernel, m.LabCache.append)
    inst.install(m)
    inst.install(m)                                  # idempotent
    assert m.sparse_decode_step_kernel is ops.sparse_decode_step_kernel
    assert m.gathered_decode_step_kernel is ops.gathered_decode_step_kernel
    assert m.LabCache.append is inst._append
    inst.uninstall(m)
    assert (m.sparse_decode_step_kernel, m.gathered_decode_step_kernel, m.LabCache.append) == orig


def test_append_keeps_the_reference_contract():
    m = fake_wrapper()
    inst.install(m)
    try:
        c = m.LabCache(capacity=4)
        with pytest.raises(RuntimeError, match="capacity"):
            c.append(0, torch.zeros(1, 2, 5, 128), torch.zeros(1, 2, 5, 128))
        c._pending = 2
        with pytest.raises(RuntimeError, match="different lengths"):
            c.append(0, torch.zeros(1, 2, 1, 128), torch.zeros(1, 2, 1, 128))
        c._pending = None
        with pytest.raises(ValueError, match="CUDA"):          # no CPU path behind the kernels
            c.append(0, torch.zeros(1, 2, 1, 128), torch.zeros(1, 2, 1, 128))
    finally:
        inst.uninstall(m)


def test_append_without_index_table_writes_kv_first(monkeypatch):
    """The reference (qwen_wrap.py:100-104) copies K and V, then raises for a z without an index table; the
    installed append issues the K/V copy first too, and counts no write."""
    calls = []
    monkeypatch.setattr(inst.ops, "append_kvz", lambda *a, **k: calls.append(a))
    m = fake_wrapper()
    inst.install(m)
    try:
        c = m.LabCache(capacity=4)
        with pytest.raises(RuntimeError, match="index table"):
            c.append(0, torch.zeros(1, 2, 1, 128), torch.zeros(1, 2, 1, 128), torch.zeros(1, 2, 32, 1))
        assert len(calls) == 1 and calls[0][2] is None and calls[0][3] == 0     # K/V only, at position 0
        assert c.writes == [0] and c.last_write == [None]
    finally:
        inst.uninstall(m)
