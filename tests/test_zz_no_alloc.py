"""The one entry point that allocates nothing: al_context_threshold_noalloc, called through the C ABI.

It is for callers that cannot call cudaMalloc where they run, such as a serving runtime that has handed all device
memory to its own pool, or code inside a CUDA-graph capture. It gathers every rank's keys into a scratch array that is
part of the library image and runs the context-split threshold over it, so its rows must equal those of the
allocating entry point (al_context_threshold over the stacked keys) exactly. Two calls in a row with different keys
check that the shared scratch carries nothing from one call into the next. This file is collected last so that a run
that stops at its first failure has already run every other test.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _keys(world, B, G, kst, k_local, seed):
    """Distinct positive 64-bit keys per rank (zero past k_local, like al_context_local_topk's padding)."""
    g = torch.Generator().manual_seed(seed)
    n = world * B * G * kst
    keys = torch.randperm(1 << 24, generator=g)[:n].to(torch.int64) * 7919 + 1
    keys = keys.view(world, B, G, kst).clone()
    keys[..., k_local:] = 0
    return keys.to(DEV)


def _noalloc(lib, keys, rank, k, F, k_local, rows):
    world, B, G, kst = keys.shape
    ptrs = torch.tensor([keys[q].data_ptr() for q in range(world)], dtype=torch.int64, device=DEV)
    out = torch.empty_like(rows)
    rc = lib.al_context_threshold_noalloc(ptrs.data_ptr(), world, rank, B, G, kst, k, F, k_local, rows.data_ptr(),
                                          out.data_ptr(), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    return rc, out


def test_no_alloc_threshold_equals_the_allocating_one_on_two_calls_in_a_row():
    from attention_lab_b200 import _lib, ops
    lib = _lib.load()
    world, B, G, kst, k_local, F = 3, 2, 4, 320, 300, 5
    k = 500
    for call, seed in enumerate((1, 2)):
        keys = _keys(world, B, G, kst, k_local, seed)
        for rank in range(world):
            rows = torch.randint(0, 1 << 30, (B, G, F + k_local), dtype=torch.int64,
                                 generator=torch.Generator().manual_seed(seed * 10 + rank)).to(DEV)
            want = ops.context_threshold(keys.contiguous(), rows, rank, k, F, k_local)
            rc, got = _noalloc(lib, keys, rank, k, F, k_local, rows)
            assert rc == _lib.AL_OK, lib.al_last_error().decode()
            torch.cuda.synchronize()
            assert torch.equal(got, want), f"call {call} rank {rank}"
            kept = int((got[..., F:] >= 0).sum())
            assert 0 < kept <= B * G * k_local
    assert _lib.device_status() == 0


def test_no_alloc_threshold_rejects_sizes_beyond_its_scratch():
    from attention_lab_b200 import _lib
    lib = _lib.load()
    world, B, G, kst = 8, 1, 64, 1025                       # 525 056 keys > 524 288
    keys = torch.zeros(world, B, G, kst, dtype=torch.int64, device=DEV)
    rows = torch.zeros(B, G, 4, dtype=torch.int64, device=DEV)
    rc, _ = _noalloc(lib, keys, 0, 16, 0, 4, rows)
    assert rc == _lib.AL_EUNSUPPORTED
    assert "no-allocation scratch" in lib.al_last_error().decode()
