"""Host-side parts of the Qwen3 decode driver on CPU: the indexers are drawn exactly as the reference's GroupedIndexer
(indexer.py:35-45, pinned through the oracle's restatement against the golden fixtures), the selector rows follow
decode.py:96-127, and the model builders give the geometry the benches name."""
from __future__ import annotations

import numpy as np
import torch

from attention_lab_b200 import runner as rn
from oracle import oracle as orc


def test_indexer_weights_are_the_references():
    for seed in (0, 1001, 35035):
        idx = rn.Indexer(8, 4, 128, 32, device="cpu", dtype=torch.float64, seed=seed)
        wq, wk, wq_t = orc.indexer_weights(8, 4, 128, 32, seed=seed)
        assert np.array_equal(idx.wq.numpy(), wq) and np.array_equal(idx.wk.numpy(), wk)
        assert np.array_equal(idx.wq_t_scaled.numpy(), wq_t)


def test_selector_rows():
    off = torch.arange(2).view(1, 2, 1) * 500
    fixed = torch.cat([torch.arange(4).view(1, 1, 4), torch.arange(236, 300).view(1, 1, 64)], -1) + off
    off_lo = off + 4
    rows = rn.select_rows_recent(fixed, off_lo, 4, 236, 10).view(2, -1)
    assert torch.equal(rows[:, 68:] - off.view(2, 1), torch.arange(226, 236).expand(2, 10))
    rng = np.random.default_rng([5, 1, 0])
    rows_c = rn.select_rows_uniform(fixed, off_lo, 4, 236, 10, rng=rng).view(2, -1)
    want = orc.select_rows_uniform(fixed.numpy(), off_lo.numpy(), 4, 236, 10, rng=np.random.default_rng([5, 1, 0]))
    assert np.array_equal(np.sort(rows_c.numpy(), -1), np.sort(want.reshape(2, -1), -1))


def test_model_shapes():
    for shape, layers, hidden, heads, groups, tied in (("0.6b", 28, 1024, 16, 8, True), ("8b", 36, 4096, 32, 8, False)):
        cfg = rn.qwen3_config(shape)
        assert (cfg.num_hidden_layers, cfg.hidden_size, cfg.num_attention_heads, cfg.num_key_value_heads,
                cfg.head_dim, cfg.vocab_size, cfg.tie_word_embeddings) == (layers, hidden, heads, groups, 128, 151936, tied)
        assert cfg.rope_parameters["rope_theta"] == 1e6
    m = rn.tiny_qwen3()
    geo = rn.geometry_of(m)
    assert (geo.layers, geo.heads, geo.groups, geo.head_dim) == (2, 4, 2, 128)
