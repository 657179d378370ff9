"""Generate the golden fixtures by running the reference (attention-lab) itself on CPU.

Run in a container where the reference source tree is available:

    python tests/golden/make_golden.py /path/to/attention-lab

For every case of `cases.CASES` it builds the seeded inputs, checks that this repository's restated indexer init
draws bit-identical weights to the reference's `GroupedIndexer`, then runs the reference's own
`sparse_decode_step_kernel` (decode.py:145-163, `return_rows=True`), `candidate_scores` (indexer.py:27-29),
`dense_decode_step` (decode.py:174-176) and the float64 brute force `GroupedIndexer.reference_scores`
(indexer.py:57-64), and stores the outputs with a sha256 of the inputs in `tests/golden/<case>.npz`.
The reference is never needed at test time; the fixtures are.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import cases as cs  # noqa: E402


def main(ref_root: str) -> None:
    sys.path.insert(0, str(Path(ref_root) / "src"))
    from attention_lab.decode import dense_decode_step, gathered_decode_step_kernel, sparse_decode_step_kernel
    from attention_lab.indexer import GroupedIndexer, candidate_scores, project_keys, project_queries
    from attention_lab.selection import fixed_budget, selection_layout

    torch.set_num_threads(8)
    for name, case in cs.CASES.items():
        t = cs.build(case)
        const = cs.step_constants(case)
        # pin: the restated plan and indexer init equal the reference's
        lay = selection_layout(case.L)
        k_ref = lay.clamp_k(fixed_budget(case.L, case.rho) if case.k0 is None else case.k0)
        assert (lay.candidate_lo, lay.candidate_hi, k_ref) == (const["lo"], const["hi"], const["k"]), name
        idx = GroupedIndexer(case.G, case.h, case.d, case.r, dtype=torch.float64, seed=case.seed)
        assert torch.equal(idx.wk, t["wk64"]) and torch.equal(idx.wq_t_scaled, t["wq_t64"]), name
        lo, hi, k, S, wc = const["lo"], const["hi"], const["k"], const["S"], const["write_col"]
        fixed_rows = torch.from_numpy(const["fixed_rows"])
        off_lo = torch.from_numpy(const["off_lo"])
        zT = t["zT"].clone()
        scale = 1.0 / case.d ** 0.5
        with torch.inference_mode():
            out, rows = sparse_decode_step_kernel(t["q"], t["q_pre"], t["k"], t["v"], zT, t["wq_t"], t["wk"],
                                                  fixed_rows, off_lo, lo, hi, k, S, k_pre_new=t["k_pre_new"],
                                                  write_col=wc, scale=scale, return_rows=True,
                                                  canonical_order=case.canonical)
            u = project_queries(t["q_pre"], t["wq_t"])
            scores = candidate_scores(u, zT, lo, hi)[:, :, 0, :]
            zcol = zT[..., wc].clone()
            z_direct = project_keys(t["k_pre_new"], t["wk"])[..., 0]
            assert torch.equal(zcol, z_direct), name
            # attention over the same rows with K/V/q upcast to float32: accuracy reference for the kernels
            f = lambda x: x.to(torch.float32)  # noqa: E731
            out32 = gathered_decode_step_kernel(f(t["q"]), f(t["k"]), f(t["v"]), rows, S, scale=scale)
            dense = dense_decode_step(t["q"], t["k"], t["v"], case.L, scale=scale)
            ref64 = idx.reference_scores(t["q_pre"].double(), torch.cat(
                [t["k_pre"][:, :, :wc].double(), t["k_pre_new"].double()], dim=2), lo, hi)[:, :, 0, :]
        np.savez_compressed(
            HERE / f"{name}.npz",
            inputs_sha256=np.array(cs.sha256_of(t)),
            lo=lo, hi=hi, k=k, S=S, write_col=wc,
            rows=rows.numpy().astype(np.int64),
            scores=scores.to(torch.float32).numpy(),
            scores_ref64=ref64.numpy() if case.B * case.G * (hi - lo) <= 20000 else np.zeros(0),
            zcol=zcol.to(torch.float32).numpy(),
            out=out.to(torch.float32).numpy(),
            out_f32=out32.to(torch.float32).numpy(),
            dense=dense.to(torch.float32).numpy(),
        )
        print(f"{name}: lo={lo} hi={hi} k={k} S={S} rows={rows.numel()} out={tuple(out.shape)}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_golden.py <attention-lab source root>")
    main(sys.argv[1])
