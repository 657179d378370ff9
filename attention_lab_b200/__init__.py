"""B200 (sm_100a) sparse-decode hot path of attention-lab behind a C ABI, with the reference's operator names.

`attention_lab_b200.ops` holds the drop-in operators; `attention_lab_b200.selection` the host-side plan rules;
`attention_lab_b200.install` rebinds the reference's Qwen3 wrapper to them; `attention_lab_b200.context_split` splits
one sequence's step over the ranks of a process group. The C ABI is declared in `include/attention_lab_b200.h` and
built by `python -m attention_lab_b200.build`.
"""
__version__ = "0.1.0"

from .ops import (append_kvz, candidate_scores, dense_decode_step, gathered_decode_step_kernel,  # noqa: E402,F401
                  project_keys, project_queries, select_rows_kernel, sparse_decode_step_kernel)
