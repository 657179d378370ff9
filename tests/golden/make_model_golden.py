"""Golden outputs of the reference's Qwen3 wrapper, made by running attention-lab's own LabRunner on CPU.

    python tests/golden/make_model_golden.py /path/to/attention-lab

A tiny randomly initialised Qwen3 with this library's head dimension (128; `attention_lab_b200.runner.tiny_qwen3`,
seeded on the CPU, float32, vocabulary 1024) is wrapped by the reference (qwen_wrap.wrap_model / make_state / LabRunner). A seeded
prompt of distinct tokens is prefilled in chunks, then a few decode steps run in the sparse mode (selector "index", rho = 1/8,
record_selection on) and in the full mode. The next-token logits of every step, every layer's row list of every
sparse step and a sha256 of the model weights go to tests/golden/model_tiny.npz. The reference is not needed at
test time; the fixture is.
"""
from __future__ import annotations

import hashlib
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

PROMPT, CHUNK, STEPS, CAPACITY, RHO, SEED, VOCAB = 300, 128, 6, 320, 1 / 8, 0, 1024


def weights_sha256(model) -> str:
    h = hashlib.sha256()
    for name, p in sorted(model.state_dict().items()):
        h.update(name.encode())
        h.update(p.detach().to(torch.float32).contiguous().numpy().tobytes())
    return h.hexdigest()


def tokens(seed: int) -> torch.Tensor:
    """PROMPT + STEPS distinct token ids: a repeated token would give layer 0 two identical pre-RoPE index keys, an
    exact score tie whose order torch.topk leaves unspecified."""
    return torch.randperm(VOCAB, generator=torch.Generator().manual_seed(seed))[:PROMPT + STEPS].view(1, -1)


def main(ref_root: str) -> None:
    sys.path.insert(0, str(Path(ref_root) / "src"))
    from attention_lab.qwen_wrap import LabRunner, make_state, wrap_model
    from attention_lab_b200.runner import tiny_qwen3

    torch.set_num_threads(8)
    model = tiny_qwen3(seed=SEED, vocab=VOCAB)
    sha = weights_sha256(model)
    seq = tokens(seed=11)
    prompt, cont = seq[:, :PROMPT], seq[:, PROMPT:]
    holder = wrap_model(model)
    out = {"weights_sha256": np.array(sha), "prompt": prompt.numpy(), "cont": cont.numpy()}
    with torch.inference_mode():
        for mode in ("sparse", "full"):
            st = make_state(model, CAPACITY, mode, seed=SEED)
            run = LabRunner(model, holder, st)
            run.prefill(prompt, CHUNK)
            if mode == "sparse":
                st.begin_request(RHO)
                st.record_selection = True
            logits, rows = [], []
            for i in range(STEPS):
                logits.append(run.step(cont[:, i:i + 1])[0, 0].numpy().copy())
                if mode == "sparse":
                    rows.append(np.stack([r.numpy().copy() for r in st.last_rows]))
            out[f"logits_{mode}"] = np.stack(logits)
            if mode == "sparse":
                out["rows_sparse"] = np.stack(rows)                     # [STEPS, layers, B*G*S]
                out["k0"] = np.array(st.k0)
    np.savez_compressed(HERE / "model_tiny.npz", **out)
    print("weights", sha[:16], {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_model_golden.py <attention-lab source root>")
    main(sys.argv[1])
