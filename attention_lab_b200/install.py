"""Route attention-lab's Qwen3 wrapper through the B200 kernels.

`install(qwen_wrap)` takes the wrapper module object (attention_lab.qwen_wrap) and rebinds the names its decode path
calls (imported by name at qwen_wrap.py:34):

    sparse_decode_step_kernel   -> ops.sparse_decode_step_kernel    (the D read, qwen_wrap.py:300-304)
    gathered_decode_step_kernel -> ops.gathered_decode_step_kernel  (the B / C selectors, qwen_wrap.py:313)
    LabCache.append             -> a version whose K/V and index-column copies run as one CUDA launch sequence
                                   with the reference's bookkeeping and errors (qwen_wrap.py:90-106)

`LabAttention` itself is untouched. The caches and models must live on a CUDA device: the kernels have no CPU path,
so a CPU tensor reaching them raises ValueError. `uninstall(qwen_wrap)` restores the original objects.
"""
from __future__ import annotations

from . import ops

_SAVED = "_attention_lab_b200_saved"


def _append(self, layer: int, k_main, v, z=None) -> None:
    """LabCache.append with the reference's contract (one append per layer per forward, equal lengths within a
    forward, capacity check) and the copies done by al_append_kvz. As in the reference, K and V are written before a
    z for a cache without an index table raises RuntimeError (the cache then holds the new K/V rows, uncounted)."""
    start, T = self.valid_length, int(k_main.shape[2])
    if start + T > self.capacity:
        raise RuntimeError(f"cache capacity {self.capacity} exceeded: valid {start} + new {T}")
    if self._pending is None:
        self._pending = T
    elif self._pending != T:
        raise RuntimeError("layers appended different lengths within one forward")
    if z is not None and self.z is None:
        ops.append_kvz(self.k[layer], self.v[layer], None, start, k_main, v)
        raise RuntimeError("this cache was created without an index table")
    ops.append_kvz(self.k[layer], self.v[layer], None if z is None else self.z[layer], start, k_main, v,
                   None if z is None else z.to(self.z[layer].dtype))
    self.writes[layer] += 1
    self.last_write[layer] = (start, T)


def install(qwen_wrap) -> None:
    """Rebind the wrapper's hot-path operators to this library (idempotent)."""
    if getattr(qwen_wrap, _SAVED, None) is not None:
        return
    setattr(qwen_wrap, _SAVED, {
        "sparse_decode_step_kernel": qwen_wrap.sparse_decode_step_kernel,
        "gathered_decode_step_kernel": qwen_wrap.gathered_decode_step_kernel,
        "append": qwen_wrap.LabCache.append,
    })
    qwen_wrap.sparse_decode_step_kernel = ops.sparse_decode_step_kernel
    qwen_wrap.gathered_decode_step_kernel = ops.gathered_decode_step_kernel
    qwen_wrap.LabCache.append = _append


def uninstall(qwen_wrap) -> None:
    saved = getattr(qwen_wrap, _SAVED, None)
    if saved is None:
        return
    qwen_wrap.sparse_decode_step_kernel = saved["sparse_decode_step_kernel"]
    qwen_wrap.gathered_decode_step_kernel = saved["gathered_decode_step_kernel"]
    qwen_wrap.LabCache.append = saved["append"]
    setattr(qwen_wrap, _SAVED, None)
