"""hearth_b200 — B200-native (sm_100a) backend for Hearth's quantized MoE expert path.

* ``native``  — the reference's ``hearth._native`` kernel entry points (``matmul``, ``dequantize``,
  ``row_bytes``) on the GPU, same names, argument meaning and errors.
* ``MoeBackend`` — the MoE half of the engine (router, Q4/Q8 experts, rank-order sum) behind one
  handle with an HBM-resident expert store.
* ``Model`` — the whole decoder of a container (embedding, GQA attention with its KV cache, MoE and
  dense FFN layers, LM head) on the GPU, evaluated like hearth_eval.

Everything runs through the C ABI of include/hearth_b200.h in ``libhearth_b200.so``; there is no
CPU fallback.
"""
from ._lib import (BF16, F16, F32, POLICY_LFU, POLICY_LRU, Q4, Q8, SCORE_SIGMOID, SCORE_SOFTMAX,  # noqa: F401
                   lib, last_error)
from . import native  # noqa: F401
from .moe import MoeBackend, container_probe  # noqa: F401
from .model import Model  # noqa: F401

__all__ = ["lib", "last_error", "native", "MoeBackend", "Model", "container_probe", "F32", "F16", "BF16", "Q8", "Q4"]
