"""CPU restatement of the CFG-parallel combine (test infrastructure only: the checker for the GPU path).

``cfg_combine_ref`` follows ``_cfg_gather_combine``
(vllm_omni_neuron/diffusion/distributed/cfg_parallel.py:48-71): after the CFG group's all_gather,
index 0 is the positive branch and index 1 the negative one, and the result is
``negative + true_cfg_scale * (positive - negative)`` evaluated by torch on tensors of the branch
dtype. torch computes each of the three operations in fp32 and rounds the result to the tensor's
dtype, with the Python scalar converted to fp32; this restatement does the same in numpy.

Pinned by ``tests/test_oracle_golden.py::test_cfg_combine_matches_torch_eager``, which evaluates the
reference's own expression with torch on the CPU for bf16 and fp32 inputs.
"""

from __future__ import annotations

import numpy as np

from .numerics import bf16_round


def cfg_combine_ref(positive: np.ndarray, negative: np.ndarray, true_cfg_scale: float, bf16: bool) -> np.ndarray:
    """``negative + true_cfg_scale * (positive - negative)`` (CFGP:71); inputs are float32 arrays holding
    the branch values (bf16 values when ``bf16``); returns float32 (bf16 values when ``bf16``)."""
    p = np.asarray(positive, np.float32)
    n = np.asarray(negative, np.float32)
    s = np.float32(true_cfg_scale)
    rnd = bf16_round if bf16 else (lambda x: np.asarray(x, np.float32))
    d = rnd(p - n)
    m = rnd(s * d)
    return rnd(n + m)


def cfg_gather_combine_ref(branch_preds, true_cfg_scale: float, bf16: bool) -> np.ndarray:
    """The all_gather + combine over a CFG group of two ranks: ``branch_preds[0]`` positive (cfg rank 0),
    ``branch_preds[1]`` negative (cfg rank 1) (CFGP:68-71, 147-151)."""
    if len(branch_preds) != 2:
        raise ValueError("the CFG group has two ranks")
    return cfg_combine_ref(branch_preds[0], branch_preds[1], true_cfg_scale, bf16)
