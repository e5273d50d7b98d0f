"""CPU restatement of the Wan FFN, ``_wan_mlp``'s torch path
(vllm_omni_neuron/diffusion/models/wan2_2/wan2_2_transformer.py:389-410):

    up  = bf16(bf16(x @ Wu) + bu)          (bf16 tensors: matmul then bias add, each rounded)
    g   = bf16(gelu_tanh(up))              (fp32 opmath: 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))))
    out = bf16(bf16(g @ Wd) + bd)

Pinned by ``tests/golden/wan_mlp.npz`` (outputs of ``_wan_mlp`` itself).
"""

from __future__ import annotations

import numpy as np

from .numerics import bf16_round


def gelu_tanh(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, np.float32)
    beta = np.float32(0.7978845608028654)
    kappa = np.float32(0.044715)
    inner = beta * (x + kappa * (x * x * x))
    return (np.float32(0.5) * x * (np.float32(1) + np.tanh(inner))).astype(np.float32)


def _linear(x, w, b):
    y = bf16_round(np.asarray(x, np.float32) @ np.asarray(w, np.float32))
    if b is not None:
        y = bf16_round(y + np.asarray(b, np.float32).reshape(1, -1))
    return y


def wan_mlp_ref(hidden, up_w, down_w, up_b, down_b) -> np.ndarray:
    lead = hidden.shape[:-1]
    x = np.asarray(hidden, np.float32).reshape(-1, hidden.shape[-1])
    up = _linear(x, up_w, up_b)
    g = bf16_round(gelu_tanh(up))
    out = _linear(g, down_w, down_b)
    return out.reshape(lead + (out.shape[-1],))


def ffn_flops(tokens: int, h: int, inner: int) -> float:
    return 4.0 * tokens * h * inner
