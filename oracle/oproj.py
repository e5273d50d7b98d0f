"""CPU restatement of the Wan self-attention output projection and the norm2 gated residual.

* ``wan_o_proj_ref`` follows ``_wan_o_proj``'s torch path
  (vllm_omni_neuron/diffusion/models/wan2_2/wan2_2_transformer.py:246-254):
  ``x = active.reshape(B, N*D, S).transpose(1, 2); y = x @ W + b`` on bf16 tensors — the matmul
  accumulates in fp32 and is rounded to bf16, then the bias add is rounded again.
* ``gated_residual_ref`` is the residual step of the block's norm2
  (``adaln_modulate(attn1_out, ..., residual=hidden_states, gate=gate_msa)``, :1470-1489):
  ``bf16(residual + gate * y)`` with the product and the sum in fp32 (``_eager_adaln``,
  diffusion/quantization/adaln_kernels.py:51-84).
* ``row_mx_o_proj_ref`` restates the FP8 o-projection ``row_mx_o_proj``
  (vllm_omni_neuron/diffusion/quantization/row_mx_kernels.py:114-138): per-token ROW quantisation of
  the d-major activation (``adaln.row_quantize`` with the NKI reciprocal multiply,
  adaln_quant.py:520-536), then the ROW_MX dequant-matmul of ``qkv.row_mx_qkv_ref``.

Pinned by ``tests/golden/wan_o_proj.npz`` (outputs of ``_wan_o_proj`` itself) and, for the residual
step, by ``tests/golden/eager_adaln.npz``. ``row_mx_o_proj_ref`` is parity unpinned as a whole: the
reference's kernel (nkilib ``output_projection_cte``) and any torch reference of it are not in the
reference tree; its two steps are pinned separately (the ROW quantiser by ``adaln_ref.npz``, the
dequant-matmul by ``qkv_row_mx.npz``).
"""

from __future__ import annotations

import numpy as np

from .adaln import row_quantize
from .numerics import bf16_round, e4m3fn_bits
from .qkv import row_mx_qkv_ref


def wan_o_proj_ref(active: np.ndarray, weight: np.ndarray, bias=None) -> np.ndarray:
    """active [B, N, D, S] (bf16 values), weight [N*D, H], bias [H] or [1, H] -> [B, S, H]."""
    B, N, D, S = active.shape
    x = np.asarray(active, np.float32).reshape(B, N * D, S).transpose(0, 2, 1)
    y = bf16_round(x @ np.asarray(weight, np.float32))
    if bias is not None:
        y = bf16_round(y + np.asarray(bias, np.float32).reshape(1, 1, -1))
    return y


def gated_residual_ref(y: np.ndarray, residual: np.ndarray, gate=None) -> np.ndarray:
    """bf16(residual + gate * y); gate [B, 1, H], [H] or None (1)."""
    g = np.asarray(y, np.float32)
    if gate is not None:
        g = (g * np.asarray(gate, np.float32)).astype(np.float32)
    return bf16_round(np.asarray(residual, np.float32) + g)


def row_mx_o_proj_ref(active: np.ndarray, w_codes: np.ndarray, w_scale: np.ndarray, bias=None) -> np.ndarray:
    """active [B, N, D, S] (bf16 values); w_codes [H, N*D] e4m3-valued; w_scale [H] fp32; bias [H].
    Returns the bf16-valued [B, S, H] output and the (codes [B*S, N*D], scales [B*S]) of the
    activation quantisation."""
    B, N, D, S = active.shape
    x = np.asarray(active, np.float32).reshape(B, N * D, S).transpose(0, 2, 1).reshape(B * S, N * D)
    codes, scale = row_quantize(x, reciprocal=True)
    packed = np.concatenate([e4m3fn_bits(codes), scale.astype(np.float32).reshape(-1, 1).view(np.uint8)], axis=1)
    y = row_mx_qkv_ref(packed, np.asarray(w_codes, np.float32).T, w_scale, bias)
    return y.reshape(B, S, -1), (codes, scale.reshape(-1))


def o_proj_flops(b: int, s: int, k: int, h: int) -> float:
    return 2.0 * b * s * k * h
