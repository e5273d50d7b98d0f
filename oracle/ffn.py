"""CPU restatement of the Wan FFN, ``_wan_mlp``'s torch path
(vllm_omni_neuron/diffusion/models/wan2_2/wan2_2_transformer.py:389-410):

    up  = bf16(bf16(x @ Wu) + bu)          (bf16 tensors: matmul then bias add, each rounded)
    g   = bf16(gelu_tanh(up))              (fp32 opmath: 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))))
    out = bf16(bf16(g @ Wd) + bd)

Pinned by ``tests/golden/wan_mlp.npz`` (outputs of ``_wan_mlp`` itself).

``wan_mlp_row_mx_ref`` restates the FP8 leaf ``row_mx_mlp``
(vllm_omni_neuron/diffusion/quantization/row_mx_kernels.py:141-198), the nkilib MLP kernel in ROW_MX
CTE mode, following its PyTorch reference ``_mlp_ref_standard``
(vllm_omni_neuron/kernels/nkilib/core/mlp/mlp_torch.py:401-600) with ``skip_gate_proj=True`` and
``GELU_Tanh_Approx``:

    up    = (Xq * row_scale) @ (Wu_q * wu_scale) + bu       (fp32; :470-486 pre-quantised ROW input,
                                                             :491-497 per-channel weight scales)
    inter = gelu_tanh(up)                                     (:580-582)
    inter_q, s = _mx_quantize(inter)                          (:587-589, 252-271: one shared
             exponent per 32 contiguous values = max biased fp32 exponent - 7, codes
             clip(inter / 2^(e-127), +-448) rounded to e4m3fn, :599)
    out   = (inter_q * s) @ (Wd_q * wd_scale) + bd           (:593-596), returned as bf16 (the
                                                             kernel's ``output_dtype="bfloat16"``)

Pinned by ``tests/golden/mlp_row_mx.npz``: outputs of the reference's own ``_mlp_ref_standard`` and
``_mx_quantize`` run from its source (``make_golden.py mlp_row_mx``), equal bit for bit. That run
stands in for helpers outside the reference tree: the MX block size ``_q_height * _q_width`` (from the
unvendored ``nkilib.core.mlp.mlp_tkg.projection_mx_constants``) is taken as 32, the MX block of the
rest of the reference (``adaln_quant_torch.py:151-175``); the fp8 round trip, the fp32 exponent
extraction and the weight-layout undo are replaced by their plain equivalents. The exponent clip to
[0, 255] (a UE8M0 byte) only differs from the unclipped reference in the scale of all-zero or
sub-2^-120 blocks, whose codes and dequantised values are the same.
"""

from __future__ import annotations

import numpy as np

from .adaln import mx_quantize
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


def wan_mlp_row_mx_ref(x_codes, row_scale, wu_codes, wu_scale, bu, wd_codes, wd_scale, bd) -> np.ndarray:
    """ROW_MX MLP on ``[T, H]`` e4m3 codes (float values) with per-row fp32 ``row_scale [T]``.
    ``wu_codes [I, H]`` / ``wd_codes [H_out, I]`` are the e4m3 weight codes (float values, K-major:
    W^T), ``wu_scale [I]`` / ``wd_scale [H_out]`` fp32 per-channel scales, ``bu`` / ``bd`` the bf16
    biases (float values, or None). Returns the bf16 output ``[T, H_out]`` as float32."""
    x = np.asarray(x_codes, np.float32) * np.asarray(row_scale, np.float32).reshape(-1, 1)
    wu = np.asarray(wu_codes, np.float32) * np.asarray(wu_scale, np.float32).reshape(-1, 1)
    up = x @ wu.T
    if bu is not None:
        up = up + np.asarray(bu, np.float32).reshape(1, -1)
    inter = gelu_tanh(up)
    _, _, inter_dq = mx_quantize(inter)
    wd = np.asarray(wd_codes, np.float32) * np.asarray(wd_scale, np.float32).reshape(-1, 1)
    out = inter_dq @ wd.T
    if bd is not None:
        out = out + np.asarray(bd, np.float32).reshape(1, -1)
    return bf16_round(out.astype(np.float32))


def wan_mlp_row_mx_intermediate_ref(x_codes, row_scale, wu_codes, wu_scale, bu):
    """The up-projection half: (codes, UE8M0 scale bytes [T, I/32], dequantised) of the MX-32
    intermediate, for checking the up kernel's epilogue on its own."""
    x = np.asarray(x_codes, np.float32) * np.asarray(row_scale, np.float32).reshape(-1, 1)
    wu = np.asarray(wu_codes, np.float32) * np.asarray(wu_scale, np.float32).reshape(-1, 1)
    up = x @ wu.T
    if bu is not None:
        up = up + np.asarray(bu, np.float32).reshape(1, -1)
    return mx_quantize(gelu_tanh(up))
