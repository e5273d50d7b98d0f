"""CPU restatement of the ROW_MX fused QKV projection and its across-heads norm + RoPE epilogue.

Follows ``_qkv_cte_mx_impl`` (vllm_omni_neuron/kernels/nkilib/core/qkv/qkv_cte.py:2725-3993):

1. ``Y = (Xq @ Wq) * row_scale[s] * chan_scale[i] + bias[i]`` (``_dequant_row_mx``, :3996-4021;
   the MX engine runs with identity micro-scales, common_types.py:77-78), stored bf16.
2. Across-heads RMS (DistributedRMSNorm over the whole Q or K segment): per-token sum of
   squares of the stored Q (and K) segment, ``inv_rms = rsqrt(sum / (n_heads * d) + eps)``
   (:3870-3898).
3. Apply pass (:3903-3991): ``x * gamma`` (segment-wide per-channel gamma), then rotate-half
   RoPE with ``inv_rms`` folded into the multiplies: ``out = x*inv*cos + [-x_hi, x_lo]*inv*sin``
   (``_rope_segment`` :4069-4114). Without fused RoPE: ``x * inv_rms * gamma``.

Also the MX-32 variant named by the benchmark configuration: activations and weights each carry
one UE8M0 scale per 32 consecutive contraction elements (``_mx_dequant`` semantics,
adaln_quant_torch.py:151-175), ``Y = sum_blocks dequant(X) dequant(W) + bias``, same epilogue.
"""

from __future__ import annotations

import numpy as np

from .adaln import mx_quantize
from .numerics import FP8_E4M3FN_MAX, bf16_round, e4m3fn_from_bits, e4m3fn_round


def unpack_row(packed: np.ndarray):
    """[..., H+4] uint8 -> (codes float32 [..., H], row scale float32 [...])."""
    packed = np.ascontiguousarray(packed)
    codes = e4m3fn_from_bits(packed[..., :-4])
    scale = packed[..., -4:].copy().view(np.float32)[..., 0]
    return codes, scale


def quantize_weight_per_tensor(w: np.ndarray, q_size: int, kv_size: int):
    """Per-tensor FP8 weight quant for Q/K/V (one scalar per tensor, as the ComfyUI checkpoints
    and ``packed_fused_qkv_scale_loader`` (row_mx_loaders.py:246-260) carry it).

    ``w``: [H, I] float32 with I = q_size + 2*kv_size. Returns (codes [H, I], chan_scale [I]).
    """
    codes = np.empty_like(w, dtype=np.float32)
    chan = np.empty(w.shape[1], np.float32)
    for lo, hi in ((0, q_size), (q_size, q_size + kv_size), (q_size + kv_size, q_size + 2 * kv_size)):
        amax = float(np.abs(w[:, lo:hi]).max())
        sc = np.float32(max(amax / FP8_E4M3FN_MAX, 1e-12))
        codes[:, lo:hi] = e4m3fn_round(w[:, lo:hi] / sc)
        chan[lo:hi] = sc
    return codes, chan


def qkv_epilogue(
    y_bf16: np.ndarray,
    *,
    num_heads: int,
    head_dim: int,
    num_kv_heads: int,
    gamma_q=None,
    gamma_k=None,
    cos=None,
    sin=None,
    eps: float = 1e-6,
):
    """Steps 2-3 on the stored bf16 ``[T, I]`` projection. cos/sin: rotate-half caches [T, d]."""
    y = np.asarray(y_bf16, np.float32).copy()
    q_dim = num_heads * head_dim
    kv_dim = num_kv_heads * head_dim
    half = head_dim // 2
    for lo, n, gamma in ((0, num_heads, gamma_q), (q_dim, num_kv_heads, gamma_k)):
        dim = n * head_dim
        if dim == 0:
            continue
        seg = y[:, lo:lo + dim]
        inv = 1.0 / np.sqrt((seg * seg).sum(axis=-1, keepdims=True) / np.float32(dim) + np.float32(eps))
        x = seg if gamma is None else bf16_round(seg * np.asarray(gamma, np.float32).reshape(1, dim))
        if cos is not None:
            x3 = x.reshape(-1, n, head_dim)
            c = np.asarray(cos, np.float32)[:, None, :]
            s = np.asarray(sin, np.float32)[:, None, :half]
            lo_h, hi_h = x3[..., :half], x3[..., half:]
            inv3 = inv[:, :, None]
            out = np.empty_like(x3)
            out[..., :half] = lo_h * inv3 * c[..., :half] - hi_h * inv3 * s
            out[..., half:] = hi_h * inv3 * c[..., half:] + lo_h * inv3 * s
            y[:, lo:lo + dim] = out.reshape(-1, dim)
        else:
            y[:, lo:lo + dim] = x * inv
    del kv_dim
    return bf16_round(y)


def row_mx_qkv_ref(
    packed: np.ndarray,
    w_codes_hi: np.ndarray,
    chan_scale: np.ndarray,
    bias=None,
    **epilogue,
):
    """ROW mode. ``packed`` [T, H+4] uint8; ``w_codes_hi`` [H, I] float32 e4m3fn-valued codes;
    ``chan_scale`` [I]; ``bias`` [I] (bf16-valued). Returns bf16-valued [T, I]."""
    xc, rs = unpack_row(packed)
    acc = xc.astype(np.float32) @ w_codes_hi.astype(np.float32)
    y = acc * rs[:, None] * np.asarray(chan_scale, np.float32)[None, :]
    if bias is not None:
        y = y + np.asarray(bias, np.float32)[None, :]
    y = bf16_round(y)
    if epilogue:
        y = qkv_epilogue(y, **epilogue)
    return y


def mx32_weight_quant(w: np.ndarray):
    """[H, I] float32 -> MX-32 along H per output column: (codes [H, I], scale_u8 [H//32, I], deq)."""
    codes, sc, deq = mx_quantize(np.ascontiguousarray(w.T))
    return codes.T, sc.T, deq.T


def mx32_qkv_ref(x_deq: np.ndarray, w_deq: np.ndarray, bias=None, **epilogue):
    """MX-32 mode on dequantised operands: [T, H] @ [H, I] + bias, bf16 store, same epilogue."""
    y = x_deq.astype(np.float32) @ w_deq.astype(np.float32)
    if bias is not None:
        y = y + np.asarray(bias, np.float32)[None, :]
    y = bf16_round(y)
    if epilogue:
        y = qkv_epilogue(y, **epilogue)
    return y


def qkv_flops(t: int, h: int, i: int) -> float:
    return 2.0 * t * h * i
