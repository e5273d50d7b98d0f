"""CPU restatements of Wan's 3-D RoPE, RMSNorm and the de-interleave weight transforms (numpy).

* ``rotary_freqs`` restates ``WanRotaryPosEmbed`` (vllm_omni_neuron/diffusion/layers/rope.py:37-114).
* ``apply_rotary_emb_wan`` restates rope.py:8-34 (interleaved lane pairs (2j, 2j+1)).
* ``rotate_half_caches`` restates ``_rope_rotate_half_caches``
  (vllm_omni_neuron/diffusion/quantization/row_mx_modules.py:51-76).
* ``deinterleave_perm`` / ``deinterleave_qk_columns`` / ``deinterleave_gamma_row`` restate
  vllm_omni_neuron/diffusion/quantization/row_mx_loaders.py:26-71.
* ``distributed_rms_norm`` restates ``DistributedRMSNorm.forward`` at TP=1
  (vllm_omni_neuron/diffusion/models/wan2_2/wan2_2_transformer.py:879-893).
"""

from __future__ import annotations

import numpy as np

from .numerics import bf16_round


def _rope_1d(dim: int, max_seq_len: int, theta: float):
    freqs = 1.0 / (theta ** (np.arange(0, dim, 2, dtype=np.float64) / dim))  # rope.py:80
    t = np.arange(max_seq_len, dtype=np.float64)
    f = np.outer(t, freqs)
    cos = np.repeat(np.cos(f).astype(np.float32), 2, axis=-1)
    sin = np.repeat(np.sin(f).astype(np.float32), 2, axis=-1)
    return cos, sin


def rotary_freqs(head_dim: int, patch_size, max_seq_len: int, latent_fhw, theta: float = 10000.0):
    """WanRotaryPosEmbed(head_dim, patch_size, max_seq_len)(latent) -> (cos, sin) [1, S, 1, head_dim]."""
    h_dim = w_dim = 2 * (head_dim // 6)
    t_dim = head_dim - h_dim - w_dim
    parts = [_rope_1d(dd, max_seq_len, theta) for dd in (t_dim, h_dim, w_dim)]
    fc = np.concatenate([p[0] for p in parts], axis=1)
    fs = np.concatenate([p[1] for p in parts], axis=1)
    f, hh, ww = latent_fhw
    pt, ph, pw = patch_size
    ppf, pph, ppw = f // pt, hh // ph, ww // pw
    split = [head_dim - 2 * (head_dim // 3), head_dim // 3, head_dim // 3]
    idx = np.cumsum([0] + split)
    out = []
    for tab in (fc, fs):
        a = tab[:ppf, idx[0]:idx[1]][:, None, None, :]
        b = tab[:pph, idx[1]:idx[2]][None, :, None, :]
        c = tab[:ppw, idx[2]:idx[3]][None, None, :, :]
        a = np.broadcast_to(a, (ppf, pph, ppw, a.shape[-1]))
        b = np.broadcast_to(b, (ppf, pph, ppw, b.shape[-1]))
        c = np.broadcast_to(c, (ppf, pph, ppw, c.shape[-1]))
        out.append(np.concatenate([a, b, c], axis=-1).reshape(1, ppf * pph * ppw, 1, head_dim).astype(np.float32))
    return out[0], out[1]


def apply_rotary_emb_wan(x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """rope.py:8-34 on ``[B, S, H, D]`` bf16-valued x with fp32 tables; result rounded to bf16."""
    x = np.asarray(x, np.float32)
    x1 = x[..., 0::2]
    x2 = x[..., 1::2]
    c = cos[..., 0::2]
    s = sin[..., 1::2]
    out = np.empty_like(x)
    out[..., 0::2] = x1 * c - x2 * s
    out[..., 1::2] = x1 * s + x2 * c
    return bf16_round(out)


def rotate_half_caches(cos: np.ndarray, sin: np.ndarray):
    """row_mx_modules.py:51-76: base angles duplicated across halves, cat([base, base])."""
    base_cos = cos[..., 0::2]
    base_sin = sin[..., 1::2]
    return np.concatenate([base_cos, base_cos], axis=-1), np.concatenate([base_sin, base_sin], axis=-1)


def deinterleave_perm(head_dim: int) -> np.ndarray:
    """row_mx_loaders.py:26-39: [0,2,...,d-2, 1,3,...,d-1]."""
    if head_dim % 2:
        raise ValueError(f"head_dim must be even for interleaved RoPE, got {head_dim}")
    half = head_dim // 2
    idx = np.arange(half)
    return np.concatenate([2 * idx, 2 * idx + 1])


def deinterleave_qk_columns(t: np.ndarray, q_size: int, kv_size: int, head_dim: int) -> np.ndarray:
    """row_mx_loaders.py:42-59: permute each Q and K head's lanes on the last axis, V untouched."""
    perm = deinterleave_perm(head_dim)
    q_idx = np.arange(q_size).reshape(-1, head_dim)[:, perm].reshape(-1)
    k_idx = q_size + np.arange(kv_size).reshape(-1, head_dim)[:, perm].reshape(-1)
    v_idx = np.arange(q_size + kv_size, t.shape[-1])
    return np.take(t, np.concatenate([q_idx, k_idx, v_idx]), axis=-1)


def deinterleave_gamma_row(gamma: np.ndarray, head_dim: int) -> np.ndarray:
    """row_mx_loaders.py:62-71: per-head permuted gamma as a [1, n*d] row."""
    perm = deinterleave_perm(head_dim)
    n = gamma.size // head_dim
    return gamma.reshape(n, head_dim)[:, perm].reshape(1, n * head_dim)


def distributed_rms_norm(x: np.ndarray, weight: np.ndarray, eps: float) -> np.ndarray:
    """wan2_2_transformer.py:879-893 at tp_size == 1, bf16 in / bf16 out."""
    xf = np.asarray(x, np.float32)
    ss = (xf * xf).sum(axis=-1, keepdims=True)
    rms = np.sqrt(ss / xf.shape[-1] + np.float32(eps))
    return bf16_round((xf / rms) * np.asarray(weight, np.float32))
