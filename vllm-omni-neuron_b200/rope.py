"""Wan 3-D RoPE tables and the FP8 leaf's weight / cache transforms (torch, host side).

* :func:`wan_rotary_freqs` — ``WanRotaryPosEmbed`` (vllm_omni_neuron/diffusion/layers/rope.py:37-114):
  per-token interleaved ``(cos, sin)`` ``[1, S, 1, head_dim]`` for a ``(frames, height, width)`` latent.
* :func:`apply_rotary_emb_wan` — rope.py:8-34 (interleaved lane pairs).
* :func:`rope_rotate_half_caches` — ``_rope_rotate_half_caches``
  (vllm_omni_neuron/diffusion/quantization/row_mx_modules.py:51-76).
* :func:`deinterleave_perm`, :func:`deinterleave_qk_columns`, :func:`deinterleave_gamma_row` —
  vllm_omni_neuron/diffusion/quantization/row_mx_loaders.py:26-71: the per-head channel permutation
  that lets a rotate-half RoPE reproduce Wan's interleaved RoPE.
"""

from __future__ import annotations

import torch


def _rope_1d(dim: int, max_seq_len: int, theta: float):
    freqs = 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.float64) / dim))
    t = torch.arange(max_seq_len, dtype=torch.float64)
    f = torch.outer(t, freqs)
    return f.cos().float().repeat_interleave(2, dim=-1), f.sin().float().repeat_interleave(2, dim=-1)


def wan_rotary_freqs(head_dim: int, patch_size, max_seq_len: int, latent_fhw, theta: float = 10000.0, device=None):
    """(cos, sin), each ``[1, S, 1, head_dim]`` fp32, for a latent of ``(frames, height, width)``."""
    h_dim = w_dim = 2 * (head_dim // 6)
    t_dim = head_dim - h_dim - w_dim
    parts = [_rope_1d(d, max_seq_len, theta) for d in (t_dim, h_dim, w_dim)]
    fc = torch.cat([p[0] for p in parts], dim=1)
    fs = torch.cat([p[1] for p in parts], dim=1)
    f, hh, ww = latent_fhw
    pt, ph, pw = patch_size
    ppf, pph, ppw = f // pt, hh // ph, ww // pw
    split = [head_dim - 2 * (head_dim // 3), head_dim // 3, head_dim // 3]
    out = []
    for tab in (fc, fs):
        a, b, c = tab.split(split, dim=1)
        a = a[:ppf].view(ppf, 1, 1, -1).expand(ppf, pph, ppw, -1)
        b = b[:pph].view(1, pph, 1, -1).expand(ppf, pph, ppw, -1)
        c = c[:ppw].view(1, 1, ppw, -1).expand(ppf, pph, ppw, -1)
        out.append(torch.cat([a, b, c], dim=-1).reshape(1, ppf * pph * ppw, 1, -1).to(device))
    return out[0], out[1]


def apply_rotary_emb_wan(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Interleaved RoPE on ``[B, S, H, D]`` (fp32 math, result in x's dtype)."""
    x1, x2 = x.unflatten(-1, (-1, 2)).unbind(-1)
    c = cos[..., 0::2]
    s = sin[..., 1::2]
    return torch.stack((x1 * c - x2 * s, x1 * s + x2 * c), dim=-1).flatten(-2, -1).to(x.dtype)


def rope_rotate_half_caches(cos: torch.Tensor, sin: torch.Tensor):
    """Rotate-half caches ``cat([base, base])`` from interleaved tables (row_mx_modules.py:51-76)."""
    base_cos = cos[..., 0::2]
    base_sin = sin[..., 1::2]
    return torch.cat([base_cos, base_cos], dim=-1), torch.cat([base_sin, base_sin], dim=-1)


def deinterleave_perm(head_dim: int) -> torch.Tensor:
    if head_dim % 2:
        raise ValueError(f"head_dim must be even for interleaved RoPE, got {head_dim}")
    idx = torch.arange(head_dim // 2)
    return torch.cat([2 * idx, 2 * idx + 1])


def deinterleave_qk_columns(t: torch.Tensor, q_size: int, kv_size: int, head_dim: int) -> torch.Tensor:
    perm = deinterleave_perm(head_dim).to(t.device)
    q_idx = torch.arange(q_size, device=t.device).reshape(-1, head_dim)[:, perm].flatten()
    k_idx = q_size + torch.arange(kv_size, device=t.device).reshape(-1, head_dim)[:, perm].flatten()
    v_idx = torch.arange(q_size + kv_size, t.shape[-1], device=t.device)
    return t.index_select(-1, torch.cat((q_idx, k_idx, v_idx)))


def deinterleave_gamma_row(gamma: torch.Tensor, head_dim: int) -> torch.Tensor:
    perm = deinterleave_perm(head_dim).to(gamma.device)
    n = gamma.numel() // head_dim
    return gamma.reshape(n, head_dim).index_select(-1, perm).reshape(1, n * head_dim)
