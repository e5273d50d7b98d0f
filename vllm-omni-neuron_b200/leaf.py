"""The FP8 attention leaves: ROW FP8 projections -> const-max attention.

Self-attention (``wan_self_attention_fp8``): fused ROW FP8 QKV projection -> const-max (ring) attention.

Mirrors ``WanSelfAttentionFP8.forward`` (vllm_omni_neuron/diffusion/quantization/row_mx_modules.py:
340-404):

1. rotate-half cos/sin caches from Wan's interleaved RoPE tables (:356-366, ``_rope_rotate_half_caches``);
2. ``row_mx_qkv_proj`` with the across-heads RMS qk-norm (gammas de-interleaved at load time) and the
   fused rotate-half RoPE (:367-389);
3. ``tensor_split`` into Q/K/V token-major views (:390-393) — passed to the attention with their row
   stride, no copy;
4. ``wan_cp_self_attention`` (:395-403), d-major ``[B, N, D, S_loc]`` result;
5. with the o-projection weights given, ``_out_proj`` (:404, 164-204): the FP8 ``row_mx_o_proj``
   (:func:`.oproj.row_mx_o_proj`) of the d-major attention, ``[B, S_loc, H]`` bf16 (TP = 1: no
   head padding, no SP exit).

Cross-attention (``wan_cross_attention_fp8``, ``project_cross_kv_fp8``): ``WanCrossAttentionFP8``
(row_mx_modules.py:407-548) up to the attention output: separate ROW FP8 Q, K and V projections of
the packed rows (Q from the block's norm2 adaLN, K/V from the once-quantised text context), the
across-heads RMS norm on Q and on K (each passing its gamma as the kernel's Q gamma, no RoPE; V not
normed; :478-542), then exact attention over the text tokens, and with the o-projection weights
given the FP8 ``row_mx_o_proj`` (:544-546).
"""

from __future__ import annotations

import math

import torch

from .attention import wan_cp_self_attention
from .block import cross_attention
from .oproj import row_mx_o_proj
from .qkv import row_mx_qkv_proj
from .rope import rope_rotate_half_caches


def wan_self_attention_fp8(
    hidden_states,
    qkv_proj_weight: torch.Tensor,
    qkv_proj_w_scale: torch.Tensor,
    qkv_proj_bias: torch.Tensor | None,
    norm_q_weight: torch.Tensor | None,
    norm_k_weight: torch.Tensor | None,
    rotary_emb=None,
    *,
    num_heads: int,
    head_dim: int = 128,
    eps: float = 1e-6,
    scale: float | None = None,
    cp_size: int = 1,
    cp_group=None,
    cp_replica_groups=None,
    o_proj_weight: torch.Tensor | None = None,
    o_proj_w_scale: torch.Tensor | None = None,
    o_proj_bias: torch.Tensor | None = None,
):
    """``hidden_states``: the packed ``[B, S_loc, H + 4]`` FP8 rows from ``adaln_modulate(quant="row")``
    or its ``(codes, scales)`` split form. Weights are the de-interleaved fused Q|K|V ``[I, H]`` FP8
    codes with per-channel scales (``quantize_qkv_weight`` of ``deinterleave_qk_columns(W)``).
    ``rotary_emb``: Wan's interleaved ``(freqs_cos, freqs_sin)`` for this rank's tokens.
    Without ``o_proj_weight`` the d-major attention ``[B, N, D, S_loc]`` is returned; with it (FP8
    ``[H, N*D]`` codes or the ``[N*D//4, H, 4]`` pack, ``o_proj_w_scale``, ``o_proj_bias``) the
    block's ``[B, S_loc, H]`` attention output, as ``WanSelfAttentionFP8.forward`` returns it."""
    if isinstance(hidden_states, (tuple, list)):
        b, s = hidden_states[0].shape[0], hidden_states[0].shape[1]
    else:
        b, s = hidden_states.shape[0], hidden_states.shape[1]
    cos_cache = sin_cache = None
    if rotary_emb is not None:
        cos_rh, sin_rh = rope_rotate_half_caches(*rotary_emb)
        cos_cache = cos_rh.reshape(1, s, head_dim).expand(b, s, head_dim).contiguous()
        sin_cache = sin_rh.reshape(1, s, head_dim).expand(b, s, head_dim).contiguous()
    qkv = row_mx_qkv_proj(
        hidden_states, qkv_proj_weight, qkv_proj_w_scale, qkv_proj_bias,
        num_heads=num_heads, head_dim=head_dim, num_kv_heads=num_heads,
        fused_rope=rotary_emb is not None, cos_cache=cos_cache, sin_cache=sin_cache,
        qk_norm_pre_rope=True, qk_norm_pre_rope_q_gamma=norm_q_weight, qk_norm_pre_rope_k_gamma=norm_k_weight,
        norm_eps=eps,
    )
    query, key, value = torch.tensor_split(qkv, 3, dim=-1)
    query = query.unflatten(2, (num_heads, head_dim))
    key = key.unflatten(2, (num_heads, head_dim))
    value = value.unflatten(2, (num_heads, head_dim))
    attention = wan_cp_self_attention(
        query, key, value, scale if scale else 1.0 / math.sqrt(head_dim), cp_size, cp_group, cp_replica_groups
    )
    if o_proj_weight is None:
        return attention
    return row_mx_o_proj(attention, o_proj_weight, o_proj_w_scale, o_proj_bias)


def project_cross_kv_fp8(
    packed_encoder_hidden_states,
    k_proj_weight: torch.Tensor,
    k_proj_w_scale: torch.Tensor,
    k_proj_bias: torch.Tensor | None,
    norm_k_weight: torch.Tensor | None,
    v_proj_weight: torch.Tensor,
    v_proj_w_scale: torch.Tensor,
    v_proj_bias: torch.Tensor | None,
    *,
    num_heads: int,
    head_dim: int = 128,
    eps: float = 1e-6,
):
    """``WanCrossAttentionFP8.project_kv`` (row_mx_modules.py:509-542): K with the across-heads RMS
    norm, V plain, from the packed ``[B, L, H + 4]`` text rows; token-major ``[B, L, N, D]`` K and V.
    Weights: ``[N*D, H]`` FP8 codes with per-channel scales (``quantize_qkv_weight(w, N*D, 0)``)."""
    key = row_mx_qkv_proj(packed_encoder_hidden_states, k_proj_weight, k_proj_w_scale, k_proj_bias,
                          num_heads=num_heads, head_dim=head_dim, num_kv_heads=0, qk_norm_pre_rope=True,
                          qk_norm_pre_rope_q_gamma=norm_k_weight, norm_eps=eps)
    value = row_mx_qkv_proj(packed_encoder_hidden_states, v_proj_weight, v_proj_w_scale, v_proj_bias,
                            num_heads=num_heads, head_dim=head_dim, num_kv_heads=0)
    return key.unflatten(-1, (num_heads, head_dim)), value.unflatten(-1, (num_heads, head_dim))


def wan_cross_attention_fp8(
    hidden_states,
    q_proj_weight: torch.Tensor,
    q_proj_w_scale: torch.Tensor,
    q_proj_bias: torch.Tensor | None,
    norm_q_weight: torch.Tensor | None,
    cross_kv,
    *,
    num_heads: int,
    head_dim: int = 128,
    eps: float = 1e-6,
    scale: float | None = None,
    o_proj_weight: torch.Tensor | None = None,
    o_proj_w_scale: torch.Tensor | None = None,
    o_proj_bias: torch.Tensor | None = None,
):
    """``WanCrossAttentionFP8._project_query`` (row_mx_modules.py:478-507) and the attention over the
    text K/V (``project_cross_kv_fp8``): packed ``[B, S, H + 4]`` rows in, d-major ``[B, N, D, S]`` out,
    or with ``o_proj_weight`` the ``[B, S, H]`` output of its FP8 o-projection (:544-546)."""
    query = row_mx_qkv_proj(hidden_states, q_proj_weight, q_proj_w_scale, q_proj_bias, num_heads=num_heads,
                            head_dim=head_dim, num_kv_heads=0, qk_norm_pre_rope=True,
                            qk_norm_pre_rope_q_gamma=norm_q_weight, norm_eps=eps)
    query = query.unflatten(-1, (num_heads, head_dim))
    attention = cross_attention(query, cross_kv[0], cross_kv[1], scale if scale else 1.0 / math.sqrt(head_dim))
    if o_proj_weight is None:
        return attention
    return row_mx_o_proj(attention, o_proj_weight, o_proj_w_scale, o_proj_bias)
