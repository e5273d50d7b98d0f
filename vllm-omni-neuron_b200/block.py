"""One Wan2.2 transformer block on B200 — ``WanTransformerBlock.forward``
(vllm_omni_neuron/diffusion/models/wan2_2/wan2_2_transformer.py:1428-1513), bf16 leaves:

1. norm1: ``adaln_modulate(hidden, 1 + scale_msa, shift_msa)`` (LayerNorm);
2. self-attention (``WanSelfAttention.forward``, :1093-1143): fused QKV projection with the per-head
   sums of squares in the GEMM epilogue, ``DistributedRMSNorm`` on Q and K plus Wan's interleaved
   RoPE as one apply pass (Q/K head dims de-interleaved at load time so the RoPE is rotate-half,
   the identity the reference's FP8 loaders use, row_mx_loaders.py:26-71), the const-max (ring)
   attention over the CP group, d-major out;
3. o-projection with the gated residual ``hidden + gate_msa * attn1_out`` fused into its epilogue,
   then norm2 (:1470-1489);
4. cross-attention (``WanCrossAttention.forward``, :1302-1326): Q projection + RMS norm, exact
   attention over the pre-projected text K/V (``project_kv``, :1237-1271, once per generation),
   o-projection with the un-gated residual fused, then norm3 (:1497-1506);
5. FFN with the closing ``hidden + c_gate_msa * ffn(norm_h)`` fused into the down projection (:1510).

Every GEMM, norm, attention and residual runs in ``libvomni_b200.so``; only the six [B, H]
modulation vectors are formed with torch (``scale_shift_table + temb``, :1459-1461).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import _lib
from .adaln import adaln_modulate
from .attention import wan_cp_self_attention
from .ffn import _gemm, quantize_mlp_weights_row_mx, row_mx_mlp, wan_mlp_gated_residual
from .oproj import o_proj_gated_residual
from .rope import deinterleave_gamma_row, deinterleave_qk_columns


@dataclass
class BlockWeights:
    """bf16 weights of one block in the layouts the B200 kernels read (see :func:`prepare_block_weights`)."""

    scale_shift_table: torch.Tensor  # [1, 6, H] fp32
    qkv_w: torch.Tensor  # [H, 3H], Q/K head dims de-interleaved
    qkv_b: torch.Tensor  # [3H]
    norm_q_w: torch.Tensor  # [H], de-interleaved
    norm_k_w: torch.Tensor  # [H], de-interleaved
    o_w: torch.Tensor  # [H, H]
    o_b: torch.Tensor  # [H]
    norm2_w: torch.Tensor | None  # [H] (cross_attn_norm) or None
    norm2_b: torch.Tensor | None
    cq_w: torch.Tensor  # [H, H]
    cq_b: torch.Tensor
    c_norm_q_w: torch.Tensor  # [H]
    co_w: torch.Tensor  # [H, H]
    co_b: torch.Tensor
    ffn_up_w: torch.Tensor  # [H, I]
    ffn_up_b: torch.Tensor
    ffn_down_w: torch.Tensor  # [I, H]
    ffn_down_b: torch.Tensor
    heads: int
    eps: float = 1e-6
    # FP8 FFN leaf (WanFeedForwardFP8, row_mx_modules.py:549-708): (up codes [I, H], up scale [I],
    # down codes [H, I], down scale [H]); when set the block runs norm3 with ROW quant and row_mx_mlp
    ffn_fp8: tuple | None = None


def prepare_block_weights(w: dict, heads: int, eps: float = 1e-6, head_dim: int = 128,
                          ffn_fp8: bool | tuple = False) -> BlockWeights:
    """From the reference's parameter names (``attn1.qkv_proj_weight`` [H, 3H] etc.) to
    :class:`BlockWeights`: Q/K columns and the Q/K norm weights de-interleaved (row_mx_loaders.py:26-71).
    ``ffn_fp8``: True quantises the FFN weights per tensor for the FP8 leaf
    (``quantize_mlp_weights_row_mx``); a ``(up codes, up scale, down codes, down scale)`` tuple (e.g.
    ``checkpoint.fp8_ffn_leaf``) is used as given."""
    H = w["attn1.qkv_proj_weight"].shape[0]
    qd = heads * head_dim
    bf = lambda t: t.to(torch.bfloat16).contiguous()
    qkv_w = deinterleave_qk_columns(w["attn1.qkv_proj_weight"], qd, qd, head_dim)
    qkv_b = deinterleave_qk_columns(w["attn1.qkv_proj_bias"].reshape(1, -1), qd, qd, head_dim).reshape(-1)
    return BlockWeights(
        scale_shift_table=w["scale_shift_table"].float().reshape(1, 6, H).contiguous(),
        qkv_w=bf(qkv_w), qkv_b=bf(qkv_b),
        norm_q_w=bf(deinterleave_gamma_row(w["attn1.norm_q.weight"].reshape(1, -1), head_dim).reshape(-1)),
        norm_k_w=bf(deinterleave_gamma_row(w["attn1.norm_k.weight"].reshape(1, -1), head_dim).reshape(-1)),
        o_w=bf(w["attn1.o_proj_weight"]), o_b=bf(w["attn1.o_proj_bias"]),
        norm2_w=bf(w["norm2.weight"]) if w.get("norm2.weight") is not None else None,
        norm2_b=bf(w["norm2.bias"]) if w.get("norm2.bias") is not None else None,
        cq_w=bf(w["attn2.q_proj_weight"]), cq_b=bf(w["attn2.q_proj_bias"]),
        c_norm_q_w=bf(w["attn2.norm_q.weight"]),
        co_w=bf(w["attn2.o_proj_weight"]), co_b=bf(w["attn2.o_proj_bias"]),
        ffn_up_w=bf(w["ffn.up_weight"]), ffn_up_b=bf(w["ffn.up_bias"]),
        ffn_down_w=bf(w["ffn.down_weight"]), ffn_down_b=bf(w["ffn.down_bias"]),
        heads=heads, eps=eps,
        ffn_fp8=(quantize_mlp_weights_row_mx(w["ffn.up_weight"], w["ffn.down_weight"]) if ffn_fp8 is True
                 else (tuple(ffn_fp8) if ffn_fp8 else None)),
    )


def _linear_normed(x2: torch.Tensor, w: torch.Tensor, b, n_norm_heads: int):
    """bf16(bf16(x @ w) + b) and the per-head sums of squares of its first n_norm_heads heads."""
    m, k = x2.shape
    n = w.shape[1]
    out = torch.empty(m, n, dtype=torch.bfloat16, device=x2.device)
    sumsq = torch.empty(m, n_norm_heads, dtype=torch.float32, device=x2.device)
    _lib.check(
        _lib.load().vomni_linear_sumsq(x2.data_ptr(), m, k, w.data_ptr(), b.data_ptr() if b is not None else None, n,
                                       sumsq.data_ptr(), n_norm_heads, out.data_ptr(),
                                       torch.cuda.current_stream(x2.device).cuda_stream),
        "vomni_linear_sumsq",
    )
    return out, sumsq


def _norm_rope(y, sumsq, q_heads, kv_heads, eps, gamma_q, gamma_k, cos=None, sin=None):
    T, I = y.shape
    ptr = lambda t: t.data_ptr() if t is not None else None
    _lib.check(
        _lib.load().vomni_qk_norm_rope(y.data_ptr(), T, I, q_heads, kv_heads, 128, sumsq.data_ptr(), float(eps),
                                       ptr(gamma_q), ptr(gamma_k), ptr(cos), ptr(sin),
                                       torch.cuda.current_stream(y.device).cuda_stream),
        "vomni_qk_norm_rope",
    )


def project_cross_kv(context: torch.Tensor, k_w, k_b, norm_k_w, v_w, v_b, heads: int, eps: float = 1e-6):
    """``WanCrossAttention.project_kv`` (:1237-1258) for a text context ``[B, L, H]``: K = RMSNorm(ctx @ Wk + bk),
    V = ctx @ Wv + bv, returned token-major ``[B, L, heads, 128]`` (done once per generation)."""
    B, L, H = context.shape
    x2 = context.reshape(B * L, H).to(torch.bfloat16).contiguous()
    k, ss = _linear_normed(x2, k_w.to(torch.bfloat16).contiguous(), k_b.to(torch.bfloat16), heads)
    _norm_rope(k, ss, heads, 0, eps, norm_k_w.to(torch.bfloat16).contiguous(), None)
    v = _gemm(x2, v_w.to(torch.bfloat16).contiguous(), v_b, 0)
    return k.reshape(B, L, heads, 128), v.reshape(B, L, heads, 128)


def cross_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float) -> torch.Tensor:
    """Exact attention of the local queries ``[B, S, N, 128]`` over the text K/V ``[B, L, N, 128]`` (token-major
    views), d-major ``[B, N, 128, S]`` out — ``_nki_attend`` (:653-674) through the const-max kernel."""
    from .attention import token_major

    B, S, N, D = q.shape
    L = k.shape[1]
    q, qs = token_major(q)
    k, ks = token_major(k)
    v, vs = token_major(v)
    if ks != vs:
        k, v = k.contiguous(), v.contiguous()
        ks = N * D
    lib = _lib.load()
    out = torch.empty(B, N, D, S, dtype=torch.bfloat16, device=q.device)
    ws_bytes = lib.vomni_cm_workspace_bytes(B, S, N, D)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device)
    _lib.check(
        lib.vomni_cm_attention_cross(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), None, B, S, L, N, D, qs, ks,
                                     float(scale), _lib.CM_OUT_DMAJOR, ws.data_ptr(), ws_bytes,
                                     torch.cuda.current_stream(q.device).cuda_stream),
        "vomni_cm_attention_cross",
    )
    return out


def wan_block_forward(hidden_states: torch.Tensor, temb: torch.Tensor, rotary_rh, cross_kv, w: BlockWeights, *,
                      cp_size: int = 1, cp_group=None, cp_replica_groups=None) -> torch.Tensor:
    """``hidden_states`` [B, S_loc, H] bf16 (this CP rank's tokens); ``temb`` [B, 6, H]; ``rotary_rh``: the
    rotate-half ``(cos, sin)`` caches [S_loc, 128] of this rank's tokens (``rope_rotate_half_caches``);
    ``cross_kv``: ``project_cross_kv`` output. Returns the block output [B, S_loc, H] bf16."""
    B, S, H = hidden_states.shape
    N = w.heads
    eps = w.eps
    mods = (w.scale_shift_table + temb.float()).chunk(6, dim=1)  # :1459-1461
    shift_msa, scale_msa, gate_msa, c_shift_msa, c_scale_msa, c_gate_msa = mods
    hidden_states = hidden_states.contiguous()
    norm_h = adaln_modulate(hidden_states, 1 + scale_msa, shift_msa, eps=eps, norm_type="layer_norm")
    # self-attention (bf16 leaf)
    qkv, ss = _linear_normed(norm_h.reshape(B * S, H), w.qkv_w, w.qkv_b, 2 * N)
    cos, sin = rotary_rh
    cos = cos.reshape(-1, 128).float()
    sin = sin.reshape(-1, 128).float()
    if cos.shape[0] != B * S:
        cos, sin = cos.repeat(B, 1).contiguous(), sin.repeat(B, 1).contiguous()
    _norm_rope(qkv, ss, N, N, eps, w.norm_q_w, w.norm_k_w, cos, sin)
    qkv = qkv.reshape(B, S, 3 * H)
    q, k, v = (t.unflatten(2, (N, 128)) for t in torch.tensor_split(qkv, 3, dim=-1))
    attn = wan_cp_self_attention(q, k, v, 1.0 / math.sqrt(128), cp_size, cp_group, cp_replica_groups)
    # o-proj + gated residual, norm2
    hidden_states = o_proj_gated_residual(attn, w.o_w, w.o_b, hidden_states, gate_msa)
    norm2_type = "layer_norm" if w.norm2_w is not None else "none"
    norm_h = adaln_modulate(hidden_states, w.norm2_w, w.norm2_b, eps=eps, norm_type=norm2_type)
    # cross-attention, o-proj + residual, norm3
    cq, ss2 = _linear_normed(norm_h.reshape(B * S, H), w.cq_w, w.cq_b, N)
    _norm_rope(cq, ss2, N, 0, eps, w.c_norm_q_w, None)
    attn2 = cross_attention(cq.reshape(B, S, N, 128), cross_kv[0], cross_kv[1], 1.0 / math.sqrt(128))
    hidden_states = o_proj_gated_residual(attn2, w.co_w, w.co_b, hidden_states, None)
    if w.ffn_fp8 is not None:
        # FP8 leaf: norm3 emits ROW-quantised rows (row_mx_modules.py:647-660), the ROW_MX MLP adds the
        # closing gated residual in its down-projection epilogue
        packed = adaln_modulate(hidden_states, 1 + c_scale_msa, c_shift_msa, eps=eps, norm_type="layer_norm",
                                quant="row", row_layout="split")
        uc, us, dc, ds = w.ffn_fp8
        return row_mx_mlp(packed, uc, dc, us, ds, w.ffn_up_b, w.ffn_down_b, residual=hidden_states, gate=c_gate_msa)
    norm_h = adaln_modulate(hidden_states, 1 + c_scale_msa, c_shift_msa, eps=eps, norm_type="layer_norm")
    # FFN + closing gated residual
    return wan_mlp_gated_residual(hidden_states, norm_h, w.ffn_up_w, w.ffn_down_w, w.ffn_up_b, w.ffn_down_b, c_gate_msa)
