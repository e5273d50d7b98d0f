"""CPU restatement of one Wan2.2 transformer block with bf16 leaves (``WanTransformerBlock.forward``,
vllm_omni_neuron/diffusion/models/wan2_2/wan2_2_transformer.py:1428-1513), composed from the pinned
restatements: adaLN (``adaln_modulate_oracle``), the bf16 self-attention projection order (:1097-1114:
matmul + bias, ``DistributedRMSNorm`` :879-893, interleaved ``apply_rotary_emb_wan``), exact attention
(``torch_attend``), ``_wan_o_proj``, cross-attention (``project_kv`` :1237-1258, ``_project_query``
:1232-1235), and ``_wan_mlp``. Small shapes only (it is plain numpy).
"""

from __future__ import annotations

import numpy as np

from .adaln import adaln_modulate_oracle
from .attention import torch_attend
from .ffn import wan_mlp_ref, wan_mlp_row_mx_ref
from .numerics import bf16_round, e4m3fn_from_bits
from .oproj import wan_o_proj_ref
from .rope import apply_rotary_emb_wan, distributed_rms_norm


def _linear(x, w, b):
    y = bf16_round(np.asarray(x, np.float32) @ np.asarray(w, np.float32))
    return bf16_round(y + np.asarray(b, np.float32).reshape(1, -1)) if b is not None else y


def project_kv_ref(ctx, k_w, k_b, norm_k_w, v_w, v_b, heads, eps):
    B, L, H = ctx.shape
    x = ctx.reshape(B * L, H)
    k = distributed_rms_norm(_linear(x, k_w, k_b), norm_k_w, eps).reshape(B, L, heads, 128)
    v = _linear(x, v_w, v_b).reshape(B, L, heads, 128)
    return k, v


def _attend_dmajor(q_tok, k_tok, v_tok, scale):
    """token-major [B, S, N, D] inputs -> _torch_attend on [B, N, S, D] -> d-major [B, N, D, S]."""
    o = torch_attend(q_tok.transpose(0, 2, 1, 3), k_tok.transpose(0, 2, 1, 3), v_tok.transpose(0, 2, 1, 3), scale)
    return np.ascontiguousarray(bf16_round(o).transpose(0, 1, 3, 2))


def wan_block_ref(hidden, temb, cos, sin, cross_kv, w: dict, heads: int, eps: float = 1e-6, ffn_fp8=None):
    """hidden [B, S, H]; temb [B, 6, H]; cos/sin interleaved RoPE tables [S, 128]; w: reference parameter names.
    ``ffn_fp8``: (up codes [I, H], up scale [I], down codes [H, I], down scale [H]) as float arrays runs the
    FFN as the FP8 leaf (WanFeedForwardFP8, row_mx_modules.py:549-708): norm3 with ROW quant, then the
    ROW_MX MLP (``wan_mlp_row_mx_ref``)."""
    B, S, H = hidden.shape
    N = heads
    scale = 1.0 / np.sqrt(128)
    mods = np.asarray(w["scale_shift_table"], np.float32).reshape(1, 6, H) + np.asarray(temb, np.float32)
    shift, scl, gate, c_shift, c_scl, c_gate = (mods[:, i:i + 1, :] for i in range(6))
    norm_h = adaln_modulate_oracle(hidden, 1 + scl, shift, eps=eps, norm_type="layer_norm")
    qkv = _linear(norm_h.reshape(B * S, H), w["attn1.qkv_proj_weight"], w["attn1.qkv_proj_bias"]).reshape(B, S, 3 * H)
    q, k, v = qkv[..., :H], qkv[..., H:2 * H], qkv[..., 2 * H:]
    q = distributed_rms_norm(q, w["attn1.norm_q.weight"], eps).reshape(B, S, N, 128)
    k = distributed_rms_norm(k, w["attn1.norm_k.weight"], eps).reshape(B, S, N, 128)
    c4 = np.asarray(cos, np.float32).reshape(1, S, 1, 128)
    s4 = np.asarray(sin, np.float32).reshape(1, S, 1, 128)
    q = apply_rotary_emb_wan(q, c4, s4)
    k = apply_rotary_emb_wan(k, c4, s4)
    attn = _attend_dmajor(q, k, v.reshape(B, S, N, 128), scale)
    y = wan_o_proj_ref(attn, w["attn1.o_proj_weight"], w["attn1.o_proj_bias"])
    norm2 = "layer_norm" if w.get("norm2.weight") is not None else "none"
    hidden, norm_h = adaln_modulate_oracle(y, w.get("norm2.weight"), w.get("norm2.bias"), eps=eps, norm_type=norm2,
                                           residual=hidden, gate=gate)
    cq = distributed_rms_norm(_linear(norm_h.reshape(B * S, H), w["attn2.q_proj_weight"], w["attn2.q_proj_bias"]),
                              w["attn2.norm_q.weight"], eps).reshape(B, S, N, 128)
    attn2 = _attend_dmajor(cq, cross_kv[0], cross_kv[1], scale)
    y2 = wan_o_proj_ref(attn2, w["attn2.o_proj_weight"], w["attn2.o_proj_bias"])
    if ffn_fp8 is not None:
        hidden, packed = adaln_modulate_oracle(y2, 1 + c_scl, c_shift, eps=eps, norm_type="layer_norm", quant="row",
                                               residual=hidden)
        packed = np.ascontiguousarray(packed).reshape(B * S, H + 4)
        codes = e4m3fn_from_bits(packed[:, :H])
        rs = np.ascontiguousarray(packed[:, H:]).view(np.float32).reshape(-1)
        uc, us, dc, ds = ffn_fp8
        f = wan_mlp_row_mx_ref(codes, rs, uc, us, w["ffn.up_bias"], dc, ds, w["ffn.down_bias"]).reshape(B, S, H)
        return bf16_round(np.asarray(hidden, np.float32) + np.asarray(f, np.float32) * c_gate)
    hidden, norm_h = adaln_modulate_oracle(y2, 1 + c_scl, c_shift, eps=eps, norm_type="layer_norm", residual=hidden)
    f = wan_mlp_ref(norm_h, w["ffn.up_weight"], w["ffn.down_weight"], w["ffn.up_bias"], w["ffn.down_bias"])
    return bf16_round(np.asarray(hidden, np.float32) + np.asarray(f, np.float32) * c_gate)


def wan_output_head_ref(hidden, temb, table, proj_w, proj_b, eps: float = 1e-6):
    """wan2_2_transformer.py:1824-1829: ``(norm_out(h.float()) * (1 + scale) + shift).type_as(h)`` with
    norm_out a LayerNorm without affine parameters and ``shift, scale = (table + temb[:, None]).chunk(2)``,
    then ``proj_out`` (``nn.Linear``, x @ W.T + b on bf16 tensors)."""
    h = np.asarray(hidden, np.float32)
    mods = np.asarray(table, np.float32).reshape(1, 2, -1) + np.asarray(temb, np.float32)[:, None, :]
    shift, scale = mods[:, 0:1, :], mods[:, 1:2, :]
    mean = h.mean(-1, keepdims=True)
    var = ((h - mean) ** 2).mean(-1, keepdims=True)
    y = bf16_round((h - mean) / np.sqrt(var + np.float32(eps)) * (1 + scale) + shift)
    B, S, H = h.shape
    return _linear(y.reshape(B * S, H), np.asarray(proj_w, np.float32).T, proj_b).reshape(B, S, -1)
