"""torch custom operators (``torch.ops.b200omni.*``) over the B200 kernels.

The reference registers its kernels as torch custom ops with ``nki_op`` so they trace as single
graph nodes (``wan_transformer::attention_cte``, ``::output_projection_cte``, ``::mlp``;
vllm_omni_neuron/diffusion/models/wan2_2/wan2_2_transformer.py:165-171, 230-241, 321-335, registered
through lite_compat.py:88-95) and calls the ring, adaLN and QKV kernels through ``wrap_nki``
(WT:713-728; adaln_kernels.py:127-148; row_mx_kernels.py:79-111). The same entry points are
registered here under the ``b200omni`` namespace, each with a fake (meta) implementation giving
output shapes and dtypes, so a traced or compiled caller sees one opaque node per kernel call:

=====================================  =====================================================
``b200omni::attention_cte``            ``wan_transformer::attention_cte`` contract: q ``[BN, S_q, D]``
                                       already scaled, k/v ``[BN, S_k, D]`` -> d-major ``[BN, D, S_q]``
``b200omni::output_projection_cte``    ``wan_transformer::output_projection_cte`` (= ``wan_o_proj``)
``b200omni::mlp``                      ``wan_transformer::mlp`` (= ``wan_mlp``)
``b200omni::ring_attention_const_max_fwd``  the kernel-call API; the ring's process group by name
``b200omni::adaln_modulate``           the adaLN bridge; list of outputs
``b200omni::row_mx_qkv_proj``          FP8 QKV projection (+ across-heads norm, rotate-half RoPE)
``b200omni::row_mx_mlp``               FP8 FFN leaf
``b200omni::cfg_combine``              CFG combine of two gathered branch outputs
=====================================  =====================================================

Importing this module registers the operators once; the package imports it.
"""

from __future__ import annotations

import math

import torch

from .adaln import adaln_modulate as _adaln
from .attention import ring_attention_const_max_fwd as _ring_fwd
from .block import cross_attention as _cross
from .cfg import cfg_combine as _cfg_combine
from .ffn import row_mx_mlp as _row_mx_mlp
from .ffn import wan_mlp as _wan_mlp
from .oproj import wan_o_proj as _wan_o_proj
from .qkv import row_mx_qkv_proj as _qkv

NS = "b200omni"


def _resolve_group(group_name):
    if group_name is None:
        return None
    from torch.distributed.distributed_c10d import _resolve_process_group

    return _resolve_process_group(group_name)


# ---------------------------------------------------------------- attention_cte


@torch.library.custom_op(f"{NS}::attention_cte", mutates_args=())
def attention_cte(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """``_wan_nki_attention(q_3d, k_3d, v_3d)`` (WT:165-171): non-causal attention with scale 1 on
    pre-scaled ``q [BN, S_q, D]``, ``k, v [BN, S_k, D]``; d-major ``[BN, D, S_q]`` out (tp_out)."""
    BN, S, D = q.shape
    L = k.shape[1]
    out = _cross(q.reshape(BN, S, 1, D), k.reshape(BN, L, 1, D), v.reshape(BN, L, 1, D), 1.0)
    return out.reshape(BN, D, S)


@attention_cte.register_fake
def _(q, k, v):
    BN, S, D = q.shape
    return q.new_empty((BN, D, S), dtype=torch.bfloat16)


# ---------------------------------------------------------------- output_projection_cte


@torch.library.custom_op(f"{NS}::output_projection_cte", mutates_args=())
def output_projection_cte(active: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    """``_wan_nki_o_proj(active [B, N, D, S], weight [N*D, H], bias [1, H])`` -> ``[B, S, H]`` (WT:230-254)."""
    return _wan_o_proj(active, weight, bias)


@output_projection_cte.register_fake
def _(active, weight, bias):
    B, N, D, S = active.shape
    return active.new_empty((B, S, weight.shape[1]), dtype=torch.bfloat16)


# ---------------------------------------------------------------- mlp


@torch.library.custom_op(f"{NS}::mlp", mutates_args=())
def mlp(hidden: torch.Tensor, up_weight: torch.Tensor, down_weight: torch.Tensor, up_bias: torch.Tensor,
        down_bias: torch.Tensor) -> torch.Tensor:
    """``_wan_nki_mlp`` / ``_wan_mlp`` (WT:321-335, 389-410): GELU-tanh MLP, bf16."""
    return _wan_mlp(hidden, up_weight, down_weight, up_bias, down_bias)


@mlp.register_fake
def _(hidden, up_weight, down_weight, up_bias, down_bias):
    return hidden.new_empty(tuple(hidden.shape[:-1]) + (down_weight.shape[1],), dtype=torch.bfloat16)


# ---------------------------------------------------------------- ring attention


@torch.library.custom_op(f"{NS}::ring_attention_const_max_fwd", mutates_args=())
def ring_attention_const_max_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, num_workers: int = 1,
                                 group_name: str | None = None, softmax_scale: float | None = None,
                                 training: bool = False) -> list[torch.Tensor]:
    """The kernel-call API (RING:958-1017) on token-major ``[b, S_loc, h, 128]``: ``[o [b, h, S_loc, 128]]``,
    plus ``lse [b, h, 128, ceil(S_loc/128)]`` when ``training``. ``group_name``: the ring's process group
    (``ProcessGroup.group_name``) when ``num_workers > 1``."""
    res = _ring_fwd(q, k, v, None, num_workers, softmax_scale, training, group=_resolve_group(group_name))
    return list(res) if training else [res]


@ring_attention_const_max_fwd.register_fake
def _(q, k, v, num_workers=1, group_name=None, softmax_scale=None, training=False):
    b, s, h, d = q.shape
    out = [q.new_empty((b, h, s, d), dtype=torch.bfloat16)]
    if training:
        out.append(q.new_empty((b, h, 128, math.ceil(s / 128)), dtype=torch.float32))
    return out


# ---------------------------------------------------------------- adaLN


@torch.library.custom_op(f"{NS}::adaln_modulate", mutates_args=())
def adaln_modulate(hidden: torch.Tensor, mul: torch.Tensor | None, add: torch.Tensor | None, eps: float,
                   norm_type: str = "layer_norm", quant: str = "none", ocp: bool = True,
                   residual: torch.Tensor | None = None, gate: torch.Tensor | None = None) -> list[torch.Tensor]:
    """``adaln_modulate`` (adaln_kernels.py:87-201) as a list: ``[out]`` (``[codes, scales]`` for
    ``quant="mx32"``), preceded by ``residual_out`` when ``residual`` is given."""
    res = _adaln(hidden, mul, add, eps=eps, norm_type=norm_type, quant=quant, ocp=ocp, residual=residual, gate=gate)
    outs = []
    if residual is not None:
        outs.append(res[0])
        res = res[1]
    outs.extend(res if isinstance(res, tuple) else (res,))
    return outs


@adaln_modulate.register_fake
def _(hidden, mul, add, eps, norm_type="layer_norm", quant="none", ocp=True, residual=None, gate=None):
    lead = tuple(hidden.shape[:-1])
    H = hidden.shape[-1]
    outs = [hidden.new_empty(tuple(hidden.shape), dtype=torch.bfloat16)] if residual is not None else []
    if quant == "none":
        outs.append(hidden.new_empty(lead + (H,), dtype=torch.bfloat16))
    elif quant == "row":
        outs.append(hidden.new_empty(lead + (H + 4,), dtype=torch.float8_e4m3fn))
    else:
        outs += [hidden.new_empty(lead + (H,), dtype=torch.float8_e4m3fn),
                 hidden.new_empty(lead + (H // 32,), dtype=torch.uint8)]
    return outs


# ---------------------------------------------------------------- FP8 QKV


@torch.library.custom_op(f"{NS}::row_mx_qkv_proj", mutates_args=())
def row_mx_qkv_proj(packed_hidden: torch.Tensor, weight: torch.Tensor, weight_scales: torch.Tensor,
                    bias: torch.Tensor | None, num_heads: int, head_dim: int, num_kv_heads: int,
                    cos_cache: torch.Tensor | None = None, sin_cache: torch.Tensor | None = None,
                    qk_norm: bool = False, q_gamma: torch.Tensor | None = None, k_gamma: torch.Tensor | None = None,
                    norm_eps: float = 1e-6) -> torch.Tensor:
    """``row_mx_qkv_proj`` (row_mx_kernels.py:48-111): fused RoPE when caches are given, the
    across-heads RMS norm (``qk_norm_pre_rope``) when ``qk_norm``."""
    return _qkv(packed_hidden, weight, weight_scales, bias, num_heads=num_heads, head_dim=head_dim,
                num_kv_heads=num_kv_heads, fused_rope=cos_cache is not None, cos_cache=cos_cache, sin_cache=sin_cache,
                qk_norm_pre_rope=True if qk_norm else None, qk_norm_pre_rope_q_gamma=q_gamma,
                qk_norm_pre_rope_k_gamma=k_gamma, norm_eps=norm_eps)


@row_mx_qkv_proj.register_fake
def _(packed_hidden, weight, weight_scales, bias, num_heads, head_dim, num_kv_heads, cos_cache=None, sin_cache=None,
      qk_norm=False, q_gamma=None, k_gamma=None, norm_eps=1e-6):
    I = (num_heads + 2 * num_kv_heads) * head_dim
    return packed_hidden.new_empty(tuple(packed_hidden.shape[:-1]) + (I,), dtype=torch.bfloat16)


# ---------------------------------------------------------------- FP8 FFN


@torch.library.custom_op(f"{NS}::row_mx_mlp", mutates_args=())
def row_mx_mlp(packed_hidden: torch.Tensor, up_weight: torch.Tensor, down_weight: torch.Tensor,
               up_w_scale: torch.Tensor, down_w_scale: torch.Tensor, up_bias: torch.Tensor | None,
               down_bias: torch.Tensor | None) -> torch.Tensor:
    """``row_mx_mlp`` (row_mx_kernels.py:141-198) on packed ROW rows ``[..., H + 4]``."""
    return _row_mx_mlp(packed_hidden, up_weight, down_weight, up_w_scale, down_w_scale, up_bias, down_bias)


@row_mx_mlp.register_fake
def _(packed_hidden, up_weight, down_weight, up_w_scale, down_w_scale, up_bias, down_bias):
    H = packed_hidden.shape[-1] - 4
    return packed_hidden.new_empty(tuple(packed_hidden.shape[:-1]) + (H,), dtype=torch.bfloat16)


# ---------------------------------------------------------------- CFG combine


@torch.library.custom_op(f"{NS}::cfg_combine", mutates_args=())
def cfg_combine(positive: torch.Tensor, negative: torch.Tensor, true_cfg_scale: float) -> torch.Tensor:
    """``negative + true_cfg_scale * (positive - negative)`` (cfg_parallel.py:71) with torch-eager rounding."""
    return _cfg_combine(positive, negative, true_cfg_scale)


@cfg_combine.register_fake
def _(positive, negative, true_cfg_scale):
    return torch.empty_like(positive)
