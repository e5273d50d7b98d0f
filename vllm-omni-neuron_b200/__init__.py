"""B200-native (sm_100a) context-parallel self-attention hot path of the Wan2.2-A14B DiT.

Drop-in for the vllm-omni-neuron plugin's attention processor and kernel-call API:

* :func:`ring_attention_const_max_fwd` — const-max ring attention (the NKI kernel's API)
* :func:`wan_cp_self_attention` — the Wan attention processor core
* :func:`adaln_modulate` — fused gated-residual + (Layer|RMS)Norm + modulation + FP8 row quant
* :func:`row_mx_qkv_proj` — FP8 QKV projection with across-heads RMS norm + rotate-half RoPE
* :func:`wan_o_proj`, :func:`attn_out_norm2` — output projection of the d-major attention output,
  with the block's gated residual + norm2 adaLN; :func:`row_mx_o_proj` — its FP8 (ROW) form
* :func:`wan_mlp` — the block's FFN (GELU-tanh MLP); :func:`row_mx_mlp` — its FP8 (ROW_MX) leaf
* :func:`wan_block_forward` — a whole transformer block (self-attn + cross-attn + FFN, bf16 leaves)
* :func:`cfg_gather_combine` — the CFG-parallel gather + combine of the two branch outputs

The same entry points are registered as torch custom operators ``torch.ops.b200omni.*``
(:mod:`.ops`). Compute runs in the C-ABI library ``libvomni_b200.so`` (``include/vomni_b200.h``) built by
:func:`build`.
"""

from .adaln import adaln_modulate
from .attention import attention_local, ring_attention_const_max_fwd, wan_cp_self_attention
from .block import BlockWeights, prepare_block_weights, project_cross_kv, wan_block_forward
from .build import build
from .cfg import cfg_combine, cfg_gather_combine
from .dit import cp_gather_sequence, cp_shard_sequence, wan_blocks_forward, wan_output_head
from .ffn import quantize_mlp_weights_row_mx, row_mx_mlp, wan_mlp
from .leaf import project_cross_kv_fp8, wan_cross_attention_fp8, wan_self_attention_fp8
from .oproj import attn_out_norm2, o_proj_gated_residual, row_mx_o_proj, wan_o_proj
from .qkv import (
    mx32_qkv_proj,
    pack_mx_scales,
    quantize_qkv_weight,
    quantize_qkv_weight_mx32,
    repack_mx_contiguous,
    row_mx_qkv_proj,
)
from .ring import destroy_rings
from . import ops  # registers torch.ops.b200omni.*

__all__ = [
    "BlockWeights",
    "adaln_modulate",
    "attention_local",
    "attn_out_norm2",
    "build",
    "cfg_combine",
    "cfg_gather_combine",
    "cp_gather_sequence",
    "cp_shard_sequence",
    "destroy_rings",
    "mx32_qkv_proj",
    "o_proj_gated_residual",
    "pack_mx_scales",
    "prepare_block_weights",
    "project_cross_kv_fp8",
    "project_cross_kv",
    "quantize_mlp_weights_row_mx",
    "quantize_qkv_weight",
    "quantize_qkv_weight_mx32",
    "repack_mx_contiguous",
    "ring_attention_const_max_fwd",
    "row_mx_mlp",
    "row_mx_o_proj",
    "row_mx_qkv_proj",
    "wan_block_forward",
    "wan_blocks_forward",
    "wan_cp_self_attention",
    "wan_cross_attention_fp8",
    "wan_mlp",
    "wan_o_proj",
    "wan_output_head",
    "wan_self_attention_fp8",
]
