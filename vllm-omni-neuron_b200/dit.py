"""DiT-level context parallelism around the B200 blocks — the CP split and gather of
``WanTransformer3DModel.forward`` (vllm_omni_neuron/diffusion/models/wan2_2/wan2_2_transformer.py:1774-1840):

* :func:`cp_shard_sequence`: before the blocks, this rank keeps tokens
  ``[cp_rank * S/cp, (cp_rank + 1) * S/cp)`` of the patchified sequence and the matching rows of the
  RoPE tables (S must divide by cp, as the reference requires, :1775-1780);
* :func:`wan_blocks_forward`: every block in order (each a const-max ring over the CP group);
* :func:`wan_output_head`: the output norm with the head's scale/shift (:1824-1828) and ``proj_out``;
* :func:`cp_gather_sequence`: after the head, the all-gather along the sequence (:1830-1831).

TP / Megatron-SP is not modelled: every rank holds whole heads (TP = 1).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from .adaln import adaln_modulate
from .block import wan_block_forward
from .ffn import _gemm


def cp_shard_sequence(hidden_states: torch.Tensor, rotary_emb, cp_rank: int, cp_size: int):
    """(local hidden [B, S/cp, H], local (cos, sin) [1, S/cp, 1, D]) for this CP rank."""
    S = hidden_states.shape[1]
    if cp_size <= 1:
        return hidden_states, rotary_emb
    if S % cp_size:
        raise ValueError(f"Sequence length {S} is not divisible by cp_size {cp_size}.")
    n = S // cp_size
    sl = slice(cp_rank * n, (cp_rank + 1) * n)
    local = hidden_states[:, sl, :]
    if rotary_emb is None:
        return local, None
    cos, sin = rotary_emb
    return local, (cos[:, sl], sin[:, sl])


def cp_gather_sequence(x: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather ``[B, S/cp, C]`` shards of the CP group along dim 1 (rank order)."""
    world = dist.get_world_size(group)
    if world == 1:
        return x
    x = x.contiguous()
    parts = [torch.empty_like(x) for _ in range(world)]
    dist.all_gather(parts, x, group=group)
    return torch.cat(parts, dim=1)


def wan_blocks_forward(hidden_states, temb_proj, rotary_rh, cross_kvs, blocks, *, cp_size=1, cp_group=None,
                       cp_replica_groups=None):
    """Run ``blocks`` (a list of :class:`BlockWeights`) on this rank's shard; ``cross_kvs`` holds each
    block's ``project_cross_kv`` output (projected once per generation)."""
    for w, kv in zip(blocks, cross_kvs):
        hidden_states = wan_block_forward(hidden_states, temb_proj, rotary_rh, kv, w, cp_size=cp_size,
                                          cp_group=cp_group, cp_replica_groups=cp_replica_groups)
    return hidden_states


def wan_output_head(hidden_states: torch.Tensor, temb: torch.Tensor, scale_shift_table: torch.Tensor,
                    proj_out_weight: torch.Tensor, proj_out_bias: torch.Tensor | None, eps: float = 1e-6):
    """``proj_out((norm_out(h) * (1 + scale) + shift))`` with ``shift, scale = (table + temb[:, None]).chunk(2)``
    (:1824-1829); ``proj_out_weight`` is the ``nn.Linear`` ``[out, in]`` weight."""
    B, S, H = hidden_states.shape
    shift, scale = (scale_shift_table.float() + temb.float().unsqueeze(1)).chunk(2, dim=1)
    y = adaln_modulate(hidden_states.contiguous(), 1 + scale, shift, eps=eps, norm_type="layer_norm")
    w = proj_out_weight.to(torch.bfloat16).t().contiguous()  # [in, out] for x @ W
    out = _gemm(y.reshape(B * S, H), w, proj_out_bias, 0)
    return out.reshape(B, S, -1)
