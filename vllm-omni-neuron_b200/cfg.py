"""CFG-parallel gather + combine on B200: the reference's ``_cfg_gather_combine(local_pred,
true_cfg_scale)`` (vllm_omni_neuron/diffusion/distributed/cfg_parallel.py:48-71).

Each CFG rank holds its branch's predicted noise (rank 0 the positive / conditional branch, rank 1
the negative one, CFGP:124-151). The two are all-gathered over the CFG group (NCCL over NVLink; a
latent of a few MB per denoising step) and combined as ``neg + scale * (pos - neg)`` by
``vomni_cfg_combine``, whose rounding equals torch eager's for that expression, so every rank
obtains the same tensor and it equals sequential CFG bit for bit.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import _lib

_DTYPES = {torch.float32: 0, torch.bfloat16: 1}  # VOMNI_CFG_F32 / VOMNI_CFG_BF16


def cfg_combine(positive: torch.Tensor, negative: torch.Tensor, true_cfg_scale: float, out: torch.Tensor | None = None) -> torch.Tensor:
    """``negative + true_cfg_scale * (positive - negative)`` on the GPU (CFGP:71)."""
    if positive.shape != negative.shape or positive.dtype != negative.dtype:
        raise ValueError(f"branch outputs differ: {tuple(positive.shape)} {positive.dtype} vs "
                         f"{tuple(negative.shape)} {negative.dtype}")
    if positive.dtype not in _DTYPES:
        raise TypeError(f"unsupported dtype {positive.dtype} (float32 or bfloat16)")
    if not (positive.is_cuda and negative.is_cuda):
        raise RuntimeError("cfg_combine needs CUDA tensors (the B200 kernel has no CPU path)")
    pos = positive.contiguous()
    neg = negative.contiguous()
    if out is None:
        out = torch.empty_like(pos)
    _lib.check(
        _lib.load().vomni_cfg_combine(pos.data_ptr(), neg.data_ptr(), out.data_ptr(), pos.numel(), _DTYPES[pos.dtype],
                                      float(true_cfg_scale), torch.cuda.current_stream(pos.device).cuda_stream),
        "vomni_cfg_combine",
    )
    return out


def cfg_gather_combine(local_pred: torch.Tensor, true_cfg_scale: float, cfg_group=None) -> torch.Tensor:
    """All-gather the two CFG branches over ``cfg_group`` and apply the combine (CFGP:48-71).

    ``cfg_group``: the CFG group's torch process group (``get_cfg_group().device_group`` in the
    reference), ``None`` for the default group. It must have exactly two ranks: index 0 of the
    gather is the positive branch, index 1 the negative one. Collective: every CFG rank calls it.
    """
    world = dist.get_world_size(cfg_group)
    if world != 2:
        raise ValueError(f"CFG-parallel combine needs a CFG group of 2 ranks, got {world}")
    if isinstance(local_pred, tuple):
        raise NotImplementedError("multi-output (tuple) predict_noise is not supported under cfg-parallel (CFGP:152-159)")
    x = local_pred.contiguous()
    gathered = torch.empty((2,) + tuple(x.shape), dtype=x.dtype, device=x.device)
    dist.all_gather_into_tensor(gathered, x, group=cfg_group)
    return cfg_combine(gathered[0], gathered[1], true_cfg_scale)
