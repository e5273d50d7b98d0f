"""Wan FFN on B200: the reference's ``_wan_mlp(hidden, up_weight, down_weight, up_bias, down_bias)``
(vllm_omni_neuron/diffusion/models/wan2_2/wan2_2_transformer.py:389-410):
``GELU_tanh(hidden @ up_weight + up_bias) @ down_weight + down_bias`` with torch's bf16 rounding
after each matmul and bias add, the GELU in fp32 opmath. Two CTA-pair tcgen05 GEMMs; the first
applies the bias and GELU-tanh in its epilogue, so the ``[T, I]`` intermediate is written once, bf16.
"""

from __future__ import annotations

import torch

from . import _lib


def _gemm(x2: torch.Tensor, w: torch.Tensor, bias, act: int, residual=None, gate=None, gate_rows: int = 0) -> torch.Tensor:
    m, k = x2.shape
    k2, n = w.shape
    if k != k2:
        raise ValueError(f"inner dims differ: {k} vs {k2}")
    b = bias.reshape(-1).to(torch.bfloat16).contiguous() if bias is not None else None
    if b is not None and b.numel() != n:
        raise ValueError(f"bias has {b.numel()} values for {n} columns")
    out = torch.empty(m, n, dtype=torch.bfloat16, device=x2.device)
    _lib.check(
        _lib.load().vomni_ffn_gemm(x2.data_ptr(), m, k, w.data_ptr(), b.data_ptr() if b is not None else None, n, act,
                                   residual.data_ptr() if residual is not None else None,
                                   gate.data_ptr() if gate is not None else None, gate_rows, out.data_ptr(),
                                   torch.cuda.current_stream(x2.device).cuda_stream),
        "vomni_ffn_gemm",
    )
    return out


def wan_mlp(hidden: torch.Tensor, up_weight: torch.Tensor, down_weight: torch.Tensor, up_bias, down_bias) -> torch.Tensor:
    """``[B, T, H]`` bf16 -> ``[B, T, H_out]`` bf16."""
    for name, t in (("hidden", hidden), ("up_weight", up_weight), ("down_weight", down_weight)):
        if t.dtype != torch.bfloat16:
            raise TypeError(f"{name} must be bfloat16, got {t.dtype}")
        if not t.is_cuda:
            raise RuntimeError(f"{name} must be a CUDA tensor (the B200 kernel has no CPU path)")
    lead = tuple(hidden.shape[:-1])
    x2 = hidden.reshape(-1, hidden.shape[-1]).contiguous()
    up = _gemm(x2, up_weight.contiguous(), up_bias, 1)
    out = _gemm(up, down_weight.contiguous(), down_bias, 0)
    return out.reshape(lead + (down_weight.shape[1],))


def wan_mlp_gated_residual(hidden_states: torch.Tensor, norm_h: torch.Tensor, up_weight, down_weight, up_bias, down_bias,
                           c_gate_msa: torch.Tensor | None) -> torch.Tensor:
    """The block's closing step (wan2_2_transformer.py:1510-1512):
    ``(hidden_states.float() + ffn(norm_h).float() * c_gate_msa).type_as(hidden_states)``, with the residual
    fused into the down projection's epilogue. ``c_gate_msa``: ``[B, 1, H]`` (per batch element) or ``[H]``."""
    B, T, H = hidden_states.shape
    x2 = norm_h.reshape(-1, norm_h.shape[-1]).contiguous()
    up = _gemm(x2, up_weight.contiguous(), up_bias, 1)
    res = hidden_states.reshape(B * T, H).contiguous()
    gate, rows = None, 0
    if c_gate_msa is not None:
        g = c_gate_msa.float()
        if g.numel() == H:
            gate, rows = g.reshape(1, H).contiguous(), B * T
        elif g.numel() == B * H:
            gate, rows = g.reshape(B, H).contiguous(), T
        else:
            raise ValueError(f"c_gate_msa must be [H] or [B, 1, H], got {tuple(c_gate_msa.shape)}")
    out = _gemm(up, down_weight.contiguous(), down_bias, 0, res, gate, rows)
    return out.reshape(B, T, H)
