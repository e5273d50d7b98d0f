"""Output projection of the Wan self-attention and the block's norm2, on B200.

* :func:`wan_o_proj` keeps the reference's ``_wan_o_proj(active, weight, bias)``
  (vllm_omni_neuron/diffusion/models/wan2_2/wan2_2_transformer.py:246-254): the d-major attention
  output ``[B, N, D, S]`` straight from ``wan_cp_self_attention``, ``weight [N*D, H]``,
  ``bias [1, H]`` -> ``[B, S, H]`` bf16. The kernel reads the d-major tensor in place (no transpose).
* :func:`attn_out_norm2` is the block step after the self-attention (:1466-1489): the projection
  with the gated residual ``hidden_states + gate_msa * attn1_out`` fused into its epilogue, then
  the norm2 adaLN (affine LayerNorm, or none) with the quantisation the next leaf wants. Returns
  ``(hidden_states, norm_h)`` as the reference's ``adaln_modulate(..., residual=, gate=)`` does.
* :func:`row_mx_o_proj` keeps the reference's FP8 o-projection ``row_mx_o_proj(attention, weight,
  weight_scales, bias)`` (vllm_omni_neuron/diffusion/quantization/row_mx_kernels.py:114-138): the
  d-major bf16 attention is ROW-quantised per token (``vomni_oproj_rowquant``) and projected by the
  FP8 ROW GEMM (``vomni_qkv_fp8_gemm``): ``y = bf16((Xq @ Wq^T) * row_scale * w_scale + bias)``.
"""

from __future__ import annotations

import torch

from . import _lib


def _prep(active: torch.Tensor, weight: torch.Tensor, bias):
    if active.dim() != 4:
        raise ValueError(f"active must be d-major [B, N, D, S], got {tuple(active.shape)}")
    B, N, D, S = active.shape
    K, H = weight.shape
    if N * D != K:
        raise ValueError(f"weight rows {K} != N*D = {N * D}")
    for name, t in (("active", active), ("weight", weight)):
        if t.dtype != torch.bfloat16:
            raise TypeError(f"{name} must be bfloat16, got {t.dtype}")
        if not t.is_cuda:
            raise RuntimeError(f"{name} must be a CUDA tensor (the B200 kernel has no CPU path)")
    s_pad = -(-S // 8) * 8  # the kernel wants 16-byte token rows in the d-major input
    act = active.contiguous()
    if s_pad != S:
        act = torch.nn.functional.pad(act, (0, s_pad - S))
    b = bias.reshape(-1).to(torch.bfloat16).contiguous() if bias is not None else None
    if b is not None and b.numel() != H:
        raise ValueError(f"bias has {b.numel()} values for {H} columns")
    return act, weight.contiguous(), b, B, K, S, s_pad, H


def _run(act, w, b, B, K, s_pad, H, residual, gate, gate_per_batch, out):
    st = torch.cuda.current_stream(act.device).cuda_stream
    ptr = lambda t: t.data_ptr() if t is not None else None
    _lib.check(
        _lib.load().vomni_oproj_gemm(act.data_ptr(), B, K, s_pad, w.data_ptr(), ptr(b), H, ptr(residual), ptr(gate),
                                     int(gate_per_batch), out.data_ptr(), st),
        "vomni_oproj_gemm",
    )


def wan_o_proj(active: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None) -> torch.Tensor:
    """``[B, N, D, S]`` d-major attention @ ``[N*D, H]`` + bias -> ``[B, S, H]`` bf16."""
    act, w, b, B, K, S, s_pad, H = _prep(active, weight, bias)
    out = torch.empty(B, s_pad, H, dtype=torch.bfloat16, device=act.device)
    _run(act, w, b, B, K, s_pad, H, None, None, 0, out)
    return out if s_pad == S else out[:, :S].contiguous()


def _gate_rows(gate: torch.Tensor | None, B: int, H: int):
    if gate is None:
        return None, 0
    g = gate.float()
    if g.numel() == H:
        return g.reshape(H).contiguous(), 0
    if g.numel() == B * H:  # [B, 1, H] per batch element (the block's gate_msa)
        return g.reshape(B, H).contiguous(), 1
    raise ValueError(f"gate must be [H], [1, H] or [B, 1, H]; got {tuple(gate.shape)}")


def o_proj_gated_residual(active, weight, bias, residual: torch.Tensor, gate: torch.Tensor | None) -> torch.Tensor:
    """``bf16(residual + gate * wan_o_proj(active, weight, bias))`` in one kernel -> ``[B, S, H]``."""
    act, w, b, B, K, S, s_pad, H = _prep(active, weight, bias)
    if tuple(residual.shape) != (B, S, H) or residual.dtype != torch.bfloat16:
        raise ValueError(f"residual must be bf16 [B, S, H] = {(B, S, H)}, got {tuple(residual.shape)} {residual.dtype}")
    res = residual.contiguous()
    if s_pad != S:
        res = torch.nn.functional.pad(res, (0, 0, 0, s_pad - S))
    g, per_batch = _gate_rows(gate, B, H)
    out = torch.empty(B, s_pad, H, dtype=torch.bfloat16, device=act.device)
    _run(act, w, b, B, K, s_pad, H, res, g, per_batch, out)
    return out if s_pad == S else out[:, :S].contiguous()


def attn_out_norm2(
    attention: torch.Tensor,
    o_proj_weight: torch.Tensor,
    o_proj_bias: torch.Tensor | None,
    hidden_states: torch.Tensor,
    gate_msa: torch.Tensor | None,
    norm2_weight: torch.Tensor | None = None,
    norm2_bias: torch.Tensor | None = None,
    *,
    eps: float = 1e-6,
    norm_type: str = "layer_norm",
    quant: str = "none",
):
    """(hidden_states, norm_h) after the self-attention of a Wan block (wan2_2_transformer.py:1466-1489)."""
    from .adaln import adaln_modulate

    t = o_proj_gated_residual(attention, o_proj_weight, o_proj_bias, hidden_states, gate_msa)
    norm_h = adaln_modulate(t, norm2_weight, norm2_bias, eps=eps, norm_type=norm_type, quant=quant)
    return t, norm_h


def row_mx_o_proj(attention: torch.Tensor, weight: torch.Tensor, weight_scales: torch.Tensor,
                  bias: torch.Tensor | None) -> torch.Tensor:
    """FP8 o-projection of the d-major ``[B, N, D, S]`` bf16 attention -> ``[B, S, H]`` bf16.

    ``weight``: the reference's ``[N*D//4, H, 4]`` FP8 pack (row_mx_modules.py:243-250) or this
    build's ``[H, N*D]`` K-major codes (``quantize_qkv_weight(w, H, 0)``). ``weight_scales``: the
    per-channel weight scale, ``[128, H]`` (the reference's expanded scalar), ``[1, H]`` or ``[H]``.
    The reference's kernel (nkilib ``output_projection_cte``) is not in its source tree, so the
    activation quantisation follows its in-tree ROW rule (adaln_quant.py:520-536)."""
    from .qkv import repack_mx_contiguous

    if attention.dim() != 4 or attention.dtype != torch.bfloat16:
        raise ValueError(f"attention must be d-major bf16 [B, N, D, S], got {tuple(attention.shape)} {attention.dtype}")
    if not attention.is_cuda:
        raise RuntimeError("attention must be a CUDA tensor (the B200 kernel has no CPU path)")
    B, N, D, S = attention.shape
    K = N * D
    if weight.dim() == 3:
        weight = repack_mx_contiguous(weight)
    H = weight.shape[0]
    if weight.shape[1] != K:
        raise ValueError(f"weight contraction {weight.shape[1]} != N*D = {K}")
    chan = weight_scales.reshape(-1, H)[0].float().contiguous()
    b = bias.reshape(-1).to(torch.bfloat16).contiguous() if bias is not None else None
    s_pad = -(-S // 8) * 8
    act = attention.contiguous()
    if s_pad != S:
        act = torch.nn.functional.pad(act, (0, s_pad - S))
    dev = act.device
    T = B * s_pad
    codes = torch.empty(T, K, dtype=torch.float8_e4m3fn, device=dev)
    scales = torch.empty(T, dtype=torch.float32, device=dev)
    st = torch.cuda.current_stream(dev).cuda_stream
    L = _lib.load()
    _lib.check(L.vomni_oproj_rowquant(act.data_ptr(), B, K, s_pad, codes.data_ptr(), scales.data_ptr(), st),
               "vomni_oproj_rowquant")
    y = torch.empty(B, s_pad, H, dtype=torch.bfloat16, device=dev)
    _lib.check(
        L.vomni_qkv_fp8_gemm(codes.data_ptr(), scales.data_ptr(), weight.contiguous().data_ptr(), chan.data_ptr(),
                             b.data_ptr() if b is not None else None, T, K, H, H, 0, y.data_ptr(), None, st),
        "vomni_qkv_fp8_gemm",
    )
    return y if s_pad == S else y[:, :S].contiguous()
