"""Wan FFN on B200: the reference's ``_wan_mlp(hidden, up_weight, down_weight, up_bias, down_bias)``
(vllm_omni_neuron/diffusion/models/wan2_2/wan2_2_transformer.py:389-410):
``GELU_tanh(hidden @ up_weight + up_bias) @ down_weight + down_bias`` with torch's bf16 rounding
after each matmul and bias add, the GELU in fp32 opmath. Two CTA-pair tcgen05 GEMMs; the first
applies the bias and GELU-tanh in its epilogue, so the ``[T, I]`` intermediate is written once, bf16.

The FP8 leaf ``row_mx_mlp`` (diffusion/quantization/row_mx_kernels.py:141-198; the nkilib MLP in
ROW_MX CTE mode, arithmetic in kernels/nkilib/core/mlp/mlp_torch.py:401-600) consumes the ROW-quantised
adaLN output: an e4m3 ROW GEMM whose epilogue applies the row and channel scales, the bias and
GELU-tanh and MX-32-quantises the result (codes plus UE8M0 scales already in the tcgen05 scale-atom
layout), then a block-scaled MX GEMM with the down weight's per-channel scale, bias and the block's
gated residual in its epilogue. The ``[T, I]`` intermediate crosses HBM once, as 1-byte codes.
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


# ---------------------------------------------------------------- FP8 (ROW_MX) leaf

_IDENTITY_SF = {}


def _identity_block_scales(rows: int, k: int, device) -> torch.Tensor:
    """Packed UE8M0 block scales that are all 1.0 (byte 127) for a ``[rows, k]`` weight; the layout
    does not matter when every byte is equal. Cached per shape and device."""
    key = (rows, k, str(device))
    t = _IDENTITY_SF.get(key)
    if t is None:
        n = _lib.load().vomni_mx_packed_scales_bytes(rows, k)
        if n == 0:
            raise ValueError(f"MX-32 block scales need k % 128 == 0, got k = {k}")
        t = torch.full((n,), 127, dtype=torch.uint8, device=device)
        _IDENTITY_SF[key] = t
    return t


def quantize_mlp_weights_row_mx(up_weight: torch.Tensor, down_weight: torch.Tensor):
    """Per-tensor e4m3fn quantisation of the FFN weights, one scale per tensor expanded per output
    channel (the ComfyUI checkpoint scalars, ``expanded_scalar_scale_loader`` in
    diffusion/quantization/row_mx_loaders.py). ``up_weight [H, I]``, ``down_weight [I, H]`` (the
    ``x @ W`` layout). Returns ``(up_codes [I, H], up_scale [I], down_codes [H, I], down_scale [H])``:
    codes are W^T (K-major), float8_e4m3fn."""
    out = []
    for w in (up_weight, down_weight):
        wf = w.float()
        sc = torch.clamp(wf.abs().amax() / 448.0, min=1e-12)
        codes = (wf / sc).t().contiguous().to(torch.float8_e4m3fn)
        out += [codes, torch.full((wf.shape[1],), float(sc), dtype=torch.float32, device=w.device)]
    return tuple(out)


def _split_row_packed(packed_hidden):
    """Packed ROW rows ``[..., H + 4]`` (codes then the fp32 scale) or a ``(codes, scale)`` pair ->
    ``(codes [T, H] e4m3, row_scale [T] fp32, lead shape)``."""
    L = _lib.load()
    if isinstance(packed_hidden, (tuple, list)):
        codes, row_scale = packed_hidden
        lead = tuple(codes.shape[:-1])
        H = codes.shape[-1]
        return codes.reshape(-1, H).contiguous(), row_scale.reshape(-1).float().contiguous(), lead
    lead = tuple(packed_hidden.shape[:-1])
    H = packed_hidden.shape[-1] - 4
    dev = packed_hidden.device
    T = packed_hidden.numel() // (H + 4)
    codes = torch.empty(T, H, dtype=torch.float8_e4m3fn, device=dev)
    row_scale = torch.empty(T, dtype=torch.float32, device=dev)
    _lib.check(L.vomni_qkv_unpack_rows(packed_hidden.contiguous().data_ptr(), T, H, codes.data_ptr(),
                                       row_scale.data_ptr(), torch.cuda.current_stream(dev).cuda_stream),
               "vomni_qkv_unpack_rows")
    return codes, row_scale, lead


def row_mx_mlp(packed_hidden, up_weight: torch.Tensor, down_weight: torch.Tensor, up_w_scale: torch.Tensor,
               down_w_scale: torch.Tensor, up_bias, down_bias, *, residual: torch.Tensor | None = None,
               gate: torch.Tensor | None = None) -> torch.Tensor:
    """The reference's ``row_mx_mlp(packed_hidden, up_weight, down_weight, up_w_scale, down_w_scale,
    up_bias, down_bias)`` (row_mx_kernels.py:141-198) -> ``[..., H]`` bf16.

    ``packed_hidden``: the ``adaln_modulate(quant="row")`` output, packed ``[..., H + 4]`` or split
    ``(codes, scale)``. Weights in this library's layout (``quantize_mlp_weights_row_mx``):
    ``up_weight [I, H]`` / ``down_weight [H, I]`` float8_e4m3fn codes (W^T), ``up_w_scale [I]`` /
    ``down_w_scale [H]`` fp32 per-channel scales, biases bf16 ``[I]`` / ``[H]`` (or None).
    With ``residual`` ``[..., H]`` bf16 the result is the block's closing gated residual
    ``bf16(residual + gate * mlp)`` (wan2_2_transformer.py:1510-1512); ``gate`` fp32 ``[H]`` or
    ``[B, 1, H]`` (per batch element of ``residual [B, T, H]``), None = 1.
    """
    codes, row_scale, lead = _split_row_packed(packed_hidden)
    T, H = codes.shape
    dev = codes.device
    if not codes.is_cuda:
        raise RuntimeError("row_mx_mlp needs CUDA tensors (the B200 kernels have no CPU path)")
    I = up_weight.shape[0]
    if up_weight.shape != (I, H) or down_weight.shape != (H, I):
        raise ValueError(f"weights must be up [I, H] and down [H, I] codes; got {tuple(up_weight.shape)}, "
                         f"{tuple(down_weight.shape)} for H = {H}")
    for name, t in (("up_weight", up_weight), ("down_weight", down_weight)):
        if t.dtype != torch.float8_e4m3fn:
            raise TypeError(f"{name} must be float8_e4m3fn codes, got {t.dtype}")
    L = _lib.load()
    st = torch.cuda.current_stream(dev).cuda_stream
    ub = up_bias.reshape(-1).to(torch.bfloat16).contiguous() if up_bias is not None else None
    db = down_bias.reshape(-1).to(torch.bfloat16).contiguous() if down_bias is not None else None
    us = up_w_scale.reshape(-1).float().contiguous()
    ds = down_w_scale.reshape(-1).float().contiguous()
    inter = torch.empty(T, I, dtype=torch.float8_e4m3fn, device=dev)
    inter_sf = torch.empty(L.vomni_mx_packed_scales_bytes(T, I), dtype=torch.uint8, device=dev)
    _lib.check(L.vomni_ffn_fp8_up(codes.data_ptr(), row_scale.data_ptr(), up_weight.contiguous().data_ptr(), us.data_ptr(),
                                  ub.data_ptr() if ub is not None else None, T, H, I, inter.data_ptr(),
                                  inter_sf.data_ptr(), st), "vomni_ffn_fp8_up")
    res, g, rows = None, None, 1
    if residual is not None:
        res = residual.reshape(T, H).to(torch.bfloat16).contiguous()
        if gate is not None:
            gf = gate.float()
            if gf.numel() == H:
                g, rows = gf.reshape(1, H).contiguous(), T
            elif residual.dim() == 3 and gf.numel() == residual.shape[0] * H:
                g, rows = gf.reshape(residual.shape[0], H).contiguous(), residual.shape[1]
            else:
                raise ValueError(f"gate must be [H] or [B, 1, H], got {tuple(gate.shape)}")
    elif gate is not None:
        raise ValueError("gate requires residual")
    out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    _lib.check(L.vomni_ffn_fp8_down(inter.data_ptr(), inter_sf.data_ptr(), down_weight.contiguous().data_ptr(),
                                    _identity_block_scales(H, I, dev).data_ptr(), ds.data_ptr(),
                                    db.data_ptr() if db is not None else None, T, I, H,
                                    res.data_ptr() if res is not None else None, g.data_ptr() if g is not None else None,
                                    rows, out.data_ptr(), st), "vomni_ffn_fp8_down")
    return out.reshape(lead + (H,))
