"""Fused adaptive-LayerNorm (+ FP8 row / MX quantisation) — the reference's ``adaln_modulate``.

Same signature and contract as ``adaln_modulate``
(vllm_omni_neuron/diffusion/quantization/adaln_kernels.py:87-201):

    Quantize(Norm(residual + gate * hidden) * mul + add)

* ``hidden``: ``[B, S, H]`` or ``[T, H]`` bf16 (H <= 16384, H % 8 == 0).
* ``mul`` / ``add``: ``[B, 1, H]`` (per-batch AdaLN ``1 + scale`` / ``shift``), ``[H]`` / ``[1, H]``
  (shared affine), or None; used in the hidden dtype (bf16) as the bridge does (:146-150).
* ``gate``: same layouts, kept fp32 (:167); requires ``residual`` (adaln_quant.py:277-281).
* ``quant="none"`` returns bf16; ``quant="row"`` returns the packed ``[..., H + 4]`` FP8 tensor whose
  last 4 bytes per row are the fp32 dequant scale (adaln_quant.py:540-565); ``quant="mx"`` raises
  ``NotImplementedError`` exactly as the reference (:36-40).
* With ``residual``, returns ``(residual_out, out)``; ``residual_out`` is the bf16
  ``residual + gate * hidden``.

B200 additions (keyword-only): ``row_layout="split"`` returns ``(codes [..., H] fp8, scales [...] fp32)``
instead of the packed rows — the 16-byte-aligned layout the FP8 QKV GEMM loads with TMA — and
``quant="mx32"`` returns ``(codes [..., H] fp8, scales [..., H/32] uint8 UE8M0)``, the MX-32 format of
``_mx_dequant`` (adaln_quant_torch.py:151-175).
"""

from __future__ import annotations

import torch

from . import _lib

_MAX_HIDDEN = 16384
_NORMS = {"layer_norm": 0, "rms_norm": 1, "none": 2}
_QUANTS = {"none": 0, "row": 1, "mx32": 2}


def _mod_rows(vec, batch: int, hidden_dim: int, dtype):
    """[B,1,H] -> [B,H] (per batch), [H]/[1,H] -> [1,H] (shared); cast to dtype, contiguous."""
    if vec is None:
        return None, False
    if vec.dim() == 3:
        if vec.shape[0] != batch or vec.shape[1] != 1:
            raise ValueError(f"per-batch modulation must be [B, 1, H], got {tuple(vec.shape)}")
        return vec.reshape(batch, hidden_dim).to(dtype).contiguous(), True
    if vec.numel() != hidden_dim:
        raise ValueError(f"modulation vector length must equal {hidden_dim}, got {tuple(vec.shape)}")
    return vec.reshape(1, hidden_dim).to(dtype).contiguous(), False


def adaln_modulate(
    hidden: torch.Tensor,
    mul: torch.Tensor | None = None,
    add: torch.Tensor | None = None,
    *,
    eps: float,
    norm_type: str = "layer_norm",
    quant: str = "none",
    ocp: bool = True,
    residual: torch.Tensor | None = None,
    gate: torch.Tensor | None = None,
    row_layout: str = "packed",
):
    if quant == "mx":
        raise NotImplementedError(
            "MX activation quantization has no fused path with the reference's packed layout; use quant='row', "
            "'none', or the B200 MX-32 format quant='mx32'."
        )
    if quant not in _QUANTS:
        raise ValueError(f"unsupported quant {quant!r}")
    if norm_type not in _NORMS:
        raise ValueError(f"unsupported norm_type {norm_type!r}")
    if hidden.dim() < 2:
        raise ValueError("hidden must have at least 2 dims")
    H = hidden.shape[-1]
    if H > _MAX_HIDDEN or H % 8:
        raise ValueError(f"hidden dim {H} unsupported (needs H <= {_MAX_HIDDEN} and H % 8 == 0)")
    if hidden.dtype != torch.bfloat16:
        raise TypeError(f"hidden must be bfloat16, got {hidden.dtype}")
    if not hidden.is_cuda:
        raise RuntimeError("hidden must be a CUDA tensor (the B200 kernel has no CPU path)")
    if gate is not None and residual is None:
        raise ValueError("gate requires residual (gate scales the sub-layer output before the residual add)")
    if row_layout not in ("packed", "split"):
        raise ValueError(f"unknown row_layout {row_layout!r}")
    dev = hidden.device
    lead = hidden.shape[:-1]
    batch = hidden.shape[0] if hidden.dim() == 3 else 1
    rows = hidden.numel() // H
    x = hidden.contiguous()
    mul_r, per_b1 = _mod_rows(mul, batch, H, torch.bfloat16)
    add_r, per_b2 = _mod_rows(add, batch, H, torch.bfloat16)
    gate_r, per_b3 = _mod_rows(gate, batch, H, torch.float32)
    per_batch = per_b1 or per_b2 or per_b3
    if per_batch:  # expand shared vectors so every modulation tensor has one row per batch element
        mul_r = mul_r.expand(batch, H).contiguous() if mul_r is not None else None
        add_r = add_r.expand(batch, H).contiguous() if add_r is not None else None
        gate_r = gate_r.expand(batch, H).contiguous() if gate_r is not None else None
    rows_per_mod = rows // batch if per_batch else rows
    res = None
    res_out = None
    if residual is not None:
        if tuple(residual.shape) != tuple(hidden.shape):
            raise ValueError(f"residual shape {tuple(residual.shape)} must match hidden shape {tuple(hidden.shape)}")
        res = residual.to(torch.bfloat16).contiguous()
        res_out = torch.empty_like(res)
    q = _QUANTS[quant]
    packed = 1 if (quant == "row" and row_layout == "packed") else 0
    scales = None
    if quant == "none":
        out = torch.empty(lead + (H,), dtype=torch.bfloat16, device=dev)
    elif quant == "row":
        if packed:
            out = torch.empty(lead + (H + 4,), dtype=torch.float8_e4m3fn, device=dev)
        else:
            out = torch.empty(lead + (H,), dtype=torch.float8_e4m3fn, device=dev)
            scales = torch.empty(lead, dtype=torch.float32, device=dev)
    else:
        if H % 32:
            raise ValueError(f"MX hidden dim {H} must be a multiple of 32")
        out = torch.empty(lead + (H,), dtype=torch.float8_e4m3fn, device=dev)
        scales = torch.empty(lead + (H // 32,), dtype=torch.uint8, device=dev)
    ptr = lambda t: t.data_ptr() if t is not None else None
    rc = _lib.load().vomni_adaln_modulate(
        x.data_ptr(), ptr(res), ptr(mul_r), ptr(add_r), ptr(gate_r), rows, H, rows_per_mod, float(eps),
        _NORMS[norm_type], q, int(bool(ocp)), packed, out.data_ptr(), ptr(scales), ptr(res_out),
        torch.cuda.current_stream(dev).cuda_stream,
    )
    _lib.check(rc, "vomni_adaln_modulate")
    result = out if scales is None else (out, scales)
    return (res_out, result) if residual is not None else result
