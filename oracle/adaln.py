"""CPU restatements of the fused adaLN (+ FP8 row / MX quant) semantics (numpy).

* ``adaln_quant_ref`` restates the reference's ground truth ``adaln_quant_torch_ref``
  (vllm_omni_neuron/kernels/nkilib/experimental/norm/adaln_quant_torch.py:41-148) and
  its MX round trip ``_mx_dequant`` (:151-175). It is pinned bit-exactly against outputs of
  that function (tests/golden/adaln_ref.npz).
* ``adaln_modulate_oracle`` restates the bridge contract ``adaln_modulate``
  (vllm_omni_neuron/diffusion/quantization/adaln_kernels.py:87-201): mul/add cast to the
  hidden dtype (bf16, :146-150), gate kept fp32 (:167), the gated residual sum rounded to
  bf16 before it is normalised and returned as ``residual_out`` (_eager_adaln :57-66,
  adaln_quant.py:568-608), and the ROW output packed as ``[..., H + 4]`` fp8 bytes with the
  fp32 dequant scale in the 4 tail bytes (adaln_quant.py:540-565).
"""

from __future__ import annotations

import numpy as np

from .numerics import FP8_E4M3_MAX, FP8_E4M3FN_MAX, bf16_round, e4m3fn_bits, e4m3fn_round

MIN_DEQUANT_SCALE = 1e-6  # adaln_quant_torch.py:29
MX_BLOCK = 32  # adaln_quant_torch.py:31
FP8_E4M3_MAX_EXP = 7  # adaln_quant_torch.py:30


def _normalize(x: np.ndarray, norm_type: str, eps: float) -> np.ndarray:
    if norm_type == "layer_norm":  # adaln_quant_torch.py:104-107
        mean = x.mean(axis=-1, keepdims=True)
        var = np.mean(np.square(x - mean), axis=-1, keepdims=True)
        return (x - mean) / np.sqrt(var + eps)
    if norm_type == "rms_norm":  # :108-110
        rms = np.sqrt(np.mean(np.square(x), axis=-1, keepdims=True) + eps)
        return x / rms
    if norm_type == "none":  # :111-112
        return x
    raise ValueError(f"unsupported norm_type {norm_type!r}")


def row_quantize(y: np.ndarray, ocp: bool = True, lower_bound: float = 0.0, reciprocal: bool = False):
    """Per-row FP8 quant, adaln_quant_torch.py:133-145: scale = max(amax/range, 1e-6),
    codes = e4m3fn(y / scale) — or, with ``reciprocal``, e4m3fn(y * (1/scale)) in fp32 as the NKI
    kernel computes it (adaln_quant.py:520-536). Returns (codes fp32-valued, dequant_scale [...,1] fp32)."""
    fp8_range = FP8_E4M3FN_MAX if ocp else FP8_E4M3_MAX
    yq = y
    amax = np.abs(yq).max(axis=-1, keepdims=True)
    if lower_bound > 0:
        amax = np.clip(amax, a_min=None, a_max=lower_bound)
        yq = np.clip(yq, a_min=-lower_bound, a_max=lower_bound)
    dequant_scale = np.maximum(amax / fp8_range, MIN_DEQUANT_SCALE)
    if reciprocal:
        inv = (np.float32(1.0) / dequant_scale.astype(np.float32)).astype(np.float32)
        codes = e4m3fn_round((yq.astype(np.float32) * inv).astype(np.float32))
    else:
        codes = e4m3fn_round(yq / dequant_scale)
    return codes, dequant_scale.astype(np.float32)


def mx_quantize(y: np.ndarray, block: int = MX_BLOCK):
    """MX micro-block quant, adaln_quant_torch.py:151-175: one UE8M0 scale per ``block``
    contiguous values = block's max biased fp32 exponent - 7 (clipped to [0, 255]);
    codes = e4m3fn(clip(y / 2^(scale-127), +-448)).

    Returns (codes float32-valued [..., H], scale_u8 [..., H//block] uint8, dequant [..., H]).
    """
    shape = y.shape
    H = shape[-1]
    if H % block != 0:
        raise ValueError(f"MX hidden dim {H} must be a multiple of block size {block}")
    flat = np.ascontiguousarray(y.reshape(-1, H).astype(np.float32))
    T = flat.shape[0]
    blocks = flat.reshape(T, H // block, block)
    exp_field = (blocks.view(np.uint32) >> 23) & 0xFF
    block_max_exp = exp_field.max(axis=2, keepdims=True).astype(np.int64)
    scale_u8 = np.clip(block_max_exp - FP8_E4M3_MAX_EXP, 0, 255)
    factor = np.power(2.0, scale_u8.astype(np.float64) - 127.0)
    safe_factor = np.where(factor == 0, 1.0, factor)
    codes = e4m3fn_round(np.clip(blocks / safe_factor, -FP8_E4M3FN_MAX, FP8_E4M3FN_MAX).astype(np.float32))
    deq = (codes.astype(np.float64) * factor).astype(np.float32)
    return (
        codes.reshape(shape),
        scale_u8.reshape(shape[:-1] + (H // block,)).astype(np.uint8),
        deq.reshape(shape),
    )


def adaln_quant_ref(
    hidden,
    mul=None,
    add=None,
    *,
    norm_type="layer_norm",
    quant="none",
    eps=1e-6,
    lower_bound=0.0,
    ocp=True,
    residual=None,
    gate=None,
):
    """Restatement of adaln_quant_torch_ref (adaln_quant_torch.py:41-148), numpy fp32."""
    x = np.asarray(hidden, np.float32)
    residual_out = None
    if residual is not None:  # :94-101
        gated = x
        if gate is not None:
            gated = gated * np.asarray(gate, np.float32)
        x = np.asarray(residual, np.float32) + gated
        residual_out = x
    xhat = _normalize(x, norm_type, eps)
    y = xhat
    if mul is not None:  # :119-122
        y = y * np.asarray(mul, np.float32)
    if add is not None:
        y = y + np.asarray(add, np.float32)
    res = {"y": y.astype(np.float32), "quant": None, "dequant_scale": None, "dequant": None, "residual_out": residual_out}
    if quant == "none":
        return res
    if quant == "row":
        codes, scale = row_quantize(y, ocp=ocp, lower_bound=lower_bound)
        res["quant"] = codes
        res["dequant_scale"] = scale
        res["dequant"] = (codes * scale).astype(np.float32)
        return res
    if quant == "mx":
        res["dequant"] = mx_quantize(y)[2]
        return res
    raise ValueError(f"unsupported quant {quant!r}")


def pack_row(codes: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """[..., H] codes + [..., 1] fp32 scale -> [..., H + 4] uint8 (adaln_quant.py:540-565)."""
    bits = e4m3fn_bits(codes)
    sc = np.ascontiguousarray(scale.astype(np.float32)).view(np.uint8).reshape(scale.shape[:-1] + (4,))
    return np.concatenate([bits, sc], axis=-1)


def adaln_modulate_oracle(
    hidden,
    mul=None,
    add=None,
    *,
    eps,
    norm_type="layer_norm",
    quant="none",
    ocp=True,
    residual=None,
    gate=None,
):
    """The bridge contract (adaln_kernels.py:87-201) with the kernel's rounding points.

    Returns ``out`` (bf16-valued float32 for quant="none"; uint8 ``[..., H+4]`` for "row";
    for "mx32": a tuple (codes uint8 [...,H], scales uint8 [...,H/32])), or
    ``(residual_out, out)`` when ``residual`` is given.
    """
    x = np.asarray(hidden, np.float32)
    mul_b = None if mul is None else bf16_round(np.asarray(mul, np.float32))
    add_b = None if add is None else bf16_round(np.asarray(add, np.float32))
    residual_out = None
    if residual is not None:
        g = x if gate is None else x * np.asarray(gate, np.float32)
        residual_out = bf16_round(np.asarray(residual, np.float32) + g)
        x = residual_out
    xhat = _normalize(x, norm_type, eps)
    y = xhat
    if mul_b is not None:
        y = y * mul_b
    if add_b is not None:
        y = y + add_b
    y = y.astype(np.float32)
    if quant == "none":
        out = bf16_round(y)
    elif quant == "row":
        codes, scale = row_quantize(y, ocp=ocp, reciprocal=True)
        out = pack_row(codes, scale)
    elif quant == "mx32":
        codes, scale_u8, _ = mx_quantize(y)
        out = (e4m3fn_bits(codes), scale_u8)
    else:
        raise ValueError(f"unsupported quant {quant!r}")
    return (residual_out, out) if residual is not None else out


def adaln_bytes(t: int, h: int, quant: str, residual: bool) -> int:
    """Algorithmic HBM bytes of one call: bf16 read of hidden (+ residual, + residual_out write),
    output write (bf16, or H+4 fp8 bytes per row for ROW)."""
    rd = 2 * t * h * (2 if residual else 1)
    wr = (t * (h + 4) if quant == "row" else 2 * t * h) + (2 * t * h if residual else 0)
    return rd + wr
