"""ComfyUI FP8-scaled Wan2.2 checkpoints -> the B200 block's weight layouts.

The checkpoint format (``Comfy-Org/Wan_2.2_ComfyUI_Repackaged``, as documented in the reference's
vllm_omni_neuron/diffusion/quantization/comfy_fp8_checkpoint.py:1-31): each quantized linear stores
``<prefix>.weight`` F8_E4M3 ``[out, in]`` (per-tensor absmax), ``<prefix>.scale_weight`` F32 scalar
(dequant scale), ``<prefix>.scale_input`` (unused) and ``<prefix>.bias`` F16 ``[out]``; names are native
Wan (``self_attn.{q,k,v,o}``, ``cross_attn.*``, ``ffn.{0,2}``, ``norm3`` = the model's norm2,
``modulation`` = ``scale_shift_table``).

* :func:`read_safetensors_header` / :func:`load_tensors`: the safetensors container (8-byte header
  length, JSON header, raw little-endian data), read without extra dependencies.
* :func:`block_key_map` / :func:`validate_fp8_checkpoint`: the model-parameter -> checkpoint-key table
  of ``build_fp8_dequant_mappings`` (:158-229) and its validation rules (:287-321).
* :func:`dequantize_to_bf16`: ``(fp8.float() * scale).bfloat16()`` (dequant_loaders.py:38-52), in the
  checkpoint's ``[out, in]`` orientation, transposed afterwards to the model's ``[in, out]``.
* :func:`block_weights_bf16`: one block as the reference parameter dict for :func:`prepare_block_weights`
  (dequantised, fused Q|K|V in q, k, v order with per-source scales, dequant_loaders.py:118-140).
* :func:`fp8_qkv_leaf`: the FP8 self-attention leaf's operands without any dequant: codes ``[I, H]``
  (the checkpoint's ``[out, in]`` is already the tcgen05 K-major B layout), Q/K rows de-interleaved per
  head, the three checkpoint scalars expanded per channel (row_mx_loaders.py:112-139, 228-260).
"""

from __future__ import annotations

import json
import struct
from pathlib import Path

import numpy as np
import torch

from .rope import deinterleave_gamma_row, deinterleave_qk_columns

FP8_DTYPE_STR = "F8_E4M3"
_DTYPES = {
    "F8_E4M3": (np.uint8, torch.float8_e4m3fn),
    "F32": (np.float32, torch.float32),
    "F16": (np.float16, torch.float16),
    "BF16": (np.uint16, torch.bfloat16),
    "F64": (np.float64, torch.float64),
    "I64": (np.int64, torch.int64),
}


class Fp8CheckpointError(RuntimeError):
    """A checkpoint does not satisfy the FP8 loaders' contract."""


def read_safetensors_header(path) -> dict:
    """``{name: {"dtype", "shape", "data_offsets"}}`` (``__metadata__`` dropped)."""
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(n))
    header.pop("__metadata__", None)
    return header


def load_tensors(path, names=None) -> dict:
    """CPU tensors for ``names`` (all when None), memory-mapped from the file."""
    path = Path(path)
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(n))
    header.pop("__metadata__", None)
    base = 8 + n
    raw = np.memmap(path, dtype=np.uint8, mode="r")
    out = {}
    for name in (names if names is not None else header):
        meta = header[name]
        if meta["dtype"] not in _DTYPES:
            raise Fp8CheckpointError(f"{name}: unsupported dtype {meta['dtype']}")
        np_t, torch_t = _DTYPES[meta["dtype"]]
        a, b = meta["data_offsets"]
        buf = np.array(raw[base + a: base + b])  # copy out of the map
        arr = buf.view(np_t).reshape(meta["shape"])
        t = torch.from_numpy(arr.copy())
        if torch_t in (torch.float8_e4m3fn, torch.bfloat16):
            t = t.view(torch_t)
        out[name] = t
    return out


def block_key_map(i: int) -> dict:
    """Model parameter -> checkpoint key(s) of block ``i`` (quantized weights map to ``[weight, scale]``;
    the fused self-attention QKV to ``[qW, qS, kW, kS, vW, vS]``)."""
    b = f"blocks.{i}"
    m = {
        f"{b}.attn1.qkv_proj_weight": [f"{b}.self_attn.{p}.{k}" for p in ("q", "k", "v") for k in ("weight", "scale_weight")],
        f"{b}.attn1.qkv_proj_bias": [f"{b}.self_attn.{p}.bias" for p in ("q", "k", "v")],
        f"{b}.attn1.o_proj_weight": [f"{b}.self_attn.o.weight", f"{b}.self_attn.o.scale_weight"],
        f"{b}.attn1.o_proj_bias": f"{b}.self_attn.o.bias",
        f"{b}.attn1.norm_q.weight": f"{b}.self_attn.norm_q.weight",
        f"{b}.attn1.norm_k.weight": f"{b}.self_attn.norm_k.weight",
    }
    for p in ("q", "k", "v"):
        m[f"{b}.attn2.{p}_proj_weight"] = [f"{b}.cross_attn.{p}.weight", f"{b}.cross_attn.{p}.scale_weight"]
        m[f"{b}.attn2.{p}_proj_bias"] = f"{b}.cross_attn.{p}.bias"
    m[f"{b}.attn2.norm_q.weight"] = f"{b}.cross_attn.norm_q.weight"
    m[f"{b}.attn2.norm_k.weight"] = f"{b}.cross_attn.norm_k.weight"
    m[f"{b}.attn2.o_proj_weight"] = [f"{b}.cross_attn.o.weight", f"{b}.cross_attn.o.scale_weight"]
    m[f"{b}.attn2.o_proj_bias"] = f"{b}.cross_attn.o.bias"
    m[f"{b}.norm2.weight"] = f"{b}.norm3.weight"  # the checkpoint's norm3 is the model's cross-attn norm2
    m[f"{b}.norm2.bias"] = f"{b}.norm3.bias"
    m[f"{b}.ffn.up_proj_weight"] = [f"{b}.ffn.0.weight", f"{b}.ffn.0.scale_weight"]
    m[f"{b}.ffn.up_proj_bias"] = f"{b}.ffn.0.bias"
    m[f"{b}.ffn.down_proj_weight"] = [f"{b}.ffn.2.weight", f"{b}.ffn.2.scale_weight"]
    m[f"{b}.ffn.down_proj_bias"] = f"{b}.ffn.2.bias"
    m[f"{b}.scale_shift_table"] = f"{b}.modulation"
    return m


def validate_fp8_checkpoint(header: dict, num_layers: int) -> None:
    """Every quantized weight of blocks [0, num_layers) is a 2-D F8_E4M3 ``[out, in]`` with a scalar
    F32 ``scale_weight``; raises :class:`Fp8CheckpointError` otherwise."""
    for i in range(num_layers):
        for name, src in block_key_map(i).items():
            if not isinstance(src, list) or not name.endswith("_weight"):
                continue
            for wk, sk in zip(src[0::2], src[1::2]):
                w = header.get(wk)
                if w is None:
                    raise Fp8CheckpointError(f"missing FP8 weight: {wk}")
                if w.get("dtype") != FP8_DTYPE_STR:
                    raise Fp8CheckpointError(f"{wk} must be {FP8_DTYPE_STR}, got {w.get('dtype')}")
                if len(w.get("shape", [])) != 2:
                    raise Fp8CheckpointError(f"{wk} must be 2-D [out, in], got shape {w.get('shape')}")
                s = header.get(sk)
                if s is None:
                    raise Fp8CheckpointError(f"missing FP8 weight scale: {sk}")
                if s.get("dtype") != "F32":
                    raise Fp8CheckpointError(f"{sk} must be F32, got {s.get('dtype')}")
                if s.get("shape") not in ([], [1]):
                    raise Fp8CheckpointError(f"{sk} must be scalar, got shape {s.get('shape')}")


def _scalar(t: torch.Tensor) -> float:
    t = t.reshape(-1).float()
    if t.numel() != 1:
        raise ValueError(f"expected a scalar per-tensor scale, got {t.numel()} elements")
    v = float(t.item())
    if not np.isfinite(v):
        raise ValueError("expected a finite per-tensor scale")
    return v


def dequantize_to_bf16(w_fp8: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """``(fp8.float() * scale).bfloat16()`` in the stored ``[out, in]`` orientation."""
    return (w_fp8.float() * _scalar(scale)).bfloat16()


def block_weights_bf16(t: dict, i: int) -> dict:
    """Block ``i`` of a loaded checkpoint as the reference's parameter dict (``[in, out]`` bf16 projection
    weights, fused Q|K|V with per-source scales), ready for :func:`prepare_block_weights`."""
    m = block_key_map(i)
    b = f"blocks.{i}"
    out = {}
    for name, src in m.items():
        if isinstance(src, list) and name.endswith("_weight"):
            pairs = list(zip(src[0::2], src[1::2]))
            out[name] = torch.cat([dequantize_to_bf16(t[wk], t[sk]).T for wk, sk in pairs], dim=1).contiguous()
        elif isinstance(src, list):  # fused bias
            out[name] = torch.cat([t[k].float() for k in src]).to(torch.bfloat16)
        else:
            out[name] = t[src].float() if name.endswith("scale_shift_table") else t[src].to(torch.bfloat16)
    # the block code reads ffn.up_weight / ffn.down_weight (the reference's ffn.up_proj_weight ...)
    out[f"{b}.ffn.up_weight"] = out.pop(f"{b}.ffn.up_proj_weight")
    out[f"{b}.ffn.down_weight"] = out.pop(f"{b}.ffn.down_proj_weight")
    out[f"{b}.ffn.up_bias"] = out.pop(f"{b}.ffn.up_proj_bias")
    out[f"{b}.ffn.down_bias"] = out.pop(f"{b}.ffn.down_proj_bias")
    return {k[len(b) + 1:]: v for k, v in out.items()}


def fp8_qkv_leaf(t: dict, i: int, heads: int, head_dim: int = 128):
    """The FP8 self-attention leaf's QKV operands from block ``i``: (codes ``[I, H]`` float8_e4m3fn with
    Q/K rows de-interleaved per head, chan_scale ``[I]`` fp32, bias ``[I]`` bf16 de-interleaved, norm_q /
    norm_k gammas de-interleaved)."""
    b = f"blocks.{i}"
    qd = heads * head_dim
    codes = torch.cat([t[f"{b}.self_attn.{p}.weight"].view(torch.uint8) for p in ("q", "k", "v")], dim=0)
    # rows = output channels; de-interleaving Q/K output channels permutes rows of [out, in]
    codes = deinterleave_qk_columns(codes.T.contiguous(), qd, qd, head_dim).T.contiguous().view(torch.float8_e4m3fn)
    chan = torch.cat([torch.full((qd,), _scalar(t[f"{b}.self_attn.{p}.scale_weight"])) for p in ("q", "k", "v")])
    bias = torch.cat([t[f"{b}.self_attn.{p}.bias"].float() for p in ("q", "k", "v")]).reshape(1, -1)
    bias = deinterleave_qk_columns(bias, qd, qd, head_dim).reshape(-1).to(torch.bfloat16)
    gq = deinterleave_gamma_row(t[f"{b}.self_attn.norm_q.weight"].float().reshape(1, -1), head_dim).reshape(-1)
    gk = deinterleave_gamma_row(t[f"{b}.self_attn.norm_k.weight"].float().reshape(1, -1), head_dim).reshape(-1)
    return codes, chan.float(), bias, gq.to(torch.bfloat16), gk.to(torch.bfloat16)


def fp8_ffn_leaf(t: dict, i: int):
    """The FP8 FFN leaf's operands from block ``i`` (``ffn.0`` = up, ``ffn.2`` = down; nn.Linear
    weights ``[out, in]`` are already the K-major W^T the kernels read): (up codes ``[I, H]``, up scale
    ``[I]``, down codes ``[H, I]``, down scale ``[H]``), the per-tensor scalars expanded per output
    channel (expanded_scalar_scale_loader, row_mx_loaders.py)."""
    b = f"blocks.{i}"
    up = t[f"{b}.ffn.0.weight"].view(torch.uint8).contiguous().view(torch.float8_e4m3fn)
    down = t[f"{b}.ffn.2.weight"].view(torch.uint8).contiguous().view(torch.float8_e4m3fn)
    us = torch.full((up.shape[0],), _scalar(t[f"{b}.ffn.0.scale_weight"]), dtype=torch.float32)
    ds = torch.full((down.shape[0],), _scalar(t[f"{b}.ffn.2.scale_weight"]), dtype=torch.float32)
    return up, us, down, ds


def write_safetensors(path, tensors: dict, metadata: dict | None = None) -> None:
    """Minimal safetensors writer (used to build test checkpoints)."""
    rev = {v[1]: k for k, v in _DTYPES.items()}
    header, blobs, off = {}, [], 0
    for name, t in tensors.items():
        t = t.contiguous().cpu()
        if t.dtype == torch.float8_e4m3fn:
            data = t.view(torch.uint8).numpy().tobytes()
        elif t.dtype == torch.bfloat16:
            data = t.view(torch.uint16).numpy().tobytes() if hasattr(torch, "uint16") else t.view(torch.int16).numpy().tobytes()
        else:
            data = t.numpy().tobytes()
        header[name] = {"dtype": rev[t.dtype], "shape": list(t.shape), "data_offsets": [off, off + len(data)]}
        blobs.append(data)
        off += len(data)
    if metadata:
        header["__metadata__"] = metadata
    h = json.dumps(header).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for d in blobs:
            f.write(d)
