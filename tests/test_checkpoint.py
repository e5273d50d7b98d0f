"""FP8 checkpoint ingestion (CPU): the key table and dequant pinned to the reference's own code,
a synthetic ComfyUI-format checkpoint round trip, validation errors."""

import json
from importlib import import_module

import numpy as np
import pytest
import torch

from oracle import rope as orope
from oracle.numerics import bf16_round

ck = import_module("vllm-omni-neuron_b200.checkpoint")


def test_key_map_matches_reference():
    from pathlib import Path

    g = json.loads((Path(__file__).parent / "golden" / "comfy_fp8_mapping.json").read_text())["mappings"]
    for i in range(2):
        for name, src in ck.block_key_map(i).items():
            assert g[name] == src, name
    ours = {k for i in range(2) for k in ck.block_key_map(i)}
    theirs = {k for k in g if k.startswith("blocks.")}
    assert ours == theirs


def test_dequant_matches_reference(golden):
    g = golden("fp8_dequant.npz")
    w = torch.from_numpy(g["codes"]).view(torch.float8_e4m3fn)
    y = ck.dequantize_to_bf16(w, torch.from_numpy(np.asarray(g["scale"])))
    assert np.array_equal(y.float().numpy(), g["y"])
    with pytest.raises(ValueError):
        ck.dequantize_to_bf16(w, torch.ones(2))


def _quant(w):  # per-tensor absmax to e4m3fn, as the ComfyUI files are made
    s = np.float32(max(np.abs(w).max() / 448.0, 1e-12))
    return torch.from_numpy((w / s).astype(np.float32)).to(torch.float8_e4m3fn), torch.tensor(s, dtype=torch.float32)


def make_checkpoint(path, n_blocks=2, H=256, heads=2, I=512, seed=0):
    rng = np.random.default_rng(seed)
    t = {}
    for i in range(n_blocks):
        b = f"blocks.{i}"
        lin = {"self_attn.q": (H, H), "self_attn.k": (H, H), "self_attn.v": (H, H), "self_attn.o": (H, H),
               "cross_attn.q": (H, H), "cross_attn.k": (H, H), "cross_attn.v": (H, H), "cross_attn.o": (H, H),
               "ffn.0": (I, H), "ffn.2": (H, I)}
        for k, (o, n) in lin.items():
            w, s = _quant((0.05 * rng.standard_normal((o, n))).astype(np.float32))
            t[f"{b}.{k}.weight"] = w
            t[f"{b}.{k}.scale_weight"] = s
            t[f"{b}.{k}.scale_input"] = torch.tensor(1.0)
            t[f"{b}.{k}.bias"] = torch.from_numpy((0.1 * rng.standard_normal(o)).astype(np.float16))
        for k in ("self_attn.norm_q", "self_attn.norm_k", "cross_attn.norm_q", "cross_attn.norm_k", "norm3"):
            t[f"{b}.{k}.weight"] = torch.from_numpy((1 + 0.1 * rng.standard_normal(H)).astype(np.float16))
        t[f"{b}.norm3.bias"] = torch.from_numpy((0.1 * rng.standard_normal(H)).astype(np.float16))
        t[f"{b}.modulation"] = torch.from_numpy(rng.standard_normal((1, 6, H)).astype(np.float32))
    t["scaled_fp8"] = torch.zeros(0, dtype=torch.float32)
    ck.write_safetensors(path, t, {"format": "pt"})
    return t


def test_roundtrip_and_layouts(tmp_path):
    p = tmp_path / "wan_fp8.safetensors"
    src = make_checkpoint(p)
    hdr = ck.read_safetensors_header(p)
    ck.validate_fp8_checkpoint(hdr, 2)
    t = ck.load_tensors(p)
    for k, v in src.items():
        got = t[k]
        assert got.dtype == v.dtype and tuple(got.shape) == tuple(v.shape), k
        if v.dtype == torch.float8_e4m3fn:
            assert torch.equal(got.view(torch.uint8), v.view(torch.uint8)), k
        else:
            assert torch.equal(got, v), k
    H, heads, qd = 256, 2, 256
    w = ck.block_weights_bf16(t, 1)
    # fused QKV: per-source dequant, [in, out], q|k|v order
    parts = [(src[f"blocks.1.self_attn.{p}.weight"].float() * float(src[f"blocks.1.self_attn.{p}.scale_weight"])).bfloat16().T
             for p in ("q", "k", "v")]
    assert torch.equal(w["attn1.qkv_proj_weight"], torch.cat(parts, dim=1))
    assert w["ffn.up_weight"].shape == (H, 512) and w["ffn.down_weight"].shape == (512, H)
    assert torch.equal(w["norm2.weight"], src["blocks.1.norm3.weight"].to(torch.bfloat16))
    assert torch.equal(w["scale_shift_table"], src["blocks.1.modulation"])
    # FP8 leaf operands: codes stay codes, Q/K rows de-interleaved, scales expanded per channel
    codes, chan, bias, gq, gk = ck.fp8_qkv_leaf(t, 1, heads)
    cat = torch.cat([src[f"blocks.1.self_attn.{p}.weight"].view(torch.uint8) for p in ("q", "k", "v")]).numpy()
    want = orope.deinterleave_qk_columns(cat.T, qd, qd, 128).T
    assert np.array_equal(codes.view(torch.uint8).numpy(), want)
    assert torch.equal(chan[:qd], torch.full((qd,), float(src["blocks.1.self_attn.q.scale_weight"])))
    assert torch.equal(chan[2 * qd:], torch.full((qd,), float(src["blocks.1.self_attn.v.scale_weight"])))
    b_cat = np.concatenate([src[f"blocks.1.self_attn.{p}.bias"].float().numpy() for p in ("q", "k", "v")])[None]
    assert np.array_equal(bias.float().numpy(), bf16_round(orope.deinterleave_qk_columns(b_cat, qd, qd, 128)).reshape(-1))
    # FP8 FFN leaf: nn.Linear [out, in] codes are the kernels' K-major W^T as stored
    uc, us, dc, ds = ck.fp8_ffn_leaf(t, 1)
    assert uc.dtype == torch.float8_e4m3fn and tuple(uc.shape) == (512, H) and tuple(dc.shape) == (H, 512)
    assert torch.equal(uc.view(torch.uint8), src["blocks.1.ffn.0.weight"].view(torch.uint8))
    assert torch.equal(dc.view(torch.uint8), src["blocks.1.ffn.2.weight"].view(torch.uint8))
    assert torch.equal(us, torch.full((512,), float(src["blocks.1.ffn.0.scale_weight"])))
    assert torch.equal(ds, torch.full((H,), float(src["blocks.1.ffn.2.scale_weight"])))
    # the dequantised bf16 leaf and the FP8 leaf describe the same weights
    assert torch.equal((uc.float() * us[:, None]).bfloat16().T, w["ffn.up_weight"])


def test_validation_errors(tmp_path):
    p = tmp_path / "bad.safetensors"
    src = make_checkpoint(p, n_blocks=1)
    hdr = ck.read_safetensors_header(p)
    bad = dict(hdr)
    del bad["blocks.0.ffn.2.scale_weight"]
    with pytest.raises(ck.Fp8CheckpointError, match="scale"):
        ck.validate_fp8_checkpoint(bad, 1)
    bad = dict(hdr)
    bad["blocks.0.self_attn.q.weight"] = dict(hdr["blocks.0.self_attn.q.weight"], dtype="BF16")
    with pytest.raises(ck.Fp8CheckpointError, match="F8_E4M3"):
        ck.validate_fp8_checkpoint(bad, 1)
    bad = dict(hdr)
    bad["blocks.0.self_attn.o.scale_weight"] = dict(hdr["blocks.0.self_attn.o.scale_weight"], shape=[3])
    with pytest.raises(ck.Fp8CheckpointError, match="scalar"):
        ck.validate_fp8_checkpoint(bad, 1)
    with pytest.raises(ck.Fp8CheckpointError, match="missing"):
        ck.validate_fp8_checkpoint(hdr, 2)  # block 1 absent
