"""GPU parity of a whole Wan transformer block (bf16 leaves: adaLN, QKV + RMS + RoPE, const-max
attention, o-proj + gated residual + norm2, cross-attention, norm3, FFN + gated residual) against the
CPU oracle composed from the pinned restatements (B200 only)."""

import math

import numpy as np
import pytest
import torch

from oracle import block as ob
from oracle import rope as orope
from oracle.numerics import bf16_round

pytestmark = pytest.mark.gpu


def make_block(B, latent, H, I, L, seed=0, cross_norm=True):
    rng = np.random.default_rng(seed)
    S = latent[0] * (latent[1] // 2) * (latent[2] // 2)
    bfn = lambda *shape, s=1.0: bf16_round((s * rng.standard_normal(shape)).astype(np.float32))
    w = {
        "scale_shift_table": (rng.standard_normal((1, 6, H)) / math.sqrt(H)).astype(np.float32),
        "attn1.qkv_proj_weight": bfn(H, 3 * H, s=0.04), "attn1.qkv_proj_bias": bfn(3 * H, s=0.1),
        "attn1.norm_q.weight": bfn(H, s=0.1) + 1, "attn1.norm_k.weight": bfn(H, s=0.1) + 1,
        "attn1.o_proj_weight": bfn(H, H, s=0.04), "attn1.o_proj_bias": bfn(H, s=0.1),
        "norm2.weight": (bfn(H, s=0.1) + 1) if cross_norm else None, "norm2.bias": bfn(H, s=0.1) if cross_norm else None,
        "attn2.q_proj_weight": bfn(H, H, s=0.04), "attn2.q_proj_bias": bfn(H, s=0.1),
        "attn2.norm_q.weight": bfn(H, s=0.1) + 1,
        "attn2.k_proj_weight": bfn(H, H, s=0.04), "attn2.k_proj_bias": bfn(H, s=0.1),
        "attn2.norm_k.weight": bfn(H, s=0.1) + 1,
        "attn2.v_proj_weight": bfn(H, H, s=0.04), "attn2.v_proj_bias": bfn(H, s=0.1),
        "attn2.o_proj_weight": bfn(H, H, s=0.04), "attn2.o_proj_bias": bfn(H, s=0.1),
        "ffn.up_weight": bfn(H, I, s=0.04), "ffn.up_bias": bfn(I, s=0.1),
        "ffn.down_weight": bfn(I, H, s=0.04), "ffn.down_bias": bfn(H, s=0.1),
    }
    hidden = bfn(B, S, H)
    temb = (0.1 * rng.standard_normal((B, 6, H))).astype(np.float32)
    ctx = bfn(B, L, H)
    cos, sin = orope.rotary_freqs(128, (1, 2, 2), 1024, latent)
    return w, hidden, temb, ctx, np.asarray(cos, np.float32).reshape(S, 128), np.asarray(sin, np.float32).reshape(S, 128)


@pytest.mark.parametrize("B,latent,H,I,L,cross_norm", [(1, (3, 20, 20), 256, 512, 40, True), (2, (1, 10, 26), 512, 768, 24, False)])
def test_block_vs_oracle(pkg, dev, B, latent, H, I, L, cross_norm):
    heads = H // 128
    w, hidden, temb, ctx, cos, sin = make_block(B, latent, H, I, L, cross_norm=cross_norm)
    tt = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(dev)
    wt = {k: (tt(v) if v is not None else None) for k, v in w.items()}
    bw = pkg.prepare_block_weights(wt, heads)
    kv = pkg.project_cross_kv(tt(ctx).to(torch.bfloat16), wt["attn2.k_proj_weight"], wt["attn2.k_proj_bias"],
                              wt["attn2.norm_k.weight"], wt["attn2.v_proj_weight"], wt["attn2.v_proj_bias"], heads)
    rope = pytest.importorskip("importlib").import_module("vllm-omni-neuron_b200.rope")
    S = hidden.shape[1]
    cos_rh, sin_rh = rope.rope_rotate_half_caches(tt(cos).reshape(1, S, 1, 128), tt(sin).reshape(1, S, 1, 128))
    out = pkg.wan_block_forward(tt(hidden).to(torch.bfloat16), tt(temb), (cos_rh, sin_rh), kv, bw)
    torch.cuda.synchronize()
    kv_ref = ob.project_kv_ref(ctx, w["attn2.k_proj_weight"], w["attn2.k_proj_bias"], w["attn2.norm_k.weight"],
                               w["attn2.v_proj_weight"], w["attn2.v_proj_bias"], heads, 1e-6)
    np.testing.assert_allclose(kv[1].float().cpu().numpy(), kv_ref[1], atol=2e-2, rtol=2e-2)
    ref = ob.wan_block_ref(hidden, temb, cos, sin, kv_ref, w, heads)
    got = out.float().cpu().numpy().astype(np.float64)
    r = ref.astype(np.float64)
    cos_sim = (got * r).sum() / math.sqrt((got * got).sum() * (r * r).sum())
    assert cos_sim > 0.99995, cos_sim
    assert np.abs(got - r).max() <= 0.05 * max(1.0, np.abs(r).max()), np.abs(got - r).max()


def test_block_fp8_ffn_vs_oracle(pkg, dev):
    """The block with the FFN's FP8 leaf (norm3 ROW-quantised, row_mx_mlp with the closing gated
    residual) against the oracle block running the ROW_MX MLP restatement on the same codes."""
    B, latent, H, I, L = 1, (3, 20, 20), 256, 512, 40
    heads = H // 128
    w, hidden, temb, ctx, cos, sin = make_block(B, latent, H, I, L, seed=3)
    tt = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(dev)
    wt = {k: (tt(v) if v is not None else None) for k, v in w.items()}
    bw = pkg.prepare_block_weights(wt, heads, ffn_fp8=True)
    assert bw.ffn_fp8 is not None
    kv = pkg.project_cross_kv(tt(ctx).to(torch.bfloat16), wt["attn2.k_proj_weight"], wt["attn2.k_proj_bias"],
                              wt["attn2.norm_k.weight"], wt["attn2.v_proj_weight"], wt["attn2.v_proj_bias"], heads)
    rope = pytest.importorskip("importlib").import_module("vllm-omni-neuron_b200.rope")
    S = hidden.shape[1]
    cos_rh, sin_rh = rope.rope_rotate_half_caches(tt(cos).reshape(1, S, 1, 128), tt(sin).reshape(1, S, 1, 128))
    out = pkg.wan_block_forward(tt(hidden).to(torch.bfloat16), tt(temb), (cos_rh, sin_rh), kv, bw)
    torch.cuda.synchronize()
    kv_ref = ob.project_kv_ref(ctx, w["attn2.k_proj_weight"], w["attn2.k_proj_bias"], w["attn2.norm_k.weight"],
                               w["attn2.v_proj_weight"], w["attn2.v_proj_bias"], heads, 1e-6)
    fp8 = tuple(t.float().cpu().numpy() for t in bw.ffn_fp8)
    ref = ob.wan_block_ref(hidden, temb, cos, sin, kv_ref, w, heads, ffn_fp8=fp8)
    got = out.float().cpu().numpy().astype(np.float64)
    r = ref.astype(np.float64)
    cos_sim = (got * r).sum() / math.sqrt((got * got).sum() * (r * r).sum())
    assert cos_sim > 0.9999, cos_sim
    assert np.abs(got - r).max() <= 0.05 * max(1.0, np.abs(r).max()), np.abs(got - r).max()


def test_two_blocks_and_output_head(pkg, dev):
    """A 2-block DiT slice plus the output head (wan2_2_transformer.py:1814-1829) at CP=1."""
    dit = pytest.importorskip("importlib").import_module("vllm-omni-neuron_b200.dit")
    rope = pytest.importorskip("importlib").import_module("vllm-omni-neuron_b200.rope")
    H, heads, I, L, latent = 256, 2, 512, 32, (2, 12, 16)
    tt = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(dev)
    blocks, kvs, refs = [], [], []
    for i in range(2):
        w, hidden0, temb, ctx, cos, sin = make_block(1, latent, H, I, L, seed=10 + i)
        if i == 0:
            hidden, temb0, cos0, sin0 = hidden0, temb, cos, sin
        wt = {k: (tt(v) if v is not None else None) for k, v in w.items()}
        blocks.append(pkg.prepare_block_weights(wt, heads))
        kvs.append(pkg.project_cross_kv(tt(ctx).to(torch.bfloat16), wt["attn2.k_proj_weight"], wt["attn2.k_proj_bias"],
                                        wt["attn2.norm_k.weight"], wt["attn2.v_proj_weight"], wt["attn2.v_proj_bias"], heads))
        refs.append((w, ob.project_kv_ref(ctx, w["attn2.k_proj_weight"], w["attn2.k_proj_bias"], w["attn2.norm_k.weight"],
                                          w["attn2.v_proj_weight"], w["attn2.v_proj_bias"], heads, 1e-6)))
    S = hidden.shape[1]
    cos_rh, sin_rh = rope.rope_rotate_half_caches(tt(cos0).reshape(1, S, 1, 128), tt(sin0).reshape(1, S, 1, 128))
    rng = np.random.default_rng(3)
    table = (rng.standard_normal((1, 2, H)) / 16).astype(np.float32)
    temb_h = (0.1 * rng.standard_normal((1, H))).astype(np.float32)
    proj_w = bf16_round((0.05 * rng.standard_normal((64, H))).astype(np.float32))
    proj_b = bf16_round((0.1 * rng.standard_normal(64)).astype(np.float32))
    x = dit.wan_blocks_forward(tt(hidden).to(torch.bfloat16), tt(temb0), (cos_rh, sin_rh), kvs, blocks)
    out = dit.wan_output_head(x, tt(temb_h), tt(table), tt(proj_w).to(torch.bfloat16), tt(proj_b).to(torch.bfloat16))
    torch.cuda.synchronize()
    r = hidden
    for w, kv in refs:
        r = ob.wan_block_ref(r, temb0, cos0, sin0, kv, w, heads)
    ref = ob.wan_output_head_ref(r, temb_h, table, proj_w, proj_b)
    got = out.float().cpu().numpy().astype(np.float64)
    cos_sim = (got * ref).sum() / math.sqrt((got * got).sum() * (ref.astype(np.float64) ** 2).sum())
    assert out.shape == (1, S, 64) and cos_sim > 0.9999, cos_sim
