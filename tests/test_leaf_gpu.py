"""The FP8 self-attention leaf end to end (adaLN row quant -> FP8 QKV + norm + RoPE -> const-max
attention on strided Q/K/V views) against the CPU oracle chain, and strided-view attention equals
contiguous attention bit for bit (B200 only)."""

import math

import numpy as np
import pytest
import torch

from oracle import attention as oat
from oracle import qkv as oq
from oracle.numerics import e4m3fn_from_bits

pytestmark = pytest.mark.gpu


def test_strided_views_equal_contiguous(pkg, dev):
    g = torch.Generator().manual_seed(0)
    b, s, h = 2, 200, 2
    qkv = (torch.randn(b, s, 3 * h * 128, generator=g) * 0.5).to(torch.bfloat16).to(dev)
    q, k, v = (t.unflatten(2, (h, 128)) for t in torch.tensor_split(qkv, 3, dim=-1))
    assert not q.is_contiguous()
    o_view = pkg.ring_attention_const_max_fwd(q, k, v)
    o_cont = pkg.ring_attention_const_max_fwd(q.contiguous(), k.contiguous(), v.contiguous())
    torch.cuda.synchronize()
    assert torch.equal(o_view, o_cont)


def test_fp8_leaf_vs_oracle(pkg, dev):
    rope = pytest.importorskip("importlib").import_module("vllm-omni-neuron_b200.rope")
    T, H, heads = 600, 512, 2
    qd = heads * 128
    g = torch.Generator().manual_seed(7)
    hidden = torch.randn(1, T, H, generator=g).to(torch.bfloat16).to(dev)
    w = (torch.randn(H, 3 * qd, generator=g) * 0.02).to(dev)
    bias = (torch.randn(3 * qd, generator=g) * 0.05).to(torch.bfloat16).to(dev)
    gq = (1 + 0.1 * torch.randn(qd, generator=g)).to(torch.bfloat16).to(dev)
    gk = (1 + 0.1 * torch.randn(qd, generator=g)).to(torch.bfloat16).to(dev)
    cos, sin = rope.wan_rotary_freqs(128, (1, 2, 2), 1024, (3, 20, 40), device=dev)
    wd = rope.deinterleave_qk_columns(w, qd, qd, 128)
    wq, chan = pkg.quantize_qkv_weight(wd, qd, qd)
    packed = pkg.adaln_modulate(hidden, None, None, eps=1e-6, norm_type="layer_norm", quant="row")
    out = pkg.wan_self_attention_fp8(packed, wq, chan, bias, gq, gk, (cos, sin), num_heads=heads)
    torch.cuda.synchronize()
    assert tuple(out.shape) == (1, heads, 128, T)
    # oracle chain on the same FP8 codes
    cos_rh, sin_rh = rope.rope_rotate_half_caches(cos, sin)
    y = oq.row_mx_qkv_ref(packed.view(torch.uint8).cpu().numpy()[0], e4m3fn_from_bits(wq.view(torch.uint8).cpu().numpy()).T,
                          chan.cpu().numpy(), bias.float().cpu().numpy(), num_heads=heads, head_dim=128, num_kv_heads=heads,
                          gamma_q=gq.float().cpu().numpy(), gamma_k=gk.float().cpu().numpy(),
                          cos=cos_rh.reshape(T, 128).cpu().numpy(), sin=sin_rh.reshape(T, 128).cpu().numpy(), eps=1e-6)
    q = y[:, :qd].reshape(1, T, heads, 128)
    k = y[:, qd:2 * qd].reshape(1, T, heads, 128)
    v = y[:, 2 * qd:].reshape(1, T, heads, 128)
    ref = oat.wan_cp_self_attention_oracle([q], [k], [v], 1 / math.sqrt(128))[0]
    got = out.float().cpu().numpy().astype(np.float64)
    r = ref.astype(np.float64)
    cos_sim = (got * r).sum() / math.sqrt((got * got).sum() * (r * r).sum())
    assert cos_sim >= 0.9999 and np.abs(got - r).max() <= 2e-2, (cos_sim, np.abs(got - r).max())


def test_fp8_cross_attention_leaf_vs_oracle(pkg, dev):
    """WanCrossAttentionFP8 up to the attention output (row_mx_modules.py:478-542): separate ROW FP8
    Q/K/V projections, across-heads RMS norm on Q and K (no RoPE), exact attention over the text
    tokens, against the oracle chain on the same FP8 codes."""
    B, S, L, H, heads = 1, 300, 64, 256, 2
    qd = heads * 128
    g = torch.Generator().manual_seed(8)
    hidden = torch.randn(B, S, H, generator=g).to(torch.bfloat16).to(dev)
    ctx = torch.randn(B, L, H, generator=g).to(torch.bfloat16).to(dev)
    ws = {n: (torch.randn(H, qd, generator=g) * 0.03).to(dev) for n in "qkv"}
    bs = {n: (torch.randn(qd, generator=g) * 0.05).to(torch.bfloat16).to(dev) for n in "qkv"}
    gq = (1 + 0.1 * torch.randn(qd, generator=g)).to(torch.bfloat16).to(dev)
    gk = (1 + 0.1 * torch.randn(qd, generator=g)).to(torch.bfloat16).to(dev)
    quant = {n: pkg.quantize_qkv_weight(ws[n], qd, 0) for n in "qkv"}
    packed = pkg.adaln_modulate(hidden, None, None, eps=1e-6, norm_type="layer_norm", quant="row")
    packed_ctx = pkg.adaln_modulate(ctx, None, None, eps=1e-6, norm_type="none", quant="row")
    kv = pkg.project_cross_kv_fp8(packed_ctx, quant["k"][0], quant["k"][1], bs["k"], gk, quant["v"][0], quant["v"][1],
                                  bs["v"], num_heads=heads)
    out = pkg.wan_cross_attention_fp8(packed, quant["q"][0], quant["q"][1], bs["q"], gq, kv, num_heads=heads)
    torch.cuda.synchronize()
    assert tuple(out.shape) == (B, heads, 128, S)

    def proj(pk, n, gamma):
        codes, chan = quant[n]
        kw = dict(num_heads=heads, head_dim=128, num_kv_heads=0, eps=1e-6)
        if gamma is not None:
            kw["gamma_q"] = gamma.float().cpu().numpy()
        return oq.row_mx_qkv_ref(pk.view(torch.uint8).cpu().numpy()[0], e4m3fn_from_bits(codes.view(torch.uint8).cpu().numpy()).T,
                                 chan.cpu().numpy(), bs[n].float().cpu().numpy(), **(kw if gamma is not None else {}))

    q = proj(packed, "q", gq).reshape(B, S, heads, 128)
    k = proj(packed_ctx, "k", gk).reshape(B, L, heads, 128)
    v = proj(packed_ctx, "v", None).reshape(B, L, heads, 128)
    np.testing.assert_allclose(kv[1].float().cpu().numpy(), v, atol=1e-2, rtol=1e-2)
    ref = oat.torch_attend(q.transpose(0, 2, 1, 3), k.transpose(0, 2, 1, 3), v.transpose(0, 2, 1, 3), 1 / math.sqrt(128))
    ref = ref.transpose(0, 1, 3, 2)  # d-major
    got = out.float().cpu().numpy().astype(np.float64)
    r = ref.astype(np.float64)
    cos_sim = (got * r).sum() / math.sqrt((got * got).sum() * (r * r).sum())
    assert cos_sim >= 0.9999 and np.abs(got - r).max() <= 2e-2, (cos_sim, np.abs(got - r).max())
