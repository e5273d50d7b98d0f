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
