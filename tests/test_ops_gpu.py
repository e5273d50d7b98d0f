"""torch.ops.b200omni.* on the GPU: each operator returns exactly what its Python entry point returns,
attention_cte matches the exact attention, and torch.library.opcheck accepts the registrations
(schema, fake-tensor consistency)."""

import math

import numpy as np
import pytest
import torch

from oracle import attention as oat

pytestmark = pytest.mark.gpu


def _bf(*shape, seed, scale=1.0, dev="cuda"):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(torch.bfloat16).to(dev)


def test_attention_cte_contract(pkg, dev):
    """``_nki_attend``'s call (WT:653-674): q pre-scaled to [BN, S_q, D], k/v [BN, S_k, D], d-major out."""
    B, N, S, L, D = 1, 3, 200, 150, 128
    q, k, v = _bf(B, N, S, D, seed=1, scale=0.5), _bf(B, N, L, D, seed=2, scale=0.5), _bf(B, N, L, D, seed=3, scale=0.5)
    scale = 1 / math.sqrt(D)
    q3 = (q.reshape(B * N, S, D) * scale).contiguous()
    out = torch.ops.b200omni.attention_cte(q3, k.reshape(B * N, L, D).contiguous(), v.reshape(B * N, L, D).contiguous())
    torch.cuda.synchronize()
    assert out.shape == (B * N, D, S)
    ref = oat.torch_attend(q3.float().cpu().numpy()[None], k.reshape(1, B * N, L, D).float().cpu().numpy(),
                           v.reshape(1, B * N, L, D).float().cpu().numpy(), 1.0)[0]  # [BN, S, D]
    got = out.float().cpu().numpy().transpose(0, 2, 1)
    cos = (got * ref).sum() / math.sqrt((got * got).sum() * (ref * ref).sum())
    assert cos >= 0.9999 and np.abs(got - ref).max() <= 2e-2


def test_ops_equal_python_entry_points(pkg, dev):
    ops = torch.ops.b200omni
    act = _bf(1, 2, 128, 64, seed=4)
    w = _bf(256, 256, seed=5, scale=0.04)
    b = _bf(1, 256, seed=6, scale=0.1)
    assert torch.equal(ops.output_projection_cte(act, w, b), pkg.wan_o_proj(act, w, b))
    h = _bf(1, 40, 256, seed=7)
    wu, wd = _bf(256, 512, seed=8, scale=0.04), _bf(512, 256, seed=9, scale=0.04)
    bu, bd = _bf(1, 512, seed=10, scale=0.1), _bf(1, 256, seed=11, scale=0.1)
    assert torch.equal(ops.mlp(h, wu, wd, bu, bd), pkg.wan_mlp(h, wu, wd, bu, bd))
    q, k, v = (_bf(1, 300, 2, 128, seed=s, scale=0.5) for s in (12, 13, 14))
    o, lse = ops.ring_attention_const_max_fwd(q, k, v, 1, None, None, True)
    o2, lse2 = pkg.ring_attention_const_max_fwd(q, k, v, training=True)
    assert torch.equal(o, o2) and torch.equal(lse, lse2)
    x = _bf(2, 33, 256, seed=15)
    res = _bf(2, 33, 256, seed=16)
    mul, add = _bf(2, 1, 256, seed=17, scale=0.1) + 1, _bf(2, 1, 256, seed=18, scale=0.1)
    got = ops.adaln_modulate(x, mul, add, 1e-6, "layer_norm", "row", True, res, None)
    want = pkg.adaln_modulate(x, mul, add, eps=1e-6, quant="row", residual=res)
    assert torch.equal(got[0], want[0]) and torch.equal(got[1].view(torch.uint8), want[1].view(torch.uint8))
    pos, neg = _bf(4099, seed=19), _bf(4099, seed=20)
    assert torch.equal(ops.cfg_combine(pos, neg, 5.0), pkg.cfg_combine(pos, neg, 5.0))


def test_fp8_ops_equal_python_entry_points(pkg, dev):
    ops = torch.ops.b200omni
    T, H, I = 64, 256, 512
    x = _bf(1, T, H, seed=21)
    packed = pkg.adaln_modulate(x, None, None, eps=1e-6, quant="row")
    g = torch.Generator().manual_seed(22)
    uc, us, dc, ds = pkg.quantize_mlp_weights_row_mx((torch.randn(H, I, generator=g) * 0.02).to(dev),
                                                     (torch.randn(I, H, generator=g) * 0.02).to(dev))
    assert torch.equal(ops.row_mx_mlp(packed, uc, dc, us, ds, None, None), pkg.row_mx_mlp(packed, uc, dc, us, ds, None, None))
    wq = torch.randn(H, 3 * H, generator=g).to(dev) * 0.02
    codes, chan = pkg.quantize_qkv_weight(wq, H, H)
    y1 = ops.row_mx_qkv_proj(packed, codes, chan, None, 2, 128, 2)
    y2 = pkg.row_mx_qkv_proj(packed, codes, chan, None, num_heads=2, head_dim=128, num_kv_heads=2)
    assert torch.equal(y1, y2)


def test_opcheck(pkg, dev):
    q3 = _bf(4, 130, 128, seed=30, scale=0.05)
    k3, v3 = _bf(4, 70, 128, seed=31, scale=0.5), _bf(4, 70, 128, seed=32, scale=0.5)
    tests = ("test_schema", "test_faketensor")
    torch.library.opcheck(torch.ops.b200omni.attention_cte.default, (q3, k3, v3), test_utils=tests)
    pos, neg = _bf(1000, seed=33), _bf(1000, seed=34)
    torch.library.opcheck(torch.ops.b200omni.cfg_combine.default, (pos, neg, 3.5), test_utils=tests)
    h = _bf(1, 40, 256, seed=35)
    torch.library.opcheck(torch.ops.b200omni.mlp.default,
                          (h, _bf(256, 512, seed=36, scale=0.04), _bf(512, 256, seed=37, scale=0.04),
                           _bf(1, 512, seed=38), _bf(1, 256, seed=39)), test_utils=tests)
