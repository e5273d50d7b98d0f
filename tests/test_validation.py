"""Host-side argument checks that run before any device call (CPU only). They mirror the
reference's error behaviour: shape contracts raise AssertionError (the NKI kernel_assert,
ring_attention_const_max_fwd.py:1019-1031), unsupported modes raise ValueError / NotImplementedError
(adaln_kernels.py:36-44; row_mx_modules.py:226-235), and every kernel refuses CPU tensors (no CPU path)."""

import pytest
import torch


def _bf(*shape):
    return torch.zeros(*shape, dtype=torch.bfloat16)


def test_attention_contracts(pkg):
    q = _bf(1, 16, 2, 64)
    with pytest.raises(AssertionError):  # head_dim must be 128
        pkg.ring_attention_const_max_fwd(q, q, q)
    with pytest.raises(AssertionError):  # q_heads == kv_heads
        pkg.attention_local(_bf(1, 16, 2, 128), _bf(1, 16, 1, 128), _bf(1, 16, 1, 128))
    with pytest.raises(ValueError):  # host tensors must be pinned
        pkg.ring_attention_const_max_fwd(_bf(1, 16, 2, 128), _bf(1, 16, 2, 128), _bf(1, 16, 2, 128))


def test_adaln_modes(pkg):
    x = _bf(4, 256)
    with pytest.raises(NotImplementedError):  # the reference's quant="mx" has no fused path
        pkg.adaln_modulate(x, eps=1e-6, quant="mx")
    with pytest.raises(ValueError):
        pkg.adaln_modulate(x, eps=1e-6, quant="int8")
    with pytest.raises(ValueError):
        pkg.adaln_modulate(x, eps=1e-6, norm_type="group_norm")
    with pytest.raises(TypeError):
        pkg.adaln_modulate(x.float(), eps=1e-6)
    with pytest.raises(RuntimeError):  # no CPU path
        pkg.adaln_modulate(x, eps=1e-6)


def test_qkv_modes(pkg):
    packed = torch.zeros(1, 8, 260, dtype=torch.uint8)
    w = torch.zeros(768, 256, dtype=torch.float8_e4m3fn)
    s = torch.ones(768)
    with pytest.raises(ValueError):
        pkg.row_mx_qkv_proj(packed, w, s, None, num_heads=2, head_dim=64, num_kv_heads=2)
    with pytest.raises(NotImplementedError):  # TP > 1
        pkg.row_mx_qkv_proj(packed, w, s, None, num_heads=2, head_dim=128, num_kv_heads=2,
                            replica_groups=[[0, 1]])


def test_fp8_ffn_and_cfg(pkg):
    codes = torch.zeros(8, 256, dtype=torch.float8_e4m3fn)
    rs = torch.ones(8)
    uc = torch.zeros(512, 256, dtype=torch.float8_e4m3fn)
    dc = torch.zeros(256, 512, dtype=torch.float8_e4m3fn)
    with pytest.raises(RuntimeError):  # no CPU path
        pkg.row_mx_mlp((codes, rs), uc, dc, torch.ones(512), torch.ones(256), None, None)
    with pytest.raises(ValueError):
        pkg.cfg_combine(_bf(4), _bf(5), 5.0)
    with pytest.raises(TypeError):
        pkg.cfg_combine(torch.zeros(4, dtype=torch.float16), torch.zeros(4, dtype=torch.float16), 5.0)
    with pytest.raises(RuntimeError):
        pkg.cfg_combine(_bf(4), _bf(4), 5.0)


def test_weight_quantisers_on_cpu(pkg):
    """The per-tensor weight quantisers are plain torch and also run on the host (load time)."""
    g = torch.Generator().manual_seed(0)
    wu, wd = torch.randn(256, 512, generator=g) * 0.02, torch.randn(512, 256, generator=g) * 0.02
    uc, us, dc, ds = pkg.quantize_mlp_weights_row_mx(wu, wd)
    assert uc.shape == (512, 256) and dc.shape == (256, 512) and uc.dtype == torch.float8_e4m3fn
    assert torch.allclose((uc.float() * us[:, None]).T, wu, rtol=0.07, atol=1e-4)
    assert float(uc.float().abs().max()) == 448.0
    codes, chan = pkg.quantize_qkv_weight(torch.randn(256, 768, generator=g), 256, 256)
    assert codes.shape == (768, 256) and chan.shape == (768,)
