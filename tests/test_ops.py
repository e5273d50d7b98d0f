"""The torch custom operators (torch.ops.b200omni.*): registration and fake (meta) shapes, on the CPU."""

import pytest
import torch

M = torch.device("meta")


def _e(*shape, dtype=torch.bfloat16):
    return torch.empty(*shape, device=M, dtype=dtype)


def test_registered(pkg):
    for name in ("attention_cte", "output_projection_cte", "mlp", "ring_attention_const_max_fwd", "adaln_modulate",
                 "row_mx_qkv_proj", "row_mx_mlp", "cfg_combine"):
        assert hasattr(torch.ops.b200omni, name), name


def test_fake_shapes(pkg):
    ops = torch.ops.b200omni
    assert ops.attention_cte(_e(80, 300, 128), _e(80, 512, 128), _e(80, 512, 128)).shape == (80, 128, 300)
    assert ops.output_projection_cte(_e(2, 40, 128, 300), _e(5120, 5120), _e(1, 5120)).shape == (2, 300, 5120)
    assert ops.mlp(_e(1, 300, 5120), _e(5120, 13824), _e(13824, 5120), _e(1, 13824), _e(1, 5120)).shape == (1, 300, 5120)
    o = ops.ring_attention_const_max_fwd(_e(1, 4095, 40, 128), _e(1, 4095, 40, 128), _e(1, 4095, 40, 128), 1, None, None, True)
    assert [t.shape for t in o] == [(1, 40, 4095, 128), (1, 40, 128, 32)] and o[1].dtype == torch.float32
    a = ops.adaln_modulate(_e(2, 10, 256), _e(2, 1, 256), _e(2, 1, 256), 1e-6, "layer_norm", "row", True, None, None)
    assert len(a) == 1 and a[0].shape == (2, 10, 260) and a[0].dtype == torch.float8_e4m3fn
    a = ops.adaln_modulate(_e(2, 10, 256), None, None, 1e-6, "rms_norm", "mx32", True, _e(2, 10, 256), None)
    assert [t.shape for t in a] == [(2, 10, 256), (2, 10, 256), (2, 10, 8)]
    y = ops.row_mx_qkv_proj(_e(1, 64, 5124, dtype=torch.float8_e4m3fn), _e(15360, 5120, dtype=torch.float8_e4m3fn),
                            _e(15360, dtype=torch.float32), None, 40, 128, 40)
    assert y.shape == (1, 64, 15360) and y.dtype == torch.bfloat16
    f = ops.row_mx_mlp(_e(64, 5124, dtype=torch.float8_e4m3fn), _e(13824, 5120, dtype=torch.float8_e4m3fn),
                       _e(5120, 13824, dtype=torch.float8_e4m3fn), _e(13824, dtype=torch.float32),
                       _e(5120, dtype=torch.float32), None, None)
    assert f.shape == (64, 5120)
    assert ops.cfg_combine(_e(1, 16, 21, 60, 104), _e(1, 16, 21, 60, 104), 5.0).shape == (1, 16, 21, 60, 104)


def test_no_cpu_path(pkg):
    x = torch.zeros(16, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError):
        torch.ops.b200omni.cfg_combine(x, x, 5.0)
