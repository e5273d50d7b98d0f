"""GPU parity of the FP8 (ROW_MX) FFN leaf ``row_mx_mlp`` against the CPU restatement of the
reference's ROW_MX MLP (``oracle.ffn.wan_mlp_row_mx_ref``; B200 only).

FP8 bound: after dequantisation the output must match with cosine >= 0.9999 and a max-abs error of at
most 2e-2 scaled by the output range, 2e-2 * max(1, max|ref|) (the north-star bound for FP8 paths,
stated for unit-range outputs; the FFN's outputs reach |y| ~ 5 at H = 5120, where one bf16 step is
0.03). The MX-32 intermediate is checked on its own: e4m3
codes and UE8M0 scale bytes equal the oracle's except where fp32 accumulation order moves a value
across a rounding boundary (a small fraction, each then one code step apart)."""

import math
from importlib import import_module

import numpy as np
import pytest
import torch

from oracle import ffn as off
from oracle.numerics import bf16_round

pytestmark = pytest.mark.gpu


def _inputs(T, H, I, seed, dev):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, H, generator=g)
    rs = torch.clamp(x.abs().amax(1) / 448.0, min=1e-6)  # ROW quant of the adaLN output
    codes = (x / rs[:, None]).to(torch.float8_e4m3fn)
    wu = torch.randn(H, I, generator=g) * 0.02
    wd = torch.randn(I, H, generator=g) * 0.02
    bu = (torch.randn(I, generator=g) * 0.1).to(torch.bfloat16)
    bd = (torch.randn(H, generator=g) * 0.1).to(torch.bfloat16)
    pkg = import_module("vllm-omni-neuron_b200")
    uc, us, dc, ds = pkg.quantize_mlp_weights_row_mx(wu, wd)
    host = dict(codes=codes, rs=rs, uc=uc, us=us, dc=dc, ds=ds, bu=bu, bd=bd)
    devt = {k: v.to(dev) for k, v in host.items()}
    return host, devt


def _np(t):
    return t.float().numpy()


def _check(got, ref, what):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    assert np.isfinite(got).all(), what
    cos = (got * ref).sum() / math.sqrt((got * got).sum() * (ref * ref).sum())
    mx = np.abs(got - ref).max()
    bound = 2e-2 * max(1.0, np.abs(ref).max())
    assert cos >= 0.9999 and mx <= bound, f"{what}: cos={cos:.6f} maxabs={mx:.3g} (bound {bound:.3g})"


@pytest.mark.parametrize("T,H,I", [(200, 256, 512), (256, 512, 768), (1, 256, 256), (300, 5120, 13824)])
def test_row_mx_mlp_vs_oracle(pkg, dev, T, H, I):
    h, d = _inputs(T, H, I, T + I, dev)
    y = pkg.row_mx_mlp((d["codes"], d["rs"]), d["uc"], d["dc"], d["us"], d["ds"], d["bu"], d["bd"])
    torch.cuda.synchronize()
    assert y.shape == (T, H) and y.dtype == torch.bfloat16
    ref = off.wan_mlp_row_mx_ref(_np(h["codes"]), _np(h["rs"]), _np(h["uc"]), _np(h["us"]), _np(h["bu"]),
                                 _np(h["dc"]), _np(h["ds"]), _np(h["bd"]))
    _check(y.float().cpu().numpy(), ref, f"row_mx_mlp {T}x{H}x{I}")


def test_packed_rows_and_gated_residual(pkg, dev):
    """Packed ``[B, T, H + 4]`` ROW rows as adaln_modulate(quant="row") emits them, and the block's
    closing gated residual fused into the down projection."""
    B, T, H, I = 2, 96, 256, 512
    h, d = _inputs(B * T, H, I, 5, dev)
    packed = torch.empty(B * T, H + 4, dtype=torch.uint8)
    packed[:, :H] = h["codes"].view(torch.uint8)
    packed[:, H:] = h["rs"].view(torch.uint8).reshape(B * T, 4)
    packed = packed.reshape(B, T, H + 4).to(dev)
    g = torch.Generator().manual_seed(6)
    res = (torch.randn(B, T, H, generator=g)).to(torch.bfloat16)
    gate = torch.randn(B, 1, H, generator=g) * 0.5
    y = pkg.row_mx_mlp(packed, d["uc"], d["dc"], d["us"], d["ds"], d["bu"], d["bd"], residual=res.to(dev), gate=gate.to(dev))
    y_plain = pkg.row_mx_mlp(packed, d["uc"], d["dc"], d["us"], d["ds"], d["bu"], d["bd"])
    torch.cuda.synchronize()
    assert y.shape == (B, T, H)
    # the fused residual equals torch's (hidden.float() + ff.float() * gate).type_as(hidden) on the plain output
    expect = (res.float() + y_plain.cpu().float() * gate).to(torch.bfloat16)
    assert torch.equal(y.cpu(), expect)
    ref = off.wan_mlp_row_mx_ref(_np(h["codes"]), _np(h["rs"]), _np(h["uc"]), _np(h["us"]), _np(h["bu"]),
                                 _np(h["dc"]), _np(h["ds"]), _np(h["bd"]))
    _check(y_plain.float().cpu().numpy().reshape(B * T, H), ref, "packed rows")


def test_intermediate_codes_and_scales(pkg, dev):
    T, H, I = 260, 256, 768
    h, d = _inputs(T, H, I, 9, dev)
    lib = import_module("vllm-omni-neuron_b200._lib")
    L = lib.load()
    inter = torch.empty(T, I, dtype=torch.uint8, device=dev)
    sf = torch.empty(L.vomni_mx_packed_scales_bytes(T, I), dtype=torch.uint8, device=dev)
    lib.check(L.vomni_ffn_fp8_up(d["codes"].data_ptr(), d["rs"].data_ptr(), d["uc"].data_ptr(), d["us"].data_ptr(),
                                 d["bu"].data_ptr(), T, H, I, inter.data_ptr(), sf.data_ptr(),
                                 torch.cuda.current_stream().cuda_stream), "up")
    torch.cuda.synchronize()
    codes_ref, su_ref, _ = off.wan_mlp_row_mx_intermediate_ref(_np(h["codes"]), _np(h["rs"]), _np(h["uc"]),
                                                               _np(h["us"]), _np(h["bu"]))
    got_codes = inter.cpu().view(torch.float8_e4m3fn).float().numpy()
    mism = got_codes != codes_ref
    assert mism.mean() < 2e-3, f"{mism.mean():.2e} of the codes differ"
    # de-tile the scale atoms: byte (kb, rb, m0*16 + m1*4 + j) holds row rb*128 + m1*32 + m0, k-block 4*kb + j
    rb_n = (T + 127) // 128
    atoms = sf.cpu().numpy().reshape(I // 128, rb_n, 32, 4, 4)  # [kb, rb, m0, m1, j]
    got_su = atoms.transpose(1, 3, 2, 0, 4).reshape(rb_n * 128, I // 32)[:T]
    assert (got_su != su_ref).mean() < 2e-3
    # pad rows of the last 128-row block carry the identity scale
    assert (atoms.transpose(1, 3, 2, 0, 4).reshape(rb_n * 128, I // 32)[T:] == 127).all()


def test_errors(pkg, dev):
    lib = import_module("vllm-omni-neuron_b200._lib")
    h, d = _inputs(8, 256, 512, 1, dev)
    with pytest.raises(ValueError):
        pkg.row_mx_mlp((d["codes"], d["rs"]), d["dc"], d["uc"], d["us"], d["ds"], None, None)  # swapped weights
    with pytest.raises(TypeError):
        pkg.row_mx_mlp((d["codes"], d["rs"]), d["uc"].float(), d["dc"], d["us"], d["ds"], None, None)
    with pytest.raises(ValueError):
        pkg.row_mx_mlp((d["codes"], d["rs"]), d["uc"], d["dc"], d["us"], d["ds"], None, None, gate=d["ds"])
    # i % 256 != 0 for the up GEMM's output width
    uc = torch.zeros(200, 256, dtype=torch.float8_e4m3fn, device=dev)
    dc = torch.zeros(256, 200, dtype=torch.float8_e4m3fn, device=dev)
    with pytest.raises(lib.VomniError):
        pkg.row_mx_mlp((d["codes"], d["rs"]), uc, dc, torch.ones(200, device=dev), d["ds"], None, None)
