"""GPU parity of the fused adaLN + FP8 quant kernel against the CPU oracle and the reference's golden
vectors (B200 only)."""

import numpy as np
import pytest
import torch

from oracle import adaln as oad
from oracle.numerics import e4m3fn_from_bits

pytestmark = pytest.mark.gpu


def _bf(x, dev):
    return torch.from_numpy(np.asarray(x, np.float32)).to(torch.bfloat16).to(dev)


def _rand(shape, seed, scale=1.0):
    from oracle.numerics import bf16_round

    return bf16_round(np.random.default_rng(seed).standard_normal(shape).astype(np.float32) * scale)


def _check_bf16(got, ref, what):
    d = np.abs(got - ref)
    tol = np.abs(ref) * 2 ** -7 + 1e-5
    assert (d <= tol).all(), f"{what}: max violation {(d - tol).max()}"
    assert (d == 0).mean() > 0.98, f"{what}: only {(d == 0).mean():.4f} exact"


def _check_codes(codes_got, scale_got, codes_ref, scale_ref, what):
    """Codes may differ only where fp32 rounding order moves a value across an fp8 rounding boundary:
    one code step at most, and rarely."""
    np.testing.assert_allclose(scale_got, scale_ref, rtol=1e-5, err_msg=what)
    dq_g = e4m3fn_from_bits(codes_got).astype(np.float64)
    dq_r = e4m3fn_from_bits(codes_ref).astype(np.float64)
    same = codes_got == codes_ref
    assert same.mean() >= 0.995, f"{what}: only {same.mean():.5f} codes equal"
    # one fp8 step at that magnitude: 2^(floor(log2|x|) - 3)
    mag = np.maximum(np.abs(dq_r), 2.0 ** -6)
    step = np.exp2(np.floor(np.log2(mag)) - 3)
    assert (np.abs(dq_g - dq_r) <= step * 1.0001).all(), what


CASES = [
    ((2, 37, 256), "per_batch"),
    ((77, 5120), "shared"),
    ((1, 130, 128), "shared"),
    ((3, 16384), "shared"),
    ((5, 1000), "shared"),
]


@pytest.mark.parametrize("shape,modk", CASES)
@pytest.mark.parametrize("norm", ["layer_norm", "rms_norm", "none"])
@pytest.mark.parametrize("res_mode", ["plain", "gated"])
def test_adaln_vs_oracle(pkg, dev, shape, modk, norm, res_mode):
    H = shape[-1]
    B = shape[0] if len(shape) == 3 else 1
    hidden = _rand(shape, 1, 1.0)
    if modk == "per_batch":
        mul = 1 + _rand((B, 1, H), 2, 0.1)
        add = _rand((B, 1, H), 3, 0.1)
        gate = np.random.default_rng(4).standard_normal((B, 1, H)).astype(np.float32) * 0.5
    else:
        mul = 1 + _rand((H,), 2, 0.1)
        add = _rand((H,), 3, 0.1)
        gate = np.random.default_rng(4).standard_normal((H,)).astype(np.float32) * 0.5
    residual = _rand(shape, 5, 1.0) if res_mode != "plain" else None
    g_gate = gate if res_mode == "gated" else None
    kw = dict(eps=1e-6, norm_type=norm)
    for quant in ("none", "row", "mx32"):
        if quant == "mx32" and H % 32:
            with pytest.raises(ValueError):
                pkg.adaln_modulate(_bf(hidden, dev), _bf(mul, dev), _bf(add, dev), quant=quant, **kw)
            continue
        args = dict(kw, quant=quant)
        targs = dict(args)
        if residual is not None:
            targs["residual"] = _bf(residual, dev)
            targs["gate"] = torch.from_numpy(g_gate).to(dev) if g_gate is not None else None
            args["residual"] = residual
            args["gate"] = g_gate
        got = pkg.adaln_modulate(_bf(hidden, dev), _bf(mul, dev), _bf(add, dev), **targs)
        ref = oad.adaln_modulate_oracle(hidden, mul, add, **args)
        torch.cuda.synchronize()
        if residual is not None:
            np.testing.assert_array_equal(got[0].float().cpu().numpy(), ref[0])
            got, ref = got[1], ref[1]
        what = f"{shape} {norm} {res_mode} {quant}"
        if quant == "none":
            _check_bf16(got.float().cpu().numpy(), ref, what)
        elif quant == "row":
            g = got.view(torch.uint8).cpu().numpy()
            assert g.shape[-1] == H + 4
            sc_g = g[..., H:].copy().view(np.float32)[..., 0]
            sc_r = ref[..., H:].copy().view(np.float32)[..., 0]
            _check_codes(g[..., :H], sc_g, ref[..., :H], sc_r, what)
        else:
            codes, scales = got
            np.testing.assert_array_equal(scales.cpu().numpy(), ref[1], err_msg=what)
            _check_codes(codes.view(torch.uint8).cpu().numpy(), 1.0, ref[0], 1.0, what)


def test_row_split_layout_matches_packed(pkg, dev):
    hidden = _bf(_rand((64, 512), 9), dev)
    mul = _bf(1 + _rand((512,), 10, 0.1), dev)
    packed = pkg.adaln_modulate(hidden, mul, None, eps=1e-6, quant="row")
    codes, scales = pkg.adaln_modulate(hidden, mul, None, eps=1e-6, quant="row", row_layout="split")
    p = packed.view(torch.uint8)
    assert torch.equal(p[:, :512], codes.view(torch.uint8))
    assert torch.equal(p[:, 512:].contiguous().view(torch.float32).squeeze(-1), scales)


def test_adt_golden(pkg, dev, golden):
    """The reference's own ground truth adaln_quant_torch_ref on its golden inputs (plain cases: the
    residual cases differ by the bridge's bf16 rounding of the residual sum, tested above)."""
    g = golden("adaln_ref.npz")
    for key in g["cases"]:
        key = str(key)
        norm, quant, res_mode, ocp = key.split("|")
        if res_mode != "plain" or quant == "mx":
            continue
        out = pkg.adaln_modulate(_bf(g["hidden"], dev), _bf(g["mul"], dev), _bf(g["add"], dev), eps=1e-6,
                                 norm_type=norm, quant=quant, ocp=bool(int(ocp)))
        torch.cuda.synchronize()
        if quant == "none":
            _check_bf16(out.float().cpu().numpy(), oad.bf16_round(g[f"{key}|y"]), key)
        else:
            u = out.view(torch.uint8).cpu().numpy()
            H = g["hidden"].shape[-1]
            sc = u[:, H:].copy().view(np.float32)[:, 0]
            from oracle.numerics import e4m3fn_bits

            _check_codes(u[:, :H], sc, e4m3fn_bits(g[f"{key}|quant"]), g[f"{key}|dequant_scale"][:, 0], key)
    # MX-32 against the reference's _mx_dequant
    for norm in ("layer_norm", "rms_norm", "none"):
        key = f"{norm}|mx|plain|1"
        codes, scales = pkg.adaln_modulate(_bf(g["hidden"], dev), _bf(g["mul"], dev), _bf(g["add"], dev), eps=1e-6,
                                           norm_type=norm, quant="mx32")
        c = e4m3fn_from_bits(codes.view(torch.uint8).cpu().numpy()).astype(np.float64)
        f = np.exp2(scales.cpu().numpy().astype(np.float64) - 127.0)
        deq = (c.reshape(c.shape[0], -1, 32) * f[..., None]).reshape(c.shape)
        ref = g[f"{key}|dequant"].astype(np.float64)
        rel = np.abs(deq - ref) / np.maximum(np.abs(ref), 1e-3)
        assert (deq == ref).mean() > 0.99 and rel.max() <= 0.13, key


def test_errors(pkg, dev):
    h = _bf(_rand((4, 64), 0), dev)
    with pytest.raises(NotImplementedError):
        pkg.adaln_modulate(h, quant="mx", eps=1e-6)
    with pytest.raises(ValueError):
        pkg.adaln_modulate(h, gate=torch.ones(64, device=dev), eps=1e-6)
    with pytest.raises(ValueError):
        pkg.adaln_modulate(h, quant="bogus", eps=1e-6)
