"""GPU parity of the output projection (d-major attention in place) and the fused norm2 gated
residual against the CPU oracle, which is pinned to the reference's ``_wan_o_proj`` (B200 only)."""

import numpy as np
import pytest
import torch

from oracle import adaln as oad
from oracle import oproj as oop

pytestmark = pytest.mark.gpu


def _bf(x, dev):
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(torch.bfloat16).to(dev)


def _one_step(got, ref, pre=None):
    """bf16 results from different fp32 summation orders: the two roundings of bf16(x @ W) may land
    one bf16 step apart, and the bias add rounds again, so allow two steps at the largest magnitude
    involved (the final values and the rounded matmul output `pre`, which the bias can cancel)."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    mag = np.maximum(np.abs(ref), np.abs(got))
    if pre is not None:
        mag = np.maximum(mag, np.abs(np.asarray(pre, np.float64)))
    step = np.exp2(np.floor(np.log2(np.maximum(mag, 2.0 ** -100))) - 7)
    assert (np.abs(got - ref) <= 2 * step * 1.0001 + 1e-30).all(), np.abs(got - ref).max()
    return (got == ref).mean()


def test_golden_reference_outputs(pkg, dev, golden):
    g = golden("wan_o_proj.npz")
    for tag in ("a", "b"):
        y = pkg.wan_o_proj(_bf(g[f"{tag}|active"], dev), _bf(g[f"{tag}|w"], dev), _bf(g[f"{tag}|bias"], dev))
        torch.cuda.synchronize()
        assert _one_step(y.float().cpu().numpy(), g[f"{tag}|y"]) > 0.99


@pytest.mark.parametrize("B,N,S,H", [(1, 4, 1000, 512), (2, 2, 136, 768), (1, 1, 8, 256), (1, 8, 4095, 1024), (1, 2, 64, 160)])
def test_o_proj_vs_oracle(pkg, dev, B, N, S, H):
    rng = np.random.default_rng(B * 1000 + S)
    from oracle.numerics import bf16_round

    active = bf16_round(rng.standard_normal((B, N, 128, S)).astype(np.float32))
    w = bf16_round((0.02 * rng.standard_normal((N * 128, H))).astype(np.float32))
    bias = bf16_round((0.5 * rng.standard_normal((1, H))).astype(np.float32))
    y = pkg.wan_o_proj(_bf(active, dev), _bf(w, dev), _bf(bias, dev))
    torch.cuda.synchronize()
    assert y.shape == (B, S, H)
    ref = oop.wan_o_proj_ref(active, w, bias)
    pre = oop.wan_o_proj_ref(active, w, None)
    assert _one_step(y.float().cpu().numpy(), ref, pre) > 0.98


@pytest.mark.parametrize("gate_kind", ["per_batch", "shared", "none"])
def test_gated_residual_and_norm2(pkg, dev, gate_kind):
    from oracle.numerics import bf16_round

    B, N, S, H = 2, 2, 520, 512
    rng = np.random.default_rng(7)
    active = bf16_round(rng.standard_normal((B, N, 128, S)).astype(np.float32))
    w = bf16_round((0.02 * rng.standard_normal((N * 128, H))).astype(np.float32))
    bias = bf16_round((0.5 * rng.standard_normal((1, H))).astype(np.float32))
    res = bf16_round(rng.standard_normal((B, S, H)).astype(np.float32))
    gate = {"per_batch": (0.3 * rng.standard_normal((B, 1, H))).astype(np.float32),
            "shared": (0.3 * rng.standard_normal((H,))).astype(np.float32), "none": None}[gate_kind]
    n2w = bf16_round((1 + 0.1 * rng.standard_normal(H)).astype(np.float32))
    n2b = bf16_round((0.1 * rng.standard_normal(H)).astype(np.float32))
    tg = torch.from_numpy(gate).to(dev) if gate is not None else None
    t, norm_h = pkg.attn_out_norm2(_bf(active, dev), _bf(w, dev), _bf(bias, dev), _bf(res, dev), tg, _bf(n2w, dev),
                                   _bf(n2b, dev), eps=1e-6, norm_type="layer_norm", quant="none")
    torch.cuda.synchronize()
    y_ref = oop.wan_o_proj_ref(active, w, bias)
    # the residual step on the kernel's own projection values must be exact; the projection itself
    # is checked against the oracle above
    y_gpu = pkg.wan_o_proj(_bf(active, dev), _bf(w, dev), _bf(bias, dev)).float().cpu().numpy()
    np.testing.assert_array_equal(t.float().cpu().numpy(), oop.gated_residual_ref(y_gpu, res, gate))
    _one_step(y_gpu, y_ref, oop.wan_o_proj_ref(active, w, None))
    # norm2 over t, as the reference's adaln_modulate(attn1_out, ..., residual=, gate=) returns it
    t_np = t.float().cpu().numpy()
    ref_norm = oad.adaln_modulate_oracle(t_np, n2w, n2b, eps=1e-6, norm_type="layer_norm", quant="none")
    got = norm_h.float().cpu().numpy()
    assert np.abs(got - ref_norm).max() <= 0.02 * max(1.0, np.abs(ref_norm).max())


def test_errors(pkg, dev):
    a = torch.zeros(1, 2, 128, 64, dtype=torch.bfloat16, device=dev)
    with pytest.raises(ValueError):
        pkg.wan_o_proj(a, torch.zeros(128, 256, dtype=torch.bfloat16, device=dev), None)  # N*D mismatch
    lib = pytest.importorskip("importlib").import_module("vllm-omni-neuron_b200._lib")
    with pytest.raises(lib.VomniError):
        pkg.wan_o_proj(a, torch.zeros(256, 200, dtype=torch.bfloat16, device=dev), None)  # H % 32


def _fp8_oproj_case(pkg, dev, B, N, S, H, seed):
    g = torch.Generator().manual_seed(seed)
    K = N * 128
    active = (torch.randn(B, N, 128, S, generator=g) * 0.5).to(torch.bfloat16)
    active[:, :, :, ::7] *= 30  # tokens with larger magnitudes: per-token scales differ
    w = torch.randn(K, H, generator=g) * 0.02
    bias = (torch.randn(H, generator=g) * 0.1).to(torch.bfloat16)
    codes, chan = pkg.quantize_qkv_weight(w.to(dev), H, 0)  # [H, K] e4m3, one per-tensor scale
    return active, codes, chan, bias


@pytest.mark.parametrize("B,N,S,H", [(1, 4, 1000, 512), (2, 2, 136, 768), (1, 1, 9, 256)])
def test_row_mx_o_proj_vs_oracle(pkg, dev, B, N, S, H):
    """FP8 o-projection (row_mx_kernels.py:114-138): the per-token ROW codes and scales of the d-major
    activation bit-exact against the oracle's ROW quantiser, and the projection against the oracle
    on the same codes (identical FP8 operands: fp32 accumulation order and the bf16 store differ)."""
    from importlib import import_module

    from oracle.numerics import e4m3fn_from_bits

    lib = import_module("vllm-omni-neuron_b200._lib")
    active, codes, chan, bias = _fp8_oproj_case(pkg, dev, B, N, S, H, seed=40 + S)
    y = pkg.row_mx_o_proj(active.to(dev), codes, chan.reshape(1, -1).expand(128, -1), bias.reshape(1, -1).to(dev))
    # the quantiser alone, on the 8-padded token count
    s_pad = -(-S // 8) * 8
    act = torch.nn.functional.pad(active, (0, s_pad - S)).to(dev).contiguous()
    qc = torch.empty(B * s_pad, N * 128, dtype=torch.float8_e4m3fn, device=dev)
    qs = torch.empty(B * s_pad, dtype=torch.float32, device=dev)
    lib.check(lib.load().vomni_oproj_rowquant(act.data_ptr(), B, N * 128, s_pad, qc.data_ptr(), qs.data_ptr(),
                                              torch.cuda.current_stream().cuda_stream), "rowquant")
    torch.cuda.synchronize()
    assert tuple(y.shape) == (B, S, H)
    wc = e4m3fn_from_bits(codes.view(torch.uint8).cpu().numpy())  # [H, K]
    ref, (ref_codes, ref_scale) = oop.row_mx_o_proj_ref(active.float().numpy(), wc, chan.cpu().numpy(),
                                                        bias.float().numpy())
    got_codes = e4m3fn_from_bits(qc.view(torch.uint8).cpu().numpy()).reshape(B, s_pad, -1)[:, :S].reshape(B * S, -1)
    got_scale = qs.cpu().numpy().reshape(B, s_pad)[:, :S].reshape(-1)
    assert np.array_equal(got_scale, ref_scale)
    assert np.array_equal(got_codes, ref_codes)
    got = y.float().cpu().numpy()
    cos = (got * ref).sum() / np.sqrt((got * got).sum() * (ref * ref).sum())
    assert cos >= 0.99999 and np.abs(got - ref).max() <= 1e-2 * max(1.0, np.abs(ref).max())
    assert (np.abs(got - ref) <= np.abs(ref) * 2 ** -7 + 1e-3).mean() > 0.999
    assert lib.device_status() == 0


def test_row_mx_o_proj_layouts_and_leaf(pkg, dev):
    """The reference's [N*D//4, H, 4] weight pack gives the same result as [H, N*D] codes, and the
    FP8 self-attention leaf with o-projection weights returns row_mx_o_proj of its attention."""
    B, N, S, H = 1, 2, 256, 512
    active, codes, chan, bias = _fp8_oproj_case(pkg, dev, B, N, S, H, seed=3)
    K = N * 128
    w3 = codes.view(torch.uint8).t().reshape(K // 4, 4, H).permute(0, 2, 1).contiguous().view(torch.float8_e4m3fn)
    a = pkg.row_mx_o_proj(active.to(dev), codes, chan, bias.to(dev))
    b = pkg.row_mx_o_proj(active.to(dev), w3, chan.reshape(1, -1).expand(128, -1), bias.reshape(1, -1).to(dev))
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    # leaf: FP8 QKV -> attention -> FP8 o-projection
    g = torch.Generator().manual_seed(4)
    Hid = 256
    hidden = torch.randn(B, S, Hid, generator=g).to(torch.bfloat16).to(dev)
    wqkv = (torch.randn(Hid, 3 * K, generator=g) * 0.02).to(dev)
    wq, qchan = pkg.quantize_qkv_weight(wqkv, K, K)
    packed = pkg.adaln_modulate(hidden, None, None, eps=1e-6, norm_type="layer_norm", quant="row")
    attn = pkg.wan_self_attention_fp8(packed, wq, qchan, None, None, None, num_heads=N)
    wo = torch.randn(K, Hid, generator=g) * 0.02
    oc, ochan = pkg.quantize_qkv_weight(wo.to(dev), Hid, 0)
    out = pkg.wan_self_attention_fp8(packed, wq, qchan, None, None, None, num_heads=N, o_proj_weight=oc,
                                     o_proj_w_scale=ochan, o_proj_bias=None)
    torch.cuda.synchronize()
    assert tuple(out.shape) == (B, S, Hid)
    assert torch.equal(out, pkg.row_mx_o_proj(attn, oc, ochan, None))
