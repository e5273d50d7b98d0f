"""Pin the CPU oracle against golden vectors produced by the reference's own code
(tests/golden/make_golden.py). CPU only."""

import numpy as np
import pytest

from oracle import adaln as oad
from oracle import attention as oat
from oracle import rope as orope
from oracle.numerics import bf16_round, e4m3fn_bits, e4m3fn_from_bits, e4m3fn_round


def test_e4m3fn_round_matches_torch():
    import torch

    rng = np.random.default_rng(0)
    x = np.concatenate([
        rng.standard_normal(20000).astype(np.float32) * 100,
        rng.standard_normal(2000).astype(np.float32) * 1e-3,
        np.array([0.0, -0.0, 448.0, -448.0, 2.0 ** -9, 2.0 ** -10, 3 * 2.0 ** -10, 0.5, 17.0, 18.0, 19.0], np.float32),
    ])
    x = np.clip(x, -448, 448)
    ref = torch.from_numpy(x).to(torch.float8_e4m3fn)
    assert np.array_equal(e4m3fn_round(x), ref.float().numpy())
    assert np.array_equal(e4m3fn_bits(x), ref.view(torch.uint8).numpy())
    allb = np.arange(256, dtype=np.uint8)
    dec = e4m3fn_from_bits(allb)
    tb = torch.from_numpy(allb).view(torch.float8_e4m3fn).float().numpy()
    assert np.array_equal(np.isnan(dec), np.isnan(tb))
    ok = ~np.isnan(tb)
    assert np.array_equal(dec[ok], tb[ok])


def test_bf16_round_matches_torch():
    import torch

    x = np.random.default_rng(1).standard_normal(50000).astype(np.float32) * 37
    assert np.array_equal(bf16_round(x), torch.from_numpy(x).to(torch.bfloat16).float().numpy())


def test_adaln_ref_pinned(golden):
    g = golden("adaln_ref.npz")
    for key in g["cases"]:
        key = str(key)
        norm, quant, res_mode, ocp = key.split("|")
        kw = dict(norm_type=norm, quant=quant, eps=1e-6, ocp=bool(int(ocp)))
        if res_mode != "plain":
            kw["residual"] = g["residual"]
        if res_mode == "gated":
            kw["gate"] = g["gate"]
        r = oad.adaln_quant_ref(g["hidden"], g["mul"], g["add"], **kw)
        # fp32 y: same numpy op order as the reference -> tight
        np.testing.assert_allclose(r["y"], g[f"{key}|y"], rtol=2e-6, atol=2e-6, err_msg=key)
        if quant == "row":
            np.testing.assert_array_equal(r["quant"], g[f"{key}|quant"], err_msg=key)
            np.testing.assert_array_equal(r["dequant_scale"], g[f"{key}|dequant_scale"], err_msg=key)
            np.testing.assert_array_equal(r["dequant"], g[f"{key}|dequant"], err_msg=key)
        if quant == "mx":
            np.testing.assert_array_equal(r["dequant"], g[f"{key}|dequant"], err_msg=key)
        if res_mode != "plain":
            np.testing.assert_array_equal(r["residual_out"], g[f"{res_mode}|residual_out"], err_msg=key)


def test_eager_adaln_pinned(golden):
    """adaln_modulate_oracle (quant='none') vs the reference's unfused fallback _eager_adaln."""
    g = golden("eager_adaln.npz")
    for norm in ("layer_norm", "rms_norm", "none"):
        o = oad.adaln_modulate_oracle(g["hidden"], g["mul"], g["add"], eps=1e-6, norm_type=norm)
        d = np.abs(o - g[f"{norm}|plain|out"])
        # bf16 outputs: equal up to one bf16 ulp from fp32 reduction order
        assert (d <= np.abs(g[f"{norm}|plain|out"]) * 2 ** -7 + 1e-6).all(), norm
        assert (d == 0).mean() > 0.97
        ro, o = oad.adaln_modulate_oracle(
            g["hidden"], g["mul"], g["add"], eps=1e-6, norm_type=norm, residual=g["residual"], gate=g["gate"]
        )
        np.testing.assert_array_equal(ro, g[f"{norm}|gated|residual_out"])
        d = np.abs(o - g[f"{norm}|gated|out"])
        assert (d <= np.abs(g[f"{norm}|gated|out"]) * 2 ** -7 + 1e-6).all(), norm


def test_torch_attend_pinned(golden):
    g = golden("torch_attend.npz")
    for tag in ("a", "b"):
        o = oat.torch_attend(g[f"{tag}|q"], g[f"{tag}|k"], g[f"{tag}|v"], float(g[f"{tag}|scale"]))
        ref = g[f"{tag}|o"]
        d = np.abs(o - ref)
        assert (d <= np.abs(ref) * 2 ** -7 + 1e-5).all(), tag
        assert (d == 0).mean() > 0.95, tag


@pytest.mark.parametrize("tag", ["a", "b"])
def test_const_max_matches_exact_attention(golden, tag):
    """The reference's own validation rule for the ring kernel (compare against exact attention):
    the const-max restatement, at 1 and 2 ring ranks, is within the north-star tolerance of the
    pinned exact attention."""
    g = golden("torch_attend.npz")
    q, k, v = g[f"{tag}|q"], g[f"{tag}|k"], g[f"{tag}|v"]
    if q.shape[2] != k.shape[2]:
        pytest.skip("ring needs S_q == S_k per rank")
    ref = g[f"{tag}|o"]
    tok = lambda x: np.ascontiguousarray(np.transpose(x, (0, 2, 1, 3)))  # [B,N,S,D] -> [B,S,N,D]
    for n in (1, 2):
        s = q.shape[2] // n
        qs = [tok(q)[:, i * s:(i + 1) * s] for i in range(n)]
        ks = [tok(k)[:, i * s:(i + 1) * s] for i in range(n)]
        vs = [tok(v)[:, i * s:(i + 1) * s] for i in range(n)]
        outs = oat.const_max_ring_attention(qs, ks, vs, float(g[f"{tag}|scale"]))
        o = np.concatenate(outs, axis=2)
        cos = (o * ref).sum() / np.sqrt((o * o).sum() * (ref * ref).sum())
        assert cos >= 0.9999, (n, cos)
        assert np.abs(o - ref).max() <= 2e-2


def test_rope_pinned(golden):
    g = golden("rope_norm.npz")
    cos, sin = orope.rotary_freqs(128, (1, 2, 2), 1024, tuple(g["latent_fhw"] * np.array([1, 1, 1])))
    np.testing.assert_array_equal(cos, g["cos"])
    np.testing.assert_array_equal(sin, g["sin"])
    xr = orope.apply_rotary_emb_wan(g["x"], g["cos"], g["sin"])
    np.testing.assert_array_equal(xr, g["x_rope"])
    c, s = orope.rotate_half_caches(g["cos"], g["sin"])
    np.testing.assert_array_equal(c, g["cos_rh"])
    np.testing.assert_array_equal(s, g["sin_rh"])
    np.testing.assert_array_equal(orope.deinterleave_qk_columns(g["w"], 256, 256, 128), g["w_deint"])
    np.testing.assert_array_equal(orope.deinterleave_gamma_row(g["gamma"], 128), g["gamma_deint"])
    yn = orope.distributed_rms_norm(g["norm_x"], g["norm_w"], 1e-6)
    d = np.abs(yn - g["norm_y"])
    assert (d <= np.abs(g["norm_y"]) * 2 ** -7 + 1e-6).all()
    assert (d == 0).mean() > 0.97


def test_rotate_half_equals_interleaved_rope(golden):
    """The de-interleave identity the FP8 leaf relies on (row_mx_loaders.py:26-39): rotate-half
    RoPE on de-interleaved lanes == interleaved RoPE on the original lanes, permuted."""
    g = golden("rope_norm.npz")
    x = g["x"]  # [1,S,2,128]
    perm = orope.deinterleave_perm(128)
    ref = orope.apply_rotary_emb_wan(x, g["cos"], g["sin"])[..., perm]
    xd = x[..., perm]
    c, s = g["cos_rh"], g["sin_rh"]
    lo, hi = xd[..., :64], xd[..., 64:]
    out = np.concatenate([lo * c[..., :64] - hi * s[..., :64], hi * c[..., 64:] + lo * s[..., 64:]], axis=-1)
    np.testing.assert_array_equal(bf16_round(out), ref)


def test_oproj_oracle_vs_reference_golden(golden):
    """The o-projection restatement reproduces ``_wan_o_proj``'s own outputs."""
    from oracle import oproj as oop

    g = golden("wan_o_proj.npz")
    for tag in ("a", "b"):
        y = oop.wan_o_proj_ref(g[f"{tag}|active"], g[f"{tag}|w"], g[f"{tag}|bias"])
        ref = g[f"{tag}|y"]
        # fp32 accumulation order differs from torch's CPU matmul: at most one bf16 step apart
        step = np.exp2(np.floor(np.log2(np.maximum(np.abs(ref), 2.0 ** -100))) - 7)
        assert (np.abs(y - ref) <= step * 1.0001).all(), tag
        assert (y == ref).mean() > 0.97, tag


def test_mlp_oracle_vs_reference_golden(golden):
    """The FFN restatement reproduces ``_wan_mlp``'s own outputs (up to one bf16 step where the
    fp32 tanh of the two implementations rounds differently)."""
    from oracle import ffn

    g = golden("wan_mlp.npz")
    for tag in ("a", "b"):
        y = ffn.wan_mlp_ref(g[f"{tag}|x"], g[f"{tag}|wu"], g[f"{tag}|wd"], g[f"{tag}|bu"], g[f"{tag}|bd"])
        ref = g[f"{tag}|y"]
        # a one-step difference of a GELU output moves the down projection slightly; after the
        # bias add that can land one or two bf16 steps away where the sum cancels
        step = np.exp2(np.floor(np.log2(np.maximum(np.maximum(np.abs(ref), np.abs(y)), 2.0 ** -100))) - 7)
        assert (np.abs(y - ref) <= 2 * step * 1.0001 + 2e-3).all(), tag
        assert (y == ref).mean() > 0.999, tag


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
@pytest.mark.parametrize("scale", [5.0, 3.5, 1.0, 7.3])
def test_cfg_combine_matches_torch_eager(dtype, scale):
    """The restated CFG combine equals the reference's own expression
    (``negative + true_cfg_scale * (positive - negative)``, cfg_parallel.py:71) run by torch eager."""
    import torch

    from oracle import cfg as ocfg

    g = torch.Generator().manual_seed(7)
    td = torch.bfloat16 if dtype == "bf16" else torch.float32
    # latent-shaped branch outputs [B, C, T, H, W] plus a ragged flat tail
    for shape in ((1, 16, 3, 12, 20), (1001,)):
        pos = torch.randn(shape, generator=g).to(td)
        neg = (torch.randn(shape, generator=g) * 0.7).to(td)
        ref = (neg + scale * (pos - neg)).float().numpy()
        got = ocfg.cfg_gather_combine_ref([pos.float().numpy(), neg.float().numpy()], scale, dtype == "bf16")
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_mlp_row_mx_oracle_vs_reference_golden(golden):
    """The ROW_MX MLP restatement equals the reference's own ``_mlp_ref_standard`` (ROW_MX, CTE,
    GELU-tanh; mlp_torch.py:401-600) bit for bit, and the MX-32 quantiser equals its ``_mx_quantize``
    (:252-271) on codes and dequantised values (fixtures: ``make_golden.py mlp_row_mx``)."""
    from oracle import adaln as oad
    from oracle import ffn as off

    g = golden("mlp_row_mx.npz")
    for tag in ("a", "b"):
        codes = e4m3fn_from_bits(g[f"{tag}|codes"])
        uc = e4m3fn_from_bits(g[f"{tag}|uc"])  # [H, I] (x @ W layout)
        dc = e4m3fn_from_bits(g[f"{tag}|dc"])  # [I, H]
        H, I = uc.shape
        y = off.wan_mlp_row_mx_ref(codes, g[f"{tag}|rs"], uc.T, np.full(I, g[f"{tag}|su"], np.float32), g[f"{tag}|bu"],
                                   dc.T, np.full(H, g[f"{tag}|sd"], np.float32), g[f"{tag}|bd"])
        assert np.array_equal(y.view(np.uint32), g[f"{tag}|y"].astype(np.float32).view(np.uint32)), tag
    codes, _, deq = oad.mx_quantize(g["mxq|x"])
    assert np.array_equal(codes, g["mxq|codes"])
    ref_deq = (g["mxq|codes"].astype(np.float64) * g["mxq|scale"]).astype(np.float32)
    assert np.array_equal(deq, ref_deq)


def test_qkv_row_mx_oracle_vs_reference_golden(golden):
    """The ROW_MX QKV restatement against the reference's own ROW_MX dequant-matmul, executed from its
    source: ``_mlp_ref_standard``'s up-projection ``(Xq * row_scale) @ (Wq * w_scale) + bias``
    (mlp_torch.py:470-497, 575-578; fixture ``make_golden.py qkv_row_mx``) on per-tensor Q/K/V scaled
    e4m3 weights. The oracle scales after the matmul, as the kernel (``_dequant_row_mx``,
    qkv_cte.py:3996-4021) does; the two orders differ only by fp32 reassociation, so the fp32 values
    agree to 2^-20 of the row's magnitude and the bf16 stores are equal except where that noise straddles a
    bf16 rounding boundary (at most 0.1 % of the elements, apart by at most the noise plus one bf16
    step)."""
    from oracle import qkv as oq

    g = golden("qkv_row_mx.npz")
    for tag in ("a", "b"):
        codes = g[f"{tag}|codes"]
        T, H = codes.shape
        packed = np.concatenate([codes, g[f"{tag}|rs"].astype(np.float32).reshape(-1, 1).view(np.uint8)], axis=1)
        wc = e4m3fn_from_bits(g[f"{tag}|wc"])  # [H, I]
        cs, bias, up = g[f"{tag}|cs"], g[f"{tag}|bias"], g[f"{tag}|up"]
        # the oracle's fp32 pre-store values
        xc, rs = oq.unpack_row(packed)
        acc = (xc @ wc) * rs[:, None] * cs[None, :] + bias[None, :]
        scale = np.abs(up).max(axis=1, keepdims=True)
        assert (np.abs(acc - up) <= scale * 2.0 ** -20).all(), tag
        y = oq.row_mx_qkv_ref(packed, wc, cs, bias)
        ref = bf16_round(up)
        diff = y != ref
        assert diff.mean() <= 1e-3, (tag, diff.mean())
        # one bf16 step is at most |x| * 2^-7; the fp32 noise is bounded per row
        tol = np.abs(ref) * 2.0 ** -7 + np.broadcast_to(scale, ref.shape) * 2.0 ** -20
        assert (np.abs(y[diff] - ref[diff]) <= tol[diff]).all(), tag
