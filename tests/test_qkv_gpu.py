"""GPU parity of the FP8 QKV projection (+ across-heads RMS norm + rotate-half RoPE) against the CPU
oracle on identical FP8 codes, and against the reference's bf16 path through the de-interleave
identity (B200 only)."""

import math

import numpy as np
import pytest
import torch

from oracle import qkv as oq
from oracle import rope as orope
from oracle.numerics import bf16_round, e4m3fn_from_bits

pytestmark = pytest.mark.gpu


def _cmp(got, ref, cos_min, abs_max, what):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    cos = (got * ref).sum() / math.sqrt((got * got).sum() * (ref * ref).sum())
    mx = np.abs(got - ref).max()
    assert cos >= cos_min and mx <= abs_max, f"{what}: cos={cos:.7f} maxabs={mx:.4g}"


def _setup(T, H, heads, dev, seed=0):
    g = torch.Generator().manual_seed(seed)
    I = 3 * heads * 128
    hidden = torch.randn(T, H, generator=g).to(torch.bfloat16)
    w = torch.randn(H, I, generator=g) * 0.02
    bias = (torch.randn(I, generator=g) * 0.1).to(torch.bfloat16)
    return hidden.to(dev), w.to(dev), bias.to(dev), I


@pytest.mark.parametrize("T,H,heads", [(300, 512, 2), (129, 1024, 4), (1, 512, 2), (1000, 1024, 2)])
def test_gemm_vs_oracle(pkg, dev, T, H, heads):
    hidden, w, bias, I = _setup(T, H, heads, dev)
    packed = pkg.adaln_modulate(hidden, None, None, eps=1e-6, norm_type="none", quant="row")
    codes, chan = pkg.quantize_qkv_weight(w, heads * 128, heads * 128)
    y = pkg.row_mx_qkv_proj(packed, codes, chan.reshape(1, -1), bias.reshape(1, -1), num_heads=heads, head_dim=128,
                            num_kv_heads=heads)
    torch.cuda.synchronize()
    wc = e4m3fn_from_bits(codes.view(torch.uint8).cpu().numpy()).T  # [H, I]
    ref = oq.row_mx_qkv_ref(packed.view(torch.uint8).cpu().numpy(), wc, chan.cpu().numpy(), bias.float().cpu().numpy())
    got = y.float().cpu().numpy()
    # identical FP8 codes: only fp32 accumulation order and the bf16 store differ
    _cmp(got, ref, 0.99999, 1e-2 * max(1.0, np.abs(ref).max()), f"gemm {T}x{H}x{I}")
    assert (np.abs(got - ref) <= np.abs(ref) * 2 ** -7 + 1e-3).mean() > 0.999


@pytest.mark.parametrize("T,H,heads", [(300, 512, 2), (257, 1024, 4)])
def test_norm_rope_epilogue_vs_oracle(pkg, dev, T, H, heads):
    hidden, w, bias, I = _setup(T, H, heads, dev, seed=1)
    g = torch.Generator().manual_seed(5)
    gq = (1 + 0.1 * torch.randn(heads * 128, generator=g)).to(torch.bfloat16).to(dev)
    gk = (1 + 0.1 * torch.randn(heads * 128, generator=g)).to(torch.bfloat16).to(dev)
    rope = pytest.importorskip("importlib").import_module("vllm-omni-neuron_b200.rope")
    cos, sin = rope.wan_rotary_freqs(128, (1, 2, 2), 1024, (3, 20, 40), device=dev)  # 600 positions
    cos_rh, sin_rh = rope.rope_rotate_half_caches(cos[:, :T], sin[:, :T])
    codes, scales = pkg.adaln_modulate(hidden, None, None, eps=1e-6, norm_type="layer_norm", quant="row", row_layout="split")
    wq, chan = pkg.quantize_qkv_weight(w, heads * 128, heads * 128)
    y = pkg.row_mx_qkv_proj((codes, scales), wq, chan, bias, num_heads=heads, head_dim=128, num_kv_heads=heads,
                            fused_rope=True, cos_cache=cos_rh.reshape(1, T, 128), sin_cache=sin_rh.reshape(1, T, 128),
                            qk_norm_pre_rope=True, qk_norm_pre_rope_q_gamma=gq, qk_norm_pre_rope_k_gamma=gk)
    torch.cuda.synchronize()
    packed_np = np.concatenate([codes.view(torch.uint8).cpu().numpy(),
                                scales.cpu().numpy().reshape(-1, 1).view(np.uint8)], axis=1)
    wc = e4m3fn_from_bits(wq.view(torch.uint8).cpu().numpy()).T
    ref = oq.row_mx_qkv_ref(packed_np, wc, chan.cpu().numpy(), bias.float().cpu().numpy(), num_heads=heads, head_dim=128,
                            num_kv_heads=heads, gamma_q=gq.float().cpu().numpy(), gamma_k=gk.float().cpu().numpy(),
                            cos=cos_rh.reshape(T, 128).cpu().numpy(), sin=sin_rh.reshape(T, 128).cpu().numpy(), eps=1e-6)
    _cmp(y.float().cpu().numpy(), ref, 0.99999, 3e-2, f"epilogue {T}x{H}")


def test_layouts_agree(pkg, dev):
    """packed [T, H+4] input == split (codes, scales) input; [H//4, I, 4] weight == [I, H] weight."""
    T, H, heads = 200, 512, 2
    hidden, w, bias, I = _setup(T, H, heads, dev, seed=2)
    packed = pkg.adaln_modulate(hidden, None, None, eps=1e-6, quant="row")
    split = pkg.adaln_modulate(hidden, None, None, eps=1e-6, quant="row", row_layout="split")
    wq, chan = pkg.quantize_qkv_weight(w, heads * 128, heads * 128)
    w3 = wq.view(torch.uint8).t().reshape(H // 4, 4, I).permute(0, 2, 1).contiguous().view(torch.float8_e4m3fn)
    assert torch.equal(pkg.repack_mx_contiguous(w3).view(torch.uint8), wq.view(torch.uint8))
    kw = dict(num_heads=heads, head_dim=128, num_kv_heads=heads)
    a = pkg.row_mx_qkv_proj(packed, wq, chan, bias, **kw)
    b = pkg.row_mx_qkv_proj(split, wq, chan, bias, **kw)
    c = pkg.row_mx_qkv_proj(packed, w3, chan, bias, **kw)
    torch.cuda.synchronize()
    assert torch.equal(a, b) and torch.equal(a, c)


def test_fp8_leaf_vs_bf16_reference_path(pkg, dev):
    """The whole FP8 leaf (adaLN row quant -> FP8 QKV with de-interleaved Q/K weights, across-heads
    norm, rotate-half RoPE) against the reference's bf16 path (matmul + DistributedRMSNorm +
    interleaved RoPE, wan2_2_transformer.py:1097-1114), permuted by the de-interleave (the FP8 leaf
    emits Q/K lanes in [even | odd] order; Q.K^T is unchanged). Differences = FP8 quantisation error."""
    T, H, heads = 600, 1024, 2
    rope = pytest.importorskip("importlib").import_module("vllm-omni-neuron_b200.rope")
    hidden, w, bias, I = _setup(T, H, heads, dev, seed=3)
    qd = heads * 128
    cos, sin = rope.wan_rotary_freqs(128, (1, 2, 2), 1024, (3, 20, 40), device=dev)
    # bf16 reference path on the (un-quantised) modulated hidden
    xm = pkg.adaln_modulate(hidden, None, None, eps=1e-6, norm_type="layer_norm")
    qkv = (xm.float() @ w.to(torch.bfloat16).float() + bias.float()).to(torch.bfloat16)
    rms = lambda x: (x.float() / torch.sqrt((x.float() ** 2).mean(-1, keepdim=True) + 1e-6)).to(torch.bfloat16)
    q = rope.apply_rotary_emb_wan(rms(qkv[:, :qd]).reshape(1, T, heads, 128), cos, sin)
    k = rope.apply_rotary_emb_wan(rms(qkv[:, qd:2 * qd]).reshape(1, T, heads, 128), cos, sin)
    perm = rope.deinterleave_perm(128).to(dev)
    # FP8 leaf with de-interleaved weights / bias and rotate-half caches
    wd = rope.deinterleave_qk_columns(w, qd, qd, 128)
    bd = rope.deinterleave_qk_columns(bias.reshape(1, -1), qd, qd, 128).reshape(-1)
    wq, chan = pkg.quantize_qkv_weight(wd, qd, qd)
    cos_rh, sin_rh = rope.rope_rotate_half_caches(cos, sin)
    split = pkg.adaln_modulate(hidden, None, None, eps=1e-6, norm_type="layer_norm", quant="row", row_layout="split")
    y = pkg.row_mx_qkv_proj(split, wq, chan, bd, num_heads=heads, head_dim=128, num_kv_heads=heads, fused_rope=True,
                            cos_cache=cos_rh, sin_cache=sin_rh, qk_norm_pre_rope=True)
    torch.cuda.synchronize()
    yq = y[:, :qd].reshape(1, T, heads, 128)
    yk = y[:, qd:2 * qd].reshape(1, T, heads, 128)
    f = lambda t: t.float().cpu().numpy()
    _cmp(f(yq), f(q[..., perm]), 0.995, 0.6, "Q fp8 leaf vs bf16 path")
    _cmp(f(yk), f(k[..., perm]), 0.995, 0.6, "K fp8 leaf vs bf16 path")
    _cmp(f(y[:, 2 * qd:]), f(qkv[:, 2 * qd:]), 0.995, 0.3, "V fp8 leaf vs bf16 path")


def test_errors(pkg, dev):
    hidden, w, bias, I = _setup(16, 200, 2, dev)  # H = 200 is not a multiple of 128
    lib = pytest.importorskip("importlib").import_module("vllm-omni-neuron_b200._lib")
    packed = pkg.adaln_modulate(hidden, None, None, eps=1e-6, quant="row")
    wq, chan = pkg.quantize_qkv_weight(w, 256, 256)
    with pytest.raises(lib.VomniError):
        pkg.row_mx_qkv_proj(packed, wq, chan, bias, num_heads=2, head_dim=128, num_kv_heads=2)
    with pytest.raises(NotImplementedError):
        pkg.row_mx_qkv_proj(packed, wq, chan, bias, num_heads=2, head_dim=128, num_kv_heads=2, replica_groups=((0, 1),))


def _mx_pack_ref(sc: np.ndarray) -> np.ndarray:
    """Scale-atom tiling of [rows, k/32] UE8M0 scales: tiles [k/128][ceil(rows/128)][512], byte
    m0*16 + m1*4 + j of a tile = row 32*m1 + m0, scale block j; rows past the end hold 127 (2^0)."""
    rows, kb = sc.shape
    rb = -(-rows // 128)
    pad = np.full((rb * 128, kb), 127, np.uint8)
    pad[:rows] = sc
    t = pad.reshape(rb, 4, 32, kb // 4, 4)  # [rb, m1, m0, kb4, j]
    return np.ascontiguousarray(t.transpose(3, 0, 2, 1, 4)).reshape(-1)


@pytest.mark.parametrize("rows,k", [(300, 512), (128, 128), (1, 256)])
def test_mx_scale_pack_layout(pkg, dev, rows, k):
    g = torch.Generator().manual_seed(rows)
    sc = torch.randint(100, 150, (rows, k // 32), generator=g, dtype=torch.uint8)
    got = pkg.pack_mx_scales(sc.to(dev)).cpu().numpy()
    assert np.array_equal(got, _mx_pack_ref(sc.numpy()))


@pytest.mark.parametrize("T,H,heads", [(300, 512, 2), (129, 1024, 4), (1, 512, 2), (1000, 1024, 2)])
def test_mx32_gemm_vs_oracle(pkg, dev, T, H, heads):
    """Block-scaled tcgen05 MMA (UE8M0 per 32 contraction values on both operands) against the oracle
    on the same dequantised operands."""
    hidden, w, bias, I = _setup(T, H, heads, dev, seed=4)
    # a few large outliers so the 32-blocks carry different scales
    hidden[:, ::97] *= 40
    xc, xs = pkg.adaln_modulate(hidden, None, None, eps=1e-6, norm_type="none", quant="mx32")
    wc, ws, wsp = pkg.quantize_qkv_weight_mx32(w)
    y = pkg.mx32_qkv_proj((xc, xs), wc, wsp, bias, num_heads=heads, head_dim=128, num_kv_heads=heads)
    torch.cuda.synchronize()
    deq = lambda c, s: (e4m3fn_from_bits(c.view(torch.uint8).cpu().numpy()).reshape(c.shape[0], -1, 32)
                        * np.exp2(s.cpu().numpy().astype(np.float64) - 127)[..., None]).reshape(c.shape[0], -1)
    xd, wd = deq(xc, xs), deq(wc, ws)  # [T, H], [I, H]
    assert len(np.unique(xs.cpu().numpy())) > 1 and len(np.unique(ws.cpu().numpy())) > 1
    # weight quant = the oracle's MX-32 quant of the bf16 weight
    _, ws_ref, wd_ref = oq.mx32_weight_quant(w.to(torch.bfloat16).float().cpu().numpy())
    assert np.array_equal(ws.cpu().numpy(), ws_ref.T) and np.array_equal(wd.astype(np.float32), wd_ref.T)
    ref = oq.mx32_qkv_ref(xd, wd.T, bias.float().cpu().numpy())
    got = y.float().cpu().numpy()
    _cmp(got, ref, 0.99999, 1e-2 * max(1.0, np.abs(ref).max()), f"mx32 gemm {T}x{H}x{I}")
    assert (np.abs(got - ref) <= np.abs(ref) * 2 ** -7 + 1e-3).mean() > 0.999


def test_mx32_norm_rope_epilogue(pkg, dev):
    T, H, heads = 257, 1024, 4
    hidden, w, bias, I = _setup(T, H, heads, dev, seed=6)
    rope = pytest.importorskip("importlib").import_module("vllm-omni-neuron_b200.rope")
    cos, sin = rope.wan_rotary_freqs(128, (1, 2, 2), 1024, (3, 20, 40), device=dev)
    cos_rh, sin_rh = rope.rope_rotate_half_caches(cos[:, :T], sin[:, :T])
    xc, xs = pkg.adaln_modulate(hidden, None, None, eps=1e-6, norm_type="layer_norm", quant="mx32")
    wc, ws, wsp = pkg.quantize_qkv_weight_mx32(w)
    y = pkg.mx32_qkv_proj((xc, xs), wc, wsp, bias, num_heads=heads, head_dim=128, num_kv_heads=heads, fused_rope=True,
                          cos_cache=cos_rh, sin_cache=sin_rh, qk_norm_pre_rope=True)
    torch.cuda.synchronize()
    deq = lambda c, s: (e4m3fn_from_bits(c.view(torch.uint8).cpu().numpy()).reshape(c.shape[0], -1, 32)
                        * np.exp2(s.cpu().numpy().astype(np.float64) - 127)[..., None]).reshape(c.shape[0], -1)
    ref = oq.mx32_qkv_ref(deq(xc, xs), deq(wc, ws).T, bias.float().cpu().numpy(), num_heads=heads, head_dim=128,
                          num_kv_heads=heads, cos=cos_rh.reshape(T, 128).cpu().numpy(),
                          sin=sin_rh.reshape(T, 128).cpu().numpy(), eps=1e-6)
    _cmp(y.float().cpu().numpy(), ref, 0.99999, 3e-2, "mx32 epilogue")


def test_c3_width_row_and_mx32_vs_oracle(pkg, dev):
    """BASELINE config 3's projection width, H=5120 -> I=3*5120 (40 heads per segment), on a 512-row
    slice: the ROW GEMM with the across-heads norm + rotate-half RoPE epilogue against the oracle
    (pinned to the reference's ROW_MX dequant-matmul by ``qkv_row_mx.npz``), and the MX-32
    block-scaled GEMM against the oracle on the same dequantised operands. LayerNorm eps 1e-6 and
    shift/scale ~ N(0, 0.1) as in config 3."""
    T, H, heads = 512, 5120, 40
    hidden, w, bias, I = _setup(T, H, heads, dev, seed=7)
    g = torch.Generator().manual_seed(8)
    mods = (torch.randn(6, H, generator=g) * 0.1).to(dev)
    mul, add = (1 + mods[1]).to(torch.bfloat16), mods[0].to(torch.bfloat16)
    rope = pytest.importorskip("importlib").import_module("vllm-omni-neuron_b200.rope")
    cos, sin = rope.wan_rotary_freqs(128, (1, 2, 2), 1024, (21, 60, 104), device=dev)
    cos_rh, sin_rh = rope.rope_rotate_half_caches(cos[:, :T], sin[:, :T])
    kw = dict(num_heads=heads, head_dim=128, num_kv_heads=heads)
    # ROW
    packed = pkg.adaln_modulate(hidden, mul, add, eps=1e-6, norm_type="layer_norm", quant="row")
    wq, chan = pkg.quantize_qkv_weight(w, heads * 128, heads * 128)
    y = pkg.row_mx_qkv_proj(packed, wq, chan, bias, fused_rope=True, cos_cache=cos_rh, sin_cache=sin_rh,
                            qk_norm_pre_rope=True, **kw)
    y_plain = pkg.row_mx_qkv_proj(packed, wq, chan, bias, **kw)
    torch.cuda.synchronize()
    pk = packed.view(torch.uint8).cpu().numpy()
    wc = e4m3fn_from_bits(wq.view(torch.uint8).cpu().numpy()).T  # [H, I]
    ref_plain = oq.row_mx_qkv_ref(pk, wc, chan.cpu().numpy(), bias.float().cpu().numpy())
    got = y_plain.float().cpu().numpy()
    _cmp(got, ref_plain, 0.99999, 1e-2 * max(1.0, np.abs(ref_plain).max()), "C3 ROW gemm")
    assert (np.abs(got - ref_plain) <= np.abs(ref_plain) * 2 ** -7 + 1e-3).mean() > 0.999
    ref = oq.qkv_epilogue(ref_plain, gamma_q=None, gamma_k=None, cos=cos_rh.reshape(T, 128).cpu().numpy(),
                          sin=sin_rh.reshape(T, 128).cpu().numpy(), eps=1e-6, **kw)
    _cmp(y.float().cpu().numpy(), ref, 0.99999, 3e-2, "C3 ROW gemm + norm + RoPE")
    # MX-32
    xc, xs = pkg.adaln_modulate(hidden, mul, add, eps=1e-6, norm_type="layer_norm", quant="mx32")
    wmc, wms, wmsp = pkg.quantize_qkv_weight_mx32(w)
    ym = pkg.mx32_qkv_proj((xc, xs), wmc, wmsp, bias, **kw)
    torch.cuda.synchronize()
    deq = lambda c, s: (e4m3fn_from_bits(c.view(torch.uint8).cpu().numpy()).reshape(c.shape[0], -1, 32)
                        * np.exp2(s.cpu().numpy().astype(np.float64) - 127)[..., None]).reshape(c.shape[0], -1)
    ref_mx = oq.mx32_qkv_ref(deq(xc, xs), deq(wmc, wms).T, bias.float().cpu().numpy())
    got_mx = ym.float().cpu().numpy()
    _cmp(got_mx, ref_mx, 0.99999, 1e-2 * max(1.0, np.abs(ref_mx).max()), "C3 MX-32 gemm")
    assert (np.abs(got_mx - ref_mx) <= np.abs(ref_mx) * 2 ** -7 + 1e-3).mean() > 0.999
