"""GPU parity of the const-max attention kernels against the CPU oracle (B200 only)."""

import math

import numpy as np
import pytest
import torch

from oracle import attention as oat

pytestmark = pytest.mark.gpu

TOL_COS = 0.9999  # north-star tolerance for bf16 attention vs an fp32 reference
TOL_ABS = 2e-2


def _f32(t):
    return t.detach().float().cpu().numpy()


def _cmp(got, ref, what=""):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    assert np.isfinite(got).all(), what
    cos = (got * ref).sum() / math.sqrt((got * got).sum() * (ref * ref).sum() + 1e-300)
    mx = np.abs(got - ref).max()
    assert cos >= TOL_COS and mx <= TOL_ABS, f"{what}: cos={cos:.6f} maxabs={mx:.4g}"


def _rand_qkv(b, s, h, seed, dev, scale=0.5):
    g = torch.Generator().manual_seed(seed)
    mk = lambda: (torch.randn(b, s, h, 128, generator=g) * scale).to(torch.bfloat16)
    return [x.to(dev) for x in (mk(), mk(), mk())]


@pytest.mark.parametrize(
    "b,s,h",
    [(1, 128, 1), (1, 256, 2), (2, 130, 3), (1, 127, 2), (1, 1, 1), (1, 1000, 2), (1, 4095, 1)],
)
def test_local_vs_oracle(pkg, dev, b, s, h):
    q, k, v = _rand_qkv(b, s, h, 1000 + s + h, dev)
    o = pkg.ring_attention_const_max_fwd(q, k, v)
    torch.cuda.synchronize()
    assert tuple(o.shape) == (b, h, s, 128)
    qn, kn, vn = _f32(q), _f32(k), _f32(v)
    ref_exact = oat.torch_attend(*(np.transpose(x, (0, 2, 1, 3)) for x in (qn, kn, vn)), 1 / math.sqrt(128))
    _cmp(_f32(o), ref_exact, "vs exact")
    ref_cm = oat.const_max_ring_attention([qn], [kn], [vn])[0]
    _cmp(_f32(o), ref_cm, "vs const-max oracle")
    from importlib import import_module

    assert import_module("vllm-omni-neuron_b200._lib").device_status() == 0


def test_golden_torch_attend(pkg, dev, golden):
    """On the inputs of the reference's own _torch_attend golden vectors (S_q == S_k case)."""
    g = golden("torch_attend.npz")
    q, k, v = (torch.from_numpy(np.ascontiguousarray(np.transpose(g[f"a|{n}"], (0, 2, 1, 3)))).to(torch.bfloat16).to(dev) for n in "qkv")
    o = pkg.ring_attention_const_max_fwd(q, k, v, softmax_scale=float(g["a|scale"]))
    _cmp(_f32(o), g["a|o"], "golden a")


def test_dmajor_and_lse(pkg, dev):
    b, s, h = 1, 300, 2
    q, k, v = _rand_qkv(b, s, h, 7, dev)
    o_bhsd, lse = pkg.ring_attention_const_max_fwd(q, k, v, training=True)
    o_bhds = pkg.wan_cp_self_attention(q, k, v, 1 / math.sqrt(128), 1, None, None)
    torch.cuda.synchronize()
    assert tuple(o_bhds.shape) == (b, h, 128, s)
    assert torch.equal(o_bhds, o_bhsd.transpose(2, 3).contiguous())
    qn, kn, vn = _f32(q), _f32(k), _f32(v)
    _, ref_lse = oat.const_max_ring_attention([qn], [kn], [vn], training=True)
    got = _f32(lse)
    ref = ref_lse[0]
    # LSE only defined on real rows; pad rows of the last group stay 0 (zero-initialised).
    assert np.abs(got - ref).max() < 2e-2
    # lse is exact softmax log-normaliser: compare with log-sum-exp of fp32 scores
    sc = np.einsum("bshd,bthd->bhst", qn, kn) / math.sqrt(128)
    lse_exact = np.log(np.exp(sc - sc.max(-1, keepdims=True)).sum(-1)) + sc.max(-1)
    for gi in range(-(-s // 128)):
        rows = min(128, s - gi * 128)
        assert np.abs(got[:, :, :rows, gi] - lse_exact[:, :, gi * 128:gi * 128 + rows]).max() < 5e-2


@pytest.mark.parametrize("n", [2, 3, 4])
def test_ring_steps_emulated(pkg, dev, n):
    """The ring's per-step path on one GPU: prologue per rank, global key max, then one
    vomni_cm_attend pass per ring step in ring order (step s consumes rank (r-s) mod n's block),
    accumulating in fp32 and normalising on the last step. Checked against the oracle ring."""
    from importlib import import_module

    lib = import_module("vllm-omni-neuron_b200._lib")
    L = lib.load()
    b, s, h = 1, 200, 2
    qs, ks, vs = [], [], []
    for r in range(n):
        q, k, v = _rand_qkv(b, s, h, 50 + r, dev)
        qs.append(q), ks.append(k), vs.append(v)
    st = torch.cuda.current_stream().cuda_stream
    qn2 = [torch.empty(b * h, s, dtype=torch.float32, device=dev) for _ in range(n)]
    km = [torch.empty(b * h, dtype=torch.float32, device=dev) for _ in range(n)]
    for r in range(n):
        lib.check(L.vomni_cm_prologue(qs[r].data_ptr(), ks[r].data_ptr(), b, s, h, 128, qn2[r].data_ptr(), km[r].data_ptr(), st), "prologue")
    kmax = torch.stack(km).amax(0)
    outs = []
    for r in range(n):
        acc_o = torch.empty(b * h, s, 128, dtype=torch.float32, device=dev)
        acc_l = torch.empty(b * h, s, dtype=torch.float32, device=dev)
        out = torch.empty(b, h, s, 128, dtype=torch.bfloat16, device=dev)
        for step in range(n):
            src = (r - step) % n
            flags = (lib.CM_ACC_IN if step > 0 else 0) | (lib.CM_FINAL if step == n - 1 else 0)
            lib.check(
                L.vomni_cm_attend(
                    qs[r].data_ptr(), ks[src].data_ptr(), vs[src].data_ptr(), b, s, s, 0, s, h, 128, 1 / math.sqrt(128),
                    qn2[r].data_ptr(), kmax.data_ptr(), acc_o.data_ptr(), acc_l.data_ptr(), flags, out.data_ptr(), None, st,
                ),
                "attend",
            )
        outs.append(out)
    torch.cuda.synchronize()
    ref = oat.const_max_ring_attention([_f32(x) for x in qs], [_f32(x) for x in ks], [_f32(x) for x in vs])
    exact = oat.wan_cp_self_attention_oracle([_f32(x) for x in qs], [_f32(x) for x in ks], [_f32(x) for x in vs], 1 / math.sqrt(128))
    for r in range(n):
        _cmp(_f32(outs[r]), ref[r], f"rank {r} vs oracle ring")
        _cmp(_f32(outs[r]).transpose(0, 1, 3, 2), exact[r], f"rank {r} vs exact")
    assert lib.device_status() == 0


@pytest.mark.parametrize("s,h", [(4095, 40), (700, 6)])
def test_overlapped_passes_equal_serial(pkg, dev, s, h):
    """Passes launched as programmatic dependents (VOMNI_CM_OVERLAP, the ring's passes after the
    first) give bit-identical results to serialised passes. (4095, 40) is the CP=8 shard of S=32760:
    320 CTA pairs per pass, a partly filled last wave that the next pass overlaps."""
    from importlib import import_module

    lib = import_module("vllm-omni-neuron_b200._lib")
    ring = import_module("vllm-omni-neuron_b200.ring")
    L = lib.load()
    world = 8
    plan = ring.phase_plan(world)
    q, k, v = _rand_qkv(1, s, h, 11, dev)
    _, kg, vg = _rand_qkv(1, (world - 1) * s, h, 12, dev)
    st = torch.cuda.current_stream().cuda_stream
    qn2 = torch.empty(h, s, dtype=torch.float32, device=dev)
    km = torch.empty(h, dtype=torch.float32, device=dev)
    lib.check(L.vomni_cm_prologue(q.data_ptr(), k.data_ptr(), 1, s, h, 128, qn2.data_ptr(), km.data_ptr(), st), "prologue")
    qn2_g = torch.empty(h, (world - 1) * s, dtype=torch.float32, device=dev)
    km_g = torch.empty(h, dtype=torch.float32, device=dev)
    lib.check(L.vomni_cm_prologue(kg.data_ptr(), kg.data_ptr(), 1, (world - 1) * s, h, 128, qn2_g.data_ptr(),
                                  km_g.data_ptr(), st), "prologue")
    km = torch.maximum(km, km_g)
    scale = 1 / math.sqrt(128)
    outs = []
    for overlap in (0, lib.CM_OVERLAP):
        acc_o = torch.empty(h, s, 128, dtype=torch.float32, device=dev)
        acc_l = torch.empty(h, s, dtype=torch.float32, device=dev)
        out = torch.empty(1, h, 128, s, dtype=torch.bfloat16, device=dev)
        lse = torch.zeros(1, h, 128, (s + 127) // 128, dtype=torch.float32, device=dev)  # pad rows stay 0
        lib.check(L.vomni_cm_attend(q.data_ptr(), k.data_ptr(), v.data_ptr(), 1, s, s, 0, s, h, 128, scale, qn2.data_ptr(),
                                    km.data_ptr(), acc_o.data_ptr(), acc_l.data_ptr(), 0, None, None, st), "pass0")
        for i, (first, count) in enumerate(plan[1:], start=1):
            fl = lib.CM_ACC_IN | overlap
            if i == len(plan) - 1:
                fl |= lib.CM_FINAL | lib.CM_OUT_DMAJOR | lib.CM_LSE
            lib.check(L.vomni_cm_attend(q.data_ptr(), kg.data_ptr(), vg.data_ptr(), 1, s, (world - 1) * s, first * s,
                                        count * s, h, 128, scale, qn2.data_ptr(), km.data_ptr(), acc_o.data_ptr(),
                                        acc_l.data_ptr(), fl, out.data_ptr(), lse.data_ptr(), st), "pass")
        outs.append((out, lse))
    torch.cuda.synchronize()
    assert torch.equal(outs[0][0], outs[1][0])
    assert torch.equal(outs[0][1], outs[1][1])
    assert lib.device_status() == 0
    if s <= 1024:
        kf = torch.cat([k, kg], dim=1)
        vf = torch.cat([v, vg], dim=1)
        ref = oat.const_max_ring_attention([_f32(q)], [_f32(kf)], [_f32(vf)])[0]
        _cmp(_f32(outs[1][0]).transpose(0, 1, 3, 2), ref, "overlapped passes vs oracle")


def test_key_subrange_masking(pkg, dev):
    """A pass over keys [k_start, k_start+n_keys) of a longer K/V must ignore the keys outside."""
    from importlib import import_module

    lib = import_module("vllm-omni-neuron_b200._lib")
    L = lib.load()
    b, s, h, skv = 1, 160, 1, 700
    q, _, _ = _rand_qkv(b, s, h, 3, dev)
    _, k, v = _rand_qkv(b, skv, h, 4, dev)
    k0, nk = 150, 301
    st = torch.cuda.current_stream().cuda_stream
    qn2 = torch.empty(b * h, s, dtype=torch.float32, device=dev)
    km = torch.empty(b * h, dtype=torch.float32, device=dev)
    ksub = k[:, k0:k0 + nk].contiguous()
    vsub = v[:, k0:k0 + nk].contiguous()
    qpad = torch.zeros(b, nk, h, 128, dtype=torch.bfloat16, device=dev)
    qpad[:, :s] = q
    # norms of q (first s rows) and of the key sub-range
    lib.check(L.vomni_cm_prologue(qpad.data_ptr(), ksub.data_ptr(), b, nk, h, 128, torch.empty(b * h, nk, device=dev).data_ptr(), km.data_ptr(), st), "p1")
    lib.check(L.vomni_cm_prologue(q.data_ptr(), q.data_ptr(), b, s, h, 128, qn2.data_ptr(), torch.empty(b * h, device=dev).data_ptr(), st), "p2")
    out = torch.empty(b, h, s, 128, dtype=torch.bfloat16, device=dev)
    lib.check(L.vomni_cm_attend(q.data_ptr(), k.data_ptr(), v.data_ptr(), b, s, skv, k0, nk, h, 128, 1 / math.sqrt(128), qn2.data_ptr(), km.data_ptr(), None, None, lib.CM_FINAL, out.data_ptr(), None, st), "attend")
    torch.cuda.synchronize()
    ref = oat.torch_attend(np.transpose(_f32(q), (0, 2, 1, 3)), np.transpose(_f32(ksub), (0, 2, 1, 3)), np.transpose(_f32(vsub), (0, 2, 1, 3)), 1 / math.sqrt(128))
    _cmp(_f32(out), ref, "subrange")
    assert lib.device_status() == 0


def test_errors(pkg, dev):
    q, k, v = _rand_qkv(1, 64, 1, 0, dev)
    with pytest.raises(AssertionError):
        pkg.ring_attention_const_max_fwd(q[..., :64].contiguous(), k[..., :64].contiguous(), v[..., :64].contiguous())
    with pytest.raises(TypeError):
        pkg.ring_attention_const_max_fwd(q.float(), k, v)


@pytest.mark.parametrize("b,s,h,training,layout",
                         [(1, 1000, 12, False, "bhds"), (2, 777, 7, True, "bhsd"), (1, 8000, 23, False, "bhds")])
def test_host_streamed_equals_device(pkg, dev, b, s, h, training, layout):
    """Pinned host q/k/v stream through head groups; heads are independent, so the host result is
    bit-identical to the device-resident call."""
    g = torch.Generator().manual_seed(11)
    q, k, v = ((torch.randn(b, s, h, 128, generator=g) * 0.5).to(torch.bfloat16) for _ in range(3))
    attn = pytest.importorskip("importlib").import_module("vllm-omni-neuron_b200.attention")
    host = attn.ring_attention_const_max_fwd(q.pin_memory(), k.pin_memory(), v.pin_memory(), training=training,
                                             out_layout=layout)
    devr = attn.ring_attention_const_max_fwd(q.to(dev), k.to(dev), v.to(dev), training=training, out_layout=layout)
    torch.cuda.synchronize()
    if training:
        assert host[0].device.type == "cpu" and torch.equal(host[0], devr[0].cpu())
        assert torch.equal(host[1], devr[1].cpu())
    else:
        assert host.device.type == "cpu" and torch.equal(host, devr.cpu())
    wan = pkg.wan_cp_self_attention(q.pin_memory(), k.pin_memory(), v.pin_memory(), 128 ** -0.5, 1, None, None)
    assert torch.equal(wan, pkg.wan_cp_self_attention(q.to(dev), k.to(dev), v.to(dev), 128 ** -0.5, 1, None, None).cpu())
    with pytest.raises(ValueError):
        attn.ring_attention_const_max_fwd(q, k, v)  # host tensors must be pinned


def test_host_stream_groups(pkg, dev):
    """Group sizing: one rank keeps 5-head groups; ring calls take enough heads per group to fill two
    waves of CTA pairs; explicit small groups (ragged last group) give the device result too."""
    attn = pytest.importorskip("importlib").import_module("vllm-omni-neuron_b200.attention")
    slots = torch.cuda.get_device_properties(dev).multi_processor_count // 2
    for s, h in ((32760, 40), (16380, 40), (8190, 40), (4095, 40), (8000, 23)):
        assert attn._host_group_heads(s, h, dev, 1) == 5
        gh = attn._host_group_heads(s, h, dev, 8)
        assert 5 <= gh <= h
        assert gh * -(-s // 512) >= min(h * -(-s // 512), 2 * slots) or gh == 5
    assert attn._host_group_heads(4095, 40, dev, 8) == 20 and attn._host_group_heads(8190, 40, dev, 4) == 10
    g = torch.Generator().manual_seed(12)
    q, k, v = ((torch.randn(1, 1000, 7, 128, generator=g) * 0.5).to(torch.bfloat16) for _ in range(3))
    fn = lambda a, b_, c: attn.attention_local(a, b_, c, out_layout="bhds")
    host = attn._host_streamed(fn, q.pin_memory(), k.pin_memory(), v.pin_memory(), out_layout="bhds", training=False,
                               group_heads=3)
    devr = attn.attention_local(q.to(dev), k.to(dev), v.to(dev), out_layout="bhds")
    torch.cuda.synchronize()
    assert torch.equal(host, devr.cpu())


def test_c1_full_shape_vs_oracle(pkg, dev):
    """BASELINE config 1 at its stated shape: B=1, S=4096, H=40, Q/K/V ~ N(0,1)*0.5 (seeds 0,1,2),
    softmax scale 1/sqrt(128), against the exact fp32 attention and the const-max restatement."""
    b, s, h = 1, 4096, 40
    qkv = []
    for seed in (0, 1, 2):
        g = torch.Generator().manual_seed(seed)
        qkv.append((torch.randn(b, s, h, 128, generator=g) * 0.5).to(torch.bfloat16))
    o = pkg.ring_attention_const_max_fwd(*(x.to(dev) for x in qkv))
    torch.cuda.synchronize()
    qn, kn, vn = (x.float().numpy() for x in qkv)
    got = _f32(o)
    ref_exact = oat.torch_attend(*(np.transpose(x, (0, 2, 1, 3)) for x in (qn, kn, vn)), 1 / math.sqrt(128))
    _cmp(got, ref_exact, "C1 vs exact")
    ref_cm = oat.const_max_ring_attention([qn], [kn], [vn])[0]
    _cmp(got, ref_cm, "C1 vs const-max oracle")
    from importlib import import_module

    assert import_module("vllm-omni-neuron_b200._lib").device_status() == 0


def test_exp2_poly_error_bound(pkg, dev):
    """The FMA-pipe exponential the softmax uses for a share of its probabilities: relative error
    against exact 2^x (float64) within the polynomial's fitted bound plus fp32 evaluation rounding
    (1e-4) wherever the result is a normal number, and 0 below x = -125.5 as the flush-to-zero
    MUFU exponential gives 0 under 2^-126. Also within that bound of CUDA's own exp2 on the GPU."""
    from importlib import import_module

    lib = import_module("vllm-omni-neuron_b200._lib")
    L = lib.load()
    xs = torch.cat([torch.linspace(-125.49, 1.0, 1 << 20, dtype=torch.float64).float(),
                    torch.tensor([0.0, -0.5, 0.5, -1.0, -64.25, -125.0, -125.49, -125.5, -125.6, -126.0, -127.0,
                                  -200.0, -1e30, float("-inf")])])
    x = xs.to(dev)
    y = torch.empty_like(x)
    lib.check(L.vomni_selftest_exp2_poly(x.data_ptr(), y.data_ptr(), x.numel(), torch.cuda.current_stream().cuda_stream),
              "vomni_selftest_exp2_poly")
    cuda_exp2 = torch.exp2(x)
    torch.cuda.synchronize()
    xd = xs.double().numpy()
    got = y.cpu().double().numpy()
    exact = np.exp2(xd)
    normal = xd > -125.5
    rel = np.abs(got[normal] - exact[normal]) / exact[normal]
    assert rel.max() <= 1e-4, rel.max()
    assert (got[~normal] == 0).all()
    cu = cuda_exp2.cpu().double().numpy()
    assert (np.abs(got[normal] - cu[normal]) / cu[normal]).max() <= 1e-4
    # odd element count: the last value is evaluated on its own
    lib.check(L.vomni_selftest_exp2_poly(x.data_ptr(), y.data_ptr(), 3, torch.cuda.current_stream().cuda_stream), "odd n")
    torch.cuda.synchronize()
    assert np.allclose(y[:3].cpu().double().numpy(), exact[:3], rtol=1e-4, atol=0)
