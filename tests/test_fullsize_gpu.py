"""Full-size checks at the BASELINE shapes through size-independent properties (B200 only).

C2 attention (B=1, S=32760, H=40, D=128), where the CPU oracle cannot run whole:
* linearity in V: attn(q, k, 2v) == 2 * attn(q, k, v) bit for bit (P and l do not change, doubling
  is exact in fp32 and bf16);
* convexity: each output is a convex combination of V rows, so |o| <= max |v| per (head, dim);
* layouts: the d-major output is the transpose of the head-major output, bit for bit;
* a sample of query rows against the exact CPU attention over all 32760 keys;
* the CP=8 pass plan over the same keys (8 blocks of 4095, fp32 partials between passes) against
  the single pass (fp32 summation order only).
C3 FP8 QKV GEMM (T=32760, H=5120, I=15360): doubling the row scales doubles the output bit for bit.
"""

import math

import numpy as np
import pytest
import torch

from oracle import attention as oat

pytestmark = pytest.mark.gpu

S, H, D = 32760, 40, 128


@pytest.fixture(scope="module")
def qkv_full(dev):
    g = torch.Generator(device=dev).manual_seed(5)
    mk = lambda: (torch.randn(1, S, H, D, generator=g, device=dev) * 0.5).to(torch.bfloat16)  # noqa: E731
    return mk(), mk(), mk()


def test_c2_linearity_convexity_layout(pkg, dev, qkv_full):
    q, k, v = qkv_full
    o = pkg.ring_attention_const_max_fwd(q, k, v)
    o2 = pkg.ring_attention_const_max_fwd(q, k, v * 2)
    od = pkg.wan_cp_self_attention(q, k, v, 1 / math.sqrt(D), 1, None, None)
    torch.cuda.synchronize()
    assert torch.equal(o2, o * 2)
    vmax = v.float().abs().amax(dim=1)  # [1, H, D]
    assert bool((o.float().abs() <= vmax[:, :, None, :] * (1 + 2 ** -7)).all())
    assert torch.equal(od, o.transpose(2, 3).contiguous())


def test_c2_row_sample_vs_exact(pkg, dev, qkv_full):
    q, k, v = qkv_full
    o = pkg.ring_attention_const_max_fwd(q, k, v)
    torch.cuda.synchronize()
    heads, rows = [0, 17, 39], np.r_[0:16, 16380:16396, S - 16:S]
    qs = q[0, rows][:, heads].float().cpu().numpy().transpose(1, 0, 2)[None]  # [1, h, r, d]
    ks = k[0][:, heads].float().cpu().numpy().transpose(1, 0, 2)[None]
    vs = v[0][:, heads].float().cpu().numpy().transpose(1, 0, 2)[None]
    ref = oat.torch_attend(qs, ks, vs, 1 / math.sqrt(D))[0]  # [h, r, d]
    got = o[0][heads][:, rows].float().cpu().numpy()
    cos = (got * ref).sum() / math.sqrt((got * got).sum() * (ref * ref).sum())
    assert cos >= 0.9999 and np.abs(got - ref).max() <= 2e-2, (cos, np.abs(got - ref).max())


def test_c2_cp8_pass_plan_equals_single_pass(pkg, dev, qkv_full):
    """The 4095-token shards of rank 0 at CP=8: its queries against all 8 key blocks through the ring's
    pass plan (local block, then 1, 2, 4 blocks, fp32 partials in between, later passes overlapped)
    equal one pass over the 32760 keys up to fp32 summation order."""
    from importlib import import_module

    lib = import_module("vllm-omni-neuron_b200._lib")
    ring = import_module("vllm-omni-neuron_b200.ring")
    L = lib.load()
    q, k, v = qkv_full
    world, s = 8, S // 8
    ql = q[:, :s].contiguous()
    st = torch.cuda.current_stream().cuda_stream
    qn2 = torch.empty(H, s, device=dev)
    km = torch.empty(H, device=dev)
    qn2_all = torch.empty(H, S, device=dev)
    lib.check(L.vomni_cm_prologue(ql.data_ptr(), ql.data_ptr(), 1, s, H, D, qn2.data_ptr(), km.data_ptr(), st), "p")
    lib.check(L.vomni_cm_prologue(k.data_ptr(), k.data_ptr(), 1, S, H, D, qn2_all.data_ptr(), km.data_ptr(), st), "p")
    scale = 1 / math.sqrt(D)
    single = torch.empty(1, H, s, D, dtype=torch.bfloat16, device=dev)
    lib.check(L.vomni_cm_attend(ql.data_ptr(), k.data_ptr(), v.data_ptr(), 1, s, S, 0, S, H, D, scale, qn2.data_ptr(),
                                km.data_ptr(), None, None, lib.CM_FINAL, single.data_ptr(), None, st), "single")
    # gather buffer in ring-step order for rank 0: step j pulls block (0 - j) mod 8
    kl, vl = k[:, :s].contiguous(), v[:, :s].contiguous()
    order = [ring.source_rank(0, world, j) for j in range(1, world)]
    kg = torch.cat([k[:, r * s:(r + 1) * s] for r in order], dim=1).contiguous()
    vg = torch.cat([v[:, r * s:(r + 1) * s] for r in order], dim=1).contiguous()
    acc_o = torch.empty(H, s, D, device=dev)
    acc_l = torch.empty(H, s, device=dev)
    out = torch.empty(1, H, s, D, dtype=torch.bfloat16, device=dev)
    lib.check(L.vomni_cm_attend(ql.data_ptr(), kl.data_ptr(), vl.data_ptr(), 1, s, s, 0, s, H, D, scale, qn2.data_ptr(),
                                km.data_ptr(), acc_o.data_ptr(), acc_l.data_ptr(), 0, None, None, st), "pass0")
    plan = ring.phase_plan(world)
    for i, (first, count) in enumerate(plan[1:], start=1):
        fl = lib.CM_ACC_IN | lib.CM_OVERLAP | (lib.CM_FINAL if i == len(plan) - 1 else 0)
        lib.check(L.vomni_cm_attend(ql.data_ptr(), kg.data_ptr(), vg.data_ptr(), 1, s, (world - 1) * s, first * s,
                                    count * s, H, D, scale, qn2.data_ptr(), km.data_ptr(), acc_o.data_ptr(),
                                    acc_l.data_ptr(), fl, out.data_ptr(), None, st), "pass")
    torch.cuda.synchronize()
    a, b = out.float(), single.float()
    cos = float((a * b).sum() / torch.sqrt((a * a).sum() * (b * b).sum()))
    assert cos >= 0.99999 and float((a - b).abs().max()) <= 8e-3, (cos, float((a - b).abs().max()))
    assert lib.device_status() == 0


def test_c3_row_scale_linearity(pkg, dev):
    from importlib import import_module

    lib = import_module("vllm-omni-neuron_b200._lib")
    L = lib.load()
    T, Hd, I = 32760, 5120, 15360
    g = torch.Generator(device=dev).manual_seed(6)
    x = (torch.randn(T, Hd, generator=g, device=dev) * 100).clamp(-448, 448).to(torch.float8_e4m3fn)
    w = (torch.randn(I, Hd, generator=g, device=dev) * 100).clamp(-448, 448).to(torch.float8_e4m3fn)
    rs = torch.rand(T, generator=g, device=dev) * 1e-3 + 1e-4
    cs = torch.rand(I, generator=g, device=dev) * 1e-3 + 1e-4
    st = torch.cuda.current_stream().cuda_stream
    y1 = torch.empty(T, I, dtype=torch.bfloat16, device=dev)
    y2 = torch.empty_like(y1)
    lib.check(L.vomni_qkv_fp8_gemm(x.data_ptr(), rs.data_ptr(), w.data_ptr(), cs.data_ptr(), None, T, Hd, I, 0, 0,
                                   y1.data_ptr(), None, st), "gemm")
    rs2 = rs * 2
    lib.check(L.vomni_qkv_fp8_gemm(x.data_ptr(), rs2.data_ptr(), w.data_ptr(), cs.data_ptr(), None, T, Hd, I, 0, 0,
                                   y2.data_ptr(), None, st), "gemm")
    torch.cuda.synchronize()
    assert torch.equal(y2, y1 * 2)
    # a sampled block against the fp32 product of the same codes
    r0, c0 = 16000, 7000
    ref = (x[r0:r0 + 64].float() @ w[c0:c0 + 64].float().T) * rs[r0:r0 + 64, None] * cs[None, c0:c0 + 64]
    got = y1[r0:r0 + 64, c0:c0 + 64].float()
    assert float(((got - ref).abs() / ref.abs().clamp(min=1.0)).max()) <= 2 ** -7


def test_c4_cp8_shard_pass_plan_vs_exact(pkg, dev):
    """BASELINE config 4 (S=75600) at CP=8, emulated on one GPU: rank 3's 9450-token query shard
    against its own block and the 7 remote blocks in the ring's gather order, through the ring's pass
    plan (local block, then 1, 2, 4 blocks; fp32 partials in between, later passes overlapped). A
    sample of query rows (3 heads, 48 rows spread over the shard) against the exact CPU attention
    over all 75600 keys, and the whole shard against one pass over the same keys."""
    from importlib import import_module

    lib = import_module("vllm-omni-neuron_b200._lib")
    ring = import_module("vllm-omni-neuron_b200.ring")
    L = lib.load()
    S4, world, rank = 75600, 8, 3
    s = S4 // world
    g = torch.Generator(device=dev).manual_seed(9)
    mk = lambda: (torch.randn(1, S4, H, D, generator=g, device=dev) * 0.5).to(torch.bfloat16)  # noqa: E731
    q, k, v = mk(), mk(), mk()
    ql = q[:, rank * s:(rank + 1) * s].contiguous()
    kl, vl = k[:, rank * s:(rank + 1) * s].contiguous(), v[:, rank * s:(rank + 1) * s].contiguous()
    st = torch.cuda.current_stream().cuda_stream
    qn2 = torch.empty(H, s, device=dev)
    km = torch.empty(H, device=dev)
    qn2_all = torch.empty(H, S4, device=dev)
    lib.check(L.vomni_cm_prologue(ql.data_ptr(), ql.data_ptr(), 1, s, H, D, qn2.data_ptr(), km.data_ptr(), st), "p")
    lib.check(L.vomni_cm_prologue(k.data_ptr(), k.data_ptr(), 1, S4, H, D, qn2_all.data_ptr(), km.data_ptr(), st), "p")
    scale = 1 / math.sqrt(D)
    order = [ring.source_rank(rank, world, j) for j in range(1, world)]
    kg = torch.cat([k[:, r * s:(r + 1) * s] for r in order], dim=1).contiguous()
    vg = torch.cat([v[:, r * s:(r + 1) * s] for r in order], dim=1).contiguous()
    acc_o = torch.empty(H, s, D, device=dev)
    acc_l = torch.empty(H, s, device=dev)
    out = torch.empty(1, H, s, D, dtype=torch.bfloat16, device=dev)
    lib.check(L.vomni_cm_attend(ql.data_ptr(), kl.data_ptr(), vl.data_ptr(), 1, s, s, 0, s, H, D, scale, qn2.data_ptr(),
                                km.data_ptr(), acc_o.data_ptr(), acc_l.data_ptr(), 0, None, None, st), "pass0")
    plan = ring.phase_plan(world)
    assert plan == [(-1, 1), (0, 1), (1, 2), (3, 4)]
    for i, (first, count) in enumerate(plan[1:], start=1):
        fl = lib.CM_ACC_IN | lib.CM_OVERLAP | (lib.CM_FINAL if i == len(plan) - 1 else 0)
        lib.check(L.vomni_cm_attend(ql.data_ptr(), kg.data_ptr(), vg.data_ptr(), 1, s, (world - 1) * s, first * s,
                                    count * s, H, D, scale, qn2.data_ptr(), km.data_ptr(), acc_o.data_ptr(),
                                    acc_l.data_ptr(), fl, out.data_ptr(), None, st), "pass")
    single = torch.empty(1, H, s, D, dtype=torch.bfloat16, device=dev)
    lib.check(L.vomni_cm_attend(ql.data_ptr(), k.data_ptr(), v.data_ptr(), 1, s, S4, 0, S4, H, D, scale, qn2.data_ptr(),
                                km.data_ptr(), None, None, lib.CM_FINAL, single.data_ptr(), None, st), "single")
    torch.cuda.synchronize()
    assert lib.device_status() == 0
    a, b = out.float(), single.float()
    cos = float((a * b).sum() / torch.sqrt((a * a).sum() * (b * b).sum()))
    assert cos >= 0.99999 and float((a - b).abs().max()) <= 8e-3, (cos, float((a - b).abs().max()))
    heads, rows = [0, 21, 39], np.r_[0:16, 4720:4736, s - 16:s]
    qs = ql[0, rows][:, heads].float().cpu().numpy().transpose(1, 0, 2)[None]  # [1, h, r, d]
    ks = k[0][:, heads].float().cpu().numpy().transpose(1, 0, 2)[None]
    vs = v[0][:, heads].float().cpu().numpy().transpose(1, 0, 2)[None]
    ref = oat.torch_attend(qs, ks, vs, scale)[0]  # [h, r, d]
    got = out[0][heads][:, rows].float().cpu().numpy()
    cos = (got * ref).sum() / math.sqrt((got * got).sum() * (ref * ref).sum())
    assert cos >= 0.9999 and np.abs(got - ref).max() <= 2e-2, (cos, np.abs(got - ref).max())
