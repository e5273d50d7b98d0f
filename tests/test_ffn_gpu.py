"""GPU parity of the Wan FFN (two CTA-pair bf16 GEMMs, GELU-tanh in the first epilogue) against the
CPU oracle, which is pinned to the reference's ``_wan_mlp`` (B200 only)."""

import numpy as np
import pytest
import torch

from oracle import ffn as off
from oracle.numerics import bf16_round

pytestmark = pytest.mark.gpu


def _bf(x, dev):
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(torch.bfloat16).to(dev)


def _close(got, ref, what):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    step = np.exp2(np.floor(np.log2(np.maximum(np.maximum(np.abs(ref), np.abs(got)), 2.0 ** -100))) - 7)
    bad = np.abs(got - ref) > 2 * step * 1.0001 + 4e-3
    assert bad.mean() < 1e-4, f"{what}: {bad.mean():.2e} beyond tolerance, max {np.abs(got - ref).max():.3g}"
    cos = (got * ref).sum() / np.sqrt((got * got).sum() * (ref * ref).sum())
    assert cos > 0.99999, f"{what}: cos {cos}"


def test_golden_reference_outputs(pkg, dev, golden):
    g = golden("wan_mlp.npz")
    for tag in ("a", "b"):
        y = pkg.wan_mlp(_bf(g[f"{tag}|x"], dev), _bf(g[f"{tag}|wu"], dev), _bf(g[f"{tag}|wd"], dev),
                        _bf(g[f"{tag}|bu"], dev), _bf(g[f"{tag}|bd"], dev))
        torch.cuda.synchronize()
        _close(y.float().cpu().numpy(), g[f"{tag}|y"], f"golden {tag}")


@pytest.mark.parametrize("B,T,H,I", [(1, 1000, 512, 1536), (2, 130, 256, 768), (1, 8, 128, 256)])
def test_mlp_vs_oracle(pkg, dev, B, T, H, I):
    rng = np.random.default_rng(T + H)
    x = bf16_round(rng.standard_normal((B, T, H)).astype(np.float32))
    wu = bf16_round((0.04 * rng.standard_normal((H, I))).astype(np.float32))
    wd = bf16_round((0.04 * rng.standard_normal((I, H))).astype(np.float32))
    bu = bf16_round((0.3 * rng.standard_normal((1, I))).astype(np.float32))
    bd = bf16_round((0.3 * rng.standard_normal((1, H))).astype(np.float32))
    y = pkg.wan_mlp(_bf(x, dev), _bf(wu, dev), _bf(wd, dev), _bf(bu, dev), _bf(bd, dev))
    torch.cuda.synchronize()
    assert y.shape == (B, T, H)
    _close(y.float().cpu().numpy(), off.wan_mlp_ref(x, wu, wd, bu, bd), f"mlp {B}x{T}x{H}x{I}")


def test_errors(pkg, dev):
    x = torch.zeros(1, 8, 100, dtype=torch.bfloat16, device=dev)  # H % 64 != 0
    lib = pytest.importorskip("importlib").import_module("vllm-omni-neuron_b200._lib")
    with pytest.raises(lib.VomniError):
        pkg.wan_mlp(x, torch.zeros(100, 256, dtype=torch.bfloat16, device=dev),
                    torch.zeros(256, 100, dtype=torch.bfloat16, device=dev), None, None)
