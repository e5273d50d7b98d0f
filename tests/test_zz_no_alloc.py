"""The allocation-free attention entry point, called through the C ABI.

vomni_cm_attention_local_noalloc serves callers that cannot allocate device memory (a plugin inside a
host runtime that owns the device heap, or a latency-critical path that must not take cudaMalloc's
implicit synchronisation): its scratch lives in a library-owned static device array. Both entry
points run the same kernels on the same inputs, so the results must be bit-identical; this checks
that on two calls in a row with different shapes (the shared scratch keeps the previous call's
contents, so the second call must not depend on them), checks the first shape against the CPU
oracle's exact attention, and checks that a shape beyond the array's limit is rejected. Collected
last so a failure here comes after every other test has run; it also passes alone in a fresh
process.
"""

import ctypes
import math
from importlib import import_module

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL_COS = 0.9999
TOL_ABS = 2e-2


def _qkv(b, s, h, seed, dev):
    g = torch.Generator().manual_seed(seed)
    return [(torch.randn(b, s, h, 128, generator=g) * 0.5).to(torch.bfloat16).to(dev) for _ in range(3)]


def _close(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    cos = (a * b).sum() / math.sqrt((a * a).sum() * (b * b).sum())
    assert cos >= TOL_COS and np.abs(a - b).max() <= TOL_ABS, (cos, np.abs(a - b).max())


def test_noalloc_matches_workspace_entry_point(pkg, dev):
    lib = import_module("vllm-omni-neuron_b200._lib")
    L = lib.load()
    stream = torch.cuda.current_stream(dev).cuda_stream
    for call, (b, s, h, flags) in enumerate([(1, 1000, 3, lib.CM_OUT_DMAJOR), (2, 333, 2, 0)]):
        q, k, v = _qkv(b, s, h, 100 + call, dev)
        shape = (b, h, 128, s) if flags & lib.CM_OUT_DMAJOR else (b, h, s, 128)
        ref = torch.empty(shape, dtype=torch.bfloat16, device=dev)
        ws_bytes = L.vomni_cm_workspace_bytes(b, s, h, 128)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
        lib.check(
            L.vomni_cm_attention_local(q.data_ptr(), k.data_ptr(), v.data_ptr(), ref.data_ptr(), None, b, s, h, 128,
                                       1 / math.sqrt(128), flags, ws.data_ptr(), ws_bytes, stream),
            "vomni_cm_attention_local",
        )
        got = torch.empty(shape, dtype=torch.bfloat16, device=dev)
        lib.check(
            L.vomni_cm_attention_local_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), got.data_ptr(), None, b, s, h,
                                               128, 1 / math.sqrt(128), flags, stream),
            "vomni_cm_attention_local_noalloc",
        )
        torch.cuda.synchronize()
        assert torch.equal(got, ref), f"call {call}: no-alloc result differs from the workspace entry point"
        if call == 0:
            from oracle import attention as oat

            tr = lambda x: np.transpose(x.float().cpu().numpy(), (0, 2, 1, 3))
            exact = oat.torch_attend(tr(q), tr(k), tr(v), 1 / math.sqrt(128))  # [b, h, s, d]
            _close(got.float().cpu().numpy().transpose(0, 1, 3, 2), exact)
    assert lib.device_status() == 0


def test_noalloc_rejects_oversized_shapes(pkg, dev):
    lib = import_module("vllm-omni-neuron_b200._lib")
    L = lib.load()
    p = ctypes.c_void_p(256)
    # 40 heads x 75600 tokens needs ~12 MB of scratch, above the 8 MiB array: rejected before any launch
    rc = L.vomni_cm_attention_local_noalloc(p, p, p, p, None, 1, 75600, 40, 128, 0.088, 0, None)
    assert rc == 8  # VOMNI_EWORKSPACE
