"""Failure detection on the GPU without a GPU fault: a bounded device wait that nothing satisfies
runs out, reports an error status the host reads, and the context stays usable."""

import ctypes
import math
from importlib import import_module

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_context_survives(pkg, dev):
    lib = import_module("vllm-omni-neuron_b200._lib")
    L = lib.load()
    assert lib.device_status(clear=True) == 0
    res = ctypes.c_int(-1)
    lib.check(L.vomni_selftest_bounded_wait(50000, ctypes.byref(res), torch.cuda.current_stream().cuda_stream), "selftest")
    assert res.value == 0, "the wait must give up, not complete"
    assert lib.device_status(clear=True) == 0x1000 + 0x7F
    assert lib.device_status(clear=False) == 0
    # the context is still usable: a real attention call runs and is correct
    g = torch.Generator().manual_seed(0)
    q, k, v = ((torch.randn(1, 256, 2, 128, generator=g) * 0.5).to(torch.bfloat16).to(dev) for _ in range(3))
    o = pkg.ring_attention_const_max_fwd(q, k, v)
    ref = torch.softmax((q.float().transpose(1, 2) @ k.float().transpose(1, 2).transpose(-1, -2)) / math.sqrt(128), -1) @ v.float().transpose(1, 2)
    assert torch.allclose(o.float(), ref, atol=2e-2)
    assert lib.device_status() == 0


def test_ready_word_wait_posted_and_never_posted(pkg, dev):
    """The ring's in-kernel block-ready gate: a word posted by the stream memory operation releases
    the wait; a word nothing posts makes it give up with its status code, and the context survives."""
    lib = import_module("vllm-omni-neuron_b200._lib")
    L = lib.load()
    st = torch.cuda.current_stream().cuda_stream
    assert lib.device_status(clear=True) == 0
    res = ctypes.c_int(-1)
    lib.check(L.vomni_selftest_ready_wait(200000, 1, ctypes.byref(res), st), "selftest posted")
    assert res.value == 1
    assert lib.device_status() == 0
    res = ctypes.c_int(-1)
    lib.check(L.vomni_selftest_ready_wait(50000, 0, ctypes.byref(res), st), "selftest never posted")
    assert res.value == 0, "the wait must give up, not complete"
    assert lib.device_status(clear=True) == 0x1000 + 0x7E
    assert lib.device_status(clear=False) == 0
    g = torch.Generator().manual_seed(1)
    q, k, v = ((torch.randn(1, 200, 3, 128, generator=g) * 0.5).to(torch.bfloat16).to(dev) for _ in range(3))
    o = pkg.ring_attention_const_max_fwd(q, k, v)
    ref = torch.softmax((q.float().transpose(1, 2) @ k.float().transpose(1, 2).transpose(-1, -2)) / math.sqrt(128), -1) @ v.float().transpose(1, 2)
    assert torch.allclose(o.float(), ref, atol=2e-2)
    assert lib.device_status() == 0


def test_selftest_rejects_bad_budget(pkg, dev):
    lib = import_module("vllm-omni-neuron_b200._lib")
    res = ctypes.c_int(-1)
    assert lib.load().vomni_selftest_bounded_wait(0, ctypes.byref(res), None) == 1
    assert lib.load().vomni_selftest_ready_wait(0, 0, ctypes.byref(res), None) == 1
    assert lib.load().vomni_selftest_ready_wait(1000, 2, ctypes.byref(res), None) == 1
