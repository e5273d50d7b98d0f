"""CPU checks of the C ABI: the library builds/loads and exports every declared entry point;
host-side argument validation works without a GPU (no compute calls)."""

import ctypes

import pytest


@pytest.fixture(scope="module")
def lib(pkg):
    pkg.build()
    from importlib import import_module

    return import_module("vllm-omni-neuron_b200._lib")


def test_exports_every_declared_symbol(lib):
    L = lib.load()
    declared = lib.declared_symbols()
    assert len(declared) >= 7
    for name in declared:
        assert hasattr(L, name), f"{name} declared in include/vomni_b200.h but not exported"
    # the ctypes signature table covers exactly the declared ABI
    assert set(declared) == set(lib.SIGNATURES), set(declared) ^ set(lib.SIGNATURES)


def test_strerror_and_version(lib):
    L = lib.load()
    assert L.vomni_abi_version() >= 1
    assert lib.strerror(0) == "ok"
    assert "shape" in lib.strerror(2)


def test_host_validation_without_gpu(lib):
    """Argument checks run before any CUDA call."""
    L = lib.load()
    # null pointers
    assert L.vomni_cm_prologue(None, None, 1, 128, 1, 128, None, None, None) == 1
    # head_dim != 128 (the reference asserts d == 128)
    p = ctypes.c_void_p(16)
    assert L.vomni_cm_prologue(p, p, 1, 128, 1, 64, p, p, None) == 2
    # misaligned pointer
    q = ctypes.c_void_p(18)
    assert L.vomni_cm_prologue(q, q, 1, 128, 1, 128, p, p, None) == 3
    # key range outside the tensor
    assert L.vomni_cm_attend(p, p, p, 1, 128, 100, 50, 60, 1, 128, 0.1, p, p, p, p, 2, p, None, None) == 2
    # unknown flag
    assert L.vomni_cm_attend(p, p, p, 1, 128, 128, 0, 128, 1, 128, 0.1, p, p, p, p, 64, p, None, None) == 1
    # workspace too small
    assert L.vomni_cm_attention_local(p, p, p, p, None, 1, 128, 1, 128, 0.1, 0, p, 16, None) == 8
    assert L.vomni_cm_workspace_bytes(1, 128, 2, 128) >= 2 * 128 * 4


def test_host_validation_new_entry_points(lib):
    """The FFN FP8 GEMMs, the CFG combine and the ready-wait self-test check their arguments before
    any CUDA call."""
    L = lib.load()
    p = ctypes.c_void_p(16)
    q = ctypes.c_void_p(18)
    assert L.vomni_cfg_combine(None, p, p, 8, 0, 1.0, None) == 1  # null pointer
    assert L.vomni_cfg_combine(p, p, p, 8, 7, 1.0, None) == 1  # unknown dtype
    assert L.vomni_cfg_combine(p, p, p, 0, 1, 1.0, None) == 0  # nothing to do
    assert L.vomni_cfg_combine(q, p, p, 8, 1, 1.0, None) == 3  # misaligned
    # up: h % 128 != 0; i % 256 != 0
    assert L.vomni_ffn_fp8_up(p, p, p, p, None, 8, 100, 512, p, p, None) == 2
    assert L.vomni_ffn_fp8_up(p, p, p, p, None, 8, 256, 200, p, p, None) == 2
    # down: gate without residual; t not a multiple of gate_rows
    assert L.vomni_ffn_fp8_down(p, p, p, p, p, None, 8, 512, 256, None, p, 8, p, None) == 1
    assert L.vomni_ffn_fp8_down(p, p, p, p, p, None, 8, 512, 256, p, p, 3, p, None) == 2
    res = ctypes.c_int(-1)
    assert L.vomni_selftest_ready_wait(0, 0, ctypes.byref(res), None) == 1
    assert L.vomni_selftest_ready_wait(100, 3, ctypes.byref(res), None) == 1
