"""Const-max (ring) attention: the reference's kernel-call API and attention processor on B200.

* :func:`ring_attention_const_max_fwd` keeps the signature and return contract of the NKI kernel
  (vllm_omni_neuron/kernels/nkilib/experimental/attention/ring_attention_const_max_fwd.py:958-1017):
  token-major ``q, k, v [b, S_loc, h, 128]`` bf16 in, head-major ``o [b, h, S_loc, 128]`` out
  (plus ``lse [b, h, 128, ceil(S_loc/128)]`` fp32 when ``training``); ``softmax_scale`` defaults
  to ``1/sqrt(d)``; ``kv_prefetch_depth`` is clamped to ``[1, num_workers-1]``; shape contract
  violations raise ``AssertionError`` as the kernel's ``kernel_assert`` does (:1019-1031).
* :func:`wan_cp_self_attention` keeps the attention-processor signature
  (vllm_omni_neuron/diffusion/models/wan2_2/wan2_2_transformer.py:806-847) and returns the d-major
  ``[B, N, D, S_loc]`` layout directly from the kernel epilogue (the reference transposes after the
  kernel, :836).

All compute runs in ``libvomni_b200.so`` (sm_100a). There is no fallback path: a missing library or
a non-sm_100 device raises.

Host-resident inputs (B200 extension): when q, k and v are pinned CPU tensors, both entry points
stream them to the current CUDA device in head groups — the copy of group i+1 (copy engine, 2-D
strided copies straight out of the token-major host layout) overlaps the attention of group i, and
the result of group i returns to pinned host memory while group i+1 computes. Heads are
independent, so the result is identical to the device-resident call; the output is a pinned CPU
tensor, complete on return.
"""

from __future__ import annotations

import math

import torch

from . import _lib

_HEAD_DIM = 128


def _check_qkv(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor):
    assert q.dim() == 4 and k.dim() == 4 and v.dim() == 4, "q, k, v must be token-major [b, seqlen, h, d]"
    b, s, h, d = q.shape
    assert k.shape[2] == h, "expects q_heads == kv_heads, broadcast before calling"
    assert d == _HEAD_DIM, f"head_dim must be 128, got {d}"
    assert tuple(k.shape) == (b, s, h, d) and tuple(v.shape) == (b, s, h, d), (
        f"q and k must be token-major [b, seqlen, h, d]; got q={tuple(q.shape)}, k={tuple(k.shape)}"
    )
    for name, t in (("q", q), ("k", k), ("v", v)):
        if t.dtype != torch.bfloat16:
            raise TypeError(f"{name} must be bfloat16, got {t.dtype}")
        if not t.is_cuda:
            raise RuntimeError(f"{name} must be a CUDA tensor (the B200 kernel has no CPU path)")
    return b, s, h, d


def token_major(t: torch.Tensor) -> tuple[torch.Tensor, int]:
    """(tensor, token stride in elements) for a token-major ``[b, s, h, d]`` view.

    Views whose heads are dense inside a token row (for example the Q/K/V column slices of a fused
    ``[b, s, 3*h*d]`` projection, ``tensor_split`` in row_mx_modules.py:390) are passed through with
    their row stride; anything else is made contiguous."""
    b, s, h, d = t.shape
    st = t.stride()
    ok = (
        st[3] == 1 and st[2] == d and st[1] >= h * d and st[1] % 8 == 0
        and (b == 1 or st[0] == s * st[1]) and t.data_ptr() % 16 == 0
    )
    if ok:
        return t, st[1]
    return t.contiguous(), h * d


_HOST_GROUP_HEADS = 5


def _host_group_heads(s: int, h: int, dev: torch.device, world: int = 1) -> int:
    """Heads per host-streamed group. One rank (PCIe-bound, cheap calls): 5, the finest split that
    measured fastest. A CP ring (every call pays an all-reduce, block copies and several pass
    launches): the finest split whose passes still fill two waves of CTA pairs (a pair covers 512
    query rows of one head on two SMs), e.g. 20 heads for S_loc = 4095, 10 for 8190."""
    if world <= 1:
        return min(h, _HOST_GROUP_HEADS)
    pairs_per_head = -(-s // 512)
    slots = max(1, torch.cuda.get_device_properties(dev).multi_processor_count // 2)
    g_min = max(_HOST_GROUP_HEADS, -(-2 * slots // pairs_per_head))
    groups = max(1, h // g_min)
    return -(-h // groups)
_AUX_STREAMS: dict = {}


def _aux_streams(dev: torch.device):
    """(host->device copy stream, device->host copy stream, second compute stream) of a device."""
    key = dev.index
    if key not in _AUX_STREAMS:
        _AUX_STREAMS[key] = tuple(torch.cuda.Stream(dev) for _ in range(3))
    return _AUX_STREAMS[key]


def _copy_2d(dst_ptr, dpitch, src_ptr, spitch, width, height, stream):
    _lib.check(_lib.load().vomni_memcpy_2d_async(dst_ptr, dpitch, src_ptr, spitch, width, height, stream.cuda_stream),
               "vomni_memcpy_2d_async")


def _host_streamed(fn, q, k, v, *, out_layout: str, training: bool, alternate: bool = True,
                   group_heads: int | None = None, world: int = 1):
    """Run ``fn(q_dev, k_dev, v_dev) -> out | (out, lse)`` over head groups of pinned host q/k/v
    (``group_heads`` heads per group, default ``_host_group_heads`` for a ring of ``world`` ranks).

    Group g's host->device copies run on a copy stream, its attention alternates between the
    caller's stream and a second compute stream (so one group's tail wave overlaps the next group;
    ``alternate=False`` keeps every group on the caller's stream, as a ring context's buffers
    require), and its output returns on a second copy stream. Returns pinned host tensors."""
    b, s, h, d = q.shape
    for name, t in (("q", q), ("k", k), ("v", v)):
        if t.device.type != "cpu" or not t.is_pinned():
            raise ValueError(f"host-resident {name} must be a pinned CPU tensor (tensor.pin_memory())")
        if t.dtype != torch.bfloat16 or tuple(t.shape) != (b, s, h, d):
            raise TypeError(f"{name} must be bfloat16 [b, s, h, d] like q")
    q, k, v = (t if t.is_contiguous() else t.contiguous().pin_memory() for t in (q, k, v))
    dev = torch.device("cuda", torch.cuda.current_device())
    main = torch.cuda.current_stream(dev)
    h2d, d2h, alt = _aux_streams(dev)
    esz = 2
    dq, dk, dv = (torch.empty((b, s, h, d), dtype=torch.bfloat16, device=dev) for _ in range(3))
    o_shape = (b, h, d, s) if out_layout == "bhds" else (b, h, s, d)
    host_o = torch.empty(o_shape, dtype=torch.bfloat16, pin_memory=True)
    n_lse = 128 * (-(-s // 128))
    host_lse = torch.empty((b, h, 128, n_lse // 128), dtype=torch.float32, pin_memory=True) if training else None
    gh = max(1, int(group_heads or _host_group_heads(s, h, dev, world)))
    row = h * d * esz
    h2d.wait_stream(main)
    alt.wait_stream(main)
    keep = []
    for gi, h0 in enumerate(range(0, h, gh)):
        h1 = min(h, h0 + gh)
        w = (h1 - h0) * d * esz
        for src, dst in ((q, dq), (k, dk), (v, dv)):
            _copy_2d(dst.data_ptr() + h0 * d * esz, row, src.data_ptr() + h0 * d * esz, row, w, b * s, h2d)
        arrived = torch.cuda.Event()
        arrived.record(h2d)
        cs = alt if (alternate and gi % 2) else main
        cs.wait_event(arrived)
        with torch.cuda.stream(cs):
            res = fn(dq[:, :, h0:h1], dk[:, :, h0:h1], dv[:, :, h0:h1])
        o, lse = res if training else (res, None)
        done = torch.cuda.Event()
        done.record(cs)
        d2h.wait_event(done)
        per_head = o[0, 0].numel() * esz
        _copy_2d(host_o.data_ptr() + h0 * per_head, h * per_head, o.data_ptr(), (h1 - h0) * per_head,
                 (h1 - h0) * per_head, b, d2h)
        if training:
            lh = 128 * (n_lse // 128) * 4
            _copy_2d(host_lse.data_ptr() + h0 * lh, h * lh, lse.data_ptr(), (h1 - h0) * lh, (h1 - h0) * lh, b, d2h)
        keep.append(res)
    d2h.synchronize()  # every group's copy-out waited for its compute, which waited for its copy-in
    main.wait_stream(alt)
    main.wait_stream(d2h)
    del keep
    return (host_o, host_lse) if training else host_o


def _stream_ptr(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def attention_local(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    softmax_scale: float | None = None,
    *,
    out_layout: str = "bhsd",
    training: bool = False,
):
    """Single-rank const-max attention (``num_workers == 1``): prologue norms + one final pass.

    ``out_layout``: ``"bhsd"`` (kernel layout) or ``"bhds"`` (d-major, the attention-processor
    layout). Returns ``o`` or ``(o, lse)``.
    """
    b, s, h, d = _check_qkv(q, k, v)
    q, q_stride = token_major(q)
    k, k_stride = token_major(k)
    v, v_stride = token_major(v)
    if k_stride != v_stride:  # K and V share one stride argument
        k, v = k.contiguous(), v.contiguous()
        k_stride = h * d
    scale = float(softmax_scale) if softmax_scale else 1.0 / math.sqrt(d)
    lib = _lib.load()
    flags = 0
    if out_layout == "bhds":
        flags |= _lib.CM_OUT_DMAJOR
        out = torch.empty((b, h, d, s), dtype=torch.bfloat16, device=q.device)
    elif out_layout == "bhsd":
        out = torch.empty((b, h, s, d), dtype=torch.bfloat16, device=q.device)
    else:
        raise ValueError(f"unknown out_layout {out_layout!r}")
    lse = None
    if training:
        flags |= _lib.CM_LSE
        lse = torch.zeros((b, h, 128, -(-s // 128)), dtype=torch.float32, device=q.device)
    ws_bytes = lib.vomni_cm_workspace_bytes(b, s, h, d)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device)
    rc = lib.vomni_cm_attention_local_strided(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), lse.data_ptr() if lse is not None else None,
        b, s, h, d, q_stride, k_stride, scale, flags, ws.data_ptr(), ws_bytes, _stream_ptr(q.device),
    )
    _lib.check(rc, "vomni_cm_attention_local_strided")
    return (out, lse) if training else out


def ring_attention_const_max_fwd(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    replica_groups: tuple | None = None,
    num_workers: int = 1,
    softmax_scale: float | None = None,
    training: bool = False,
    lse_dtype: torch.dtype = torch.float32,
    kv_prefetch_depth: int = 2,
    *,
    group=None,
    out_layout: str = "bhsd",
):
    """Fixed-max ring attention forward (non-causal); see the module docstring for the contract.

    ``group`` (B200 addition): the ``torch.distributed`` process group of this rank's ring when
    ``num_workers > 1``; defaults to the group matching ``replica_groups`` (built once per ring).
    Pinned host q/k/v are streamed by head groups (module docstring) and give host results.
    """
    if q.device.type == "cpu" and k.device.type == "cpu" and v.device.type == "cpu":
        assert q.dim() == 4 and q.shape[-1] == _HEAD_DIM, "q, k, v must be token-major [b, seqlen, h, 128]"

        def dev_call(qd, kd, vd):
            return ring_attention_const_max_fwd(qd, kd, vd, replica_groups, num_workers, softmax_scale, training,
                                                torch.float32, kv_prefetch_depth, group=group, out_layout=out_layout)

        res = _host_streamed(dev_call, q, k, v, out_layout=out_layout, training=training, alternate=num_workers <= 1,
                             world=num_workers)
        return (res[0], res[1].to(lse_dtype)) if training else res
    _check_qkv(q, k, v)
    if num_workers <= 1:
        res = attention_local(q, k, v, softmax_scale, out_layout=out_layout, training=training)
    else:
        from .ring import ring_attention

        res = ring_attention(
            q, k, v, replica_groups=replica_groups, num_workers=num_workers, softmax_scale=softmax_scale,
            training=training, kv_prefetch_depth=kv_prefetch_depth, group=group, out_layout=out_layout,
        )
    if training:
        o, lse = res
        return o, lse.to(lse_dtype)
    return res


def wan_cp_self_attention(query, key, value, scale, cp_size, cp_group, cp_replica_groups):
    """Context-parallel self-attention core (wan2_2_transformer.py:806-847).

    ``query/key/value``: token-major ``[B, local_S, N, D]`` bf16. Returns d-major ``[B, N, D, local_S]``.
    ``cp_group``: a ``torch.distributed`` ProcessGroup, or an object exposing one as
    ``device_group`` (vLLM's GroupCoordinator), or None when ``cp_size == 1``. The ring kernel runs at
    every ``cp_size`` (``num_workers=1`` included); there is no all-gather fallback.
    """
    group = getattr(cp_group, "device_group", cp_group)
    return ring_attention_const_max_fwd(
        query, key, value, replica_groups=cp_replica_groups, num_workers=int(cp_size), softmax_scale=scale,
        group=group, out_layout="bhds",
    )
