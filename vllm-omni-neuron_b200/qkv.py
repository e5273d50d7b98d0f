"""FP8 QKV projection with the across-heads RMS norm and rotate-half RoPE epilogue — the reference's
``row_mx_qkv_proj`` (vllm_omni_neuron/diffusion/quantization/row_mx_kernels.py:48-111).

Semantics (ROW_MX mode of ``_qkv_cte_mx_impl``, kernels/nkilib/core/qkv/qkv_cte.py:2725-4114):
``Y = (Xq @ Wq) * row_scale * chan_scale + bias`` (bf16), then — when ``qk_norm_pre_rope`` asks for
``RMS_NORM_ACROSS_HEADS`` — per-token ``inv = rsqrt(sum(Y_seg^2) / (n_heads*d) + eps)`` over the whole
Q (and K) segment, ``Y_seg * gamma`` and rotate-half RoPE with ``inv`` folded in (``fused_rope``).

Weight layout: the B200 kernel reads ``W`` as ``[I, H]`` fp8 (K-major rows, 16-byte aligned), the
natural tcgen05 B operand. :func:`repack_mx_contiguous` converts the reference's MX_CONTIGUOUS
``[H//4, I, 4]`` pack (row_mx_loaders.py:194-223) once at load time; ``row_mx_qkv_proj`` also
accepts the 3-D pack directly and repacks it per call.

Activation layout: the packed ``[..., H + 4]`` rows from ``adaln_modulate(quant="row")`` (fp32 scale
in the 4 tail bytes), or the ``(codes [..., H], scales [...])`` pair from
``adaln_modulate(quant="row", row_layout="split")``, which the GEMM reads with TMA directly (packed
rows are 5124 bytes apart, not a 16-byte multiple, so they are unpacked first).
"""

from __future__ import annotations

import torch

from . import _lib



def repack_mx_contiguous(w3: torch.Tensor) -> torch.Tensor:
    """``[H//4, I, 4]`` (four consecutive contraction values innermost) -> ``[I, H]``."""
    hq, i, four = w3.shape
    assert four == 4, "expected the [H//4, I, 4] MX_CONTIGUOUS pack"
    return w3.permute(1, 0, 2).reshape(i, hq * 4).contiguous()


def quantize_qkv_weight(w: torch.Tensor, q_size: int, kv_size: int):
    """Per-tensor FP8 e4m3fn quantisation of a fused ``[H, I]`` Q|K|V weight, one scale per tensor
    (the ComfyUI checkpoint scalars expanded per channel, row_mx_loaders.py:115-140, 246-260).
    Returns (codes ``[I, H]`` float8_e4m3fn, chan_scale ``[I]`` fp32)."""
    w = w.float()
    chan = torch.empty(w.shape[1], dtype=torch.float32, device=w.device)
    codes = torch.empty_like(w)
    for lo, hi in ((0, q_size), (q_size, q_size + kv_size), (q_size + kv_size, q_size + 2 * kv_size)):
        if hi == lo:  # a single projection (kv_size = 0), e.g. the cross-attention's separate Q, K, V
            continue
        sc = torch.clamp(w[:, lo:hi].abs().amax() / 448.0, min=1e-12)
        codes[:, lo:hi] = w[:, lo:hi] / sc
        chan[lo:hi] = sc
    return codes.t().contiguous().to(torch.float8_e4m3fn), chan


def pack_mx_scales(scales: torch.Tensor) -> torch.Tensor:
    """UE8M0 scales ``[rows, k/32]`` (row-major, as ``adaln_modulate(quant="mx32")`` emits them) ->
    the tcgen05 scale-atom tiling the block-scaled GEMM streams (``vomni_mx_pack_scales``)."""
    rows, kb = scales.shape[-2] if scales.dim() > 1 else 1, scales.shape[-1]
    sc = scales.reshape(-1, kb).contiguous()
    rows = sc.shape[0]
    L = _lib.load()
    nbytes = L.vomni_mx_packed_scales_bytes(rows, kb * 32)
    if nbytes == 0:
        raise ValueError(f"MX-32 scales need k % 128 == 0, got k = {kb * 32}")
    out = torch.empty(nbytes, dtype=torch.uint8, device=sc.device)
    _lib.check(L.vomni_mx_pack_scales(sc.data_ptr(), rows, kb * 32, out.data_ptr(),
                                      torch.cuda.current_stream(sc.device).cuda_stream), "vomni_mx_pack_scales")
    return out


def quantize_qkv_weight_mx32(w: torch.Tensor):
    """MX-32 quantisation of a fused ``[H, I]`` weight along the contraction (one UE8M0 scale per 32
    consecutive H values of every output channel, the ``_mx_dequant`` format,
    adaln_quant_torch.py:151-175). Returns (codes ``[I, H]`` fp8, scales ``[I, H/32]`` uint8,
    packed scales for the GEMM)."""
    from .adaln import adaln_modulate

    codes, scales = adaln_modulate(w.t().contiguous().to(torch.bfloat16), None, None, eps=0.0, norm_type="none",
                                   quant="mx32")
    return codes, scales, pack_mx_scales(scales)


def _wants_across_heads_norm(cfg) -> bool:
    if cfg is None or cfg is False:
        return False
    if cfg is True or isinstance(cfg, str):
        return True
    for name in ("q_norm", "k_norm"):
        v = getattr(cfg, name, None)
        if v is not None and "ACROSS_HEADS" not in str(getattr(v, "name", v)).upper():
            raise NotImplementedError(f"only RMS_NORM_ACROSS_HEADS qk-norm is implemented, got {v}")
    return True


def _apply_norm_rope(y, T, I, num_heads, num_kv_heads, head_dim, sumsq, norm, rope, cfg, norm_eps, gamma_q, gamma_k,
                     cos_cache, sin_cache, st):
    """Across-heads RMS norm (+ gamma) and rotate-half RoPE on the Q/K segments of y, in place."""
    if norm:
        eps = float(getattr(cfg, "eps", norm_eps) or norm_eps)
    else:
        # RoPE without the across-heads norm: inv = 1 via a zero sum and eps = 1.
        sumsq.zero_()
        eps = 1.0
    gq = gamma_q.reshape(-1).to(torch.bfloat16).contiguous() if (norm and gamma_q is not None) else None
    gk = gamma_k.reshape(-1).to(torch.bfloat16).contiguous() if (norm and gamma_k is not None) else None
    cs = sn = None
    if rope:
        if cos_cache is None or sin_cache is None:
            raise ValueError("fused_rope needs cos_cache and sin_cache")
        cs = cos_cache.reshape(-1, head_dim).float().contiguous()
        sn = sin_cache.reshape(-1, head_dim).float().contiguous()
        if cs.shape[0] != T:
            if cs.shape[0] * (T // cs.shape[0]) == T:  # per-position caches shared across the batch
                cs = cs.repeat(T // cs.shape[0], 1)
                sn = sn.repeat(T // sn.shape[0], 1)
            else:
                raise ValueError(f"cos/sin caches have {cs.shape[0]} rows for {T} tokens")
    ptr = lambda t: t.data_ptr() if t is not None else None
    _lib.check(
        _lib.load().vomni_qk_norm_rope(y.data_ptr(), T, I, num_heads, num_kv_heads, head_dim, sumsq.data_ptr(), eps,
                                       ptr(gq), ptr(gk), ptr(cs), ptr(sn), st),
        "vomni_qk_norm_rope",
    )


def row_mx_qkv_proj(
    packed_hidden,
    weight: torch.Tensor,
    weight_scales: torch.Tensor,
    bias: torch.Tensor | None,
    *,
    num_heads: int,
    head_dim: int,
    num_kv_heads: int,
    fused_rope: bool = False,
    cos_cache: torch.Tensor | None = None,
    sin_cache: torch.Tensor | None = None,
    qk_norm_pre_rope=None,
    qk_norm_pre_rope_q_gamma: torch.Tensor | None = None,
    qk_norm_pre_rope_k_gamma: torch.Tensor | None = None,
    norm_eps: float = 1e-6,
    replica_groups=None,
    output_layout=None,
) -> torch.Tensor:
    """``[B, S, I]`` bf16 (BSD), I = (num_heads + 2*num_kv_heads) * head_dim."""
    if output_layout is not None and "BSD" not in str(getattr(output_layout, "name", output_layout)).upper():
        raise NotImplementedError("only the BSD output layout is implemented")
    if replica_groups and any(len(g) > 1 for g in replica_groups):
        raise NotImplementedError("TP > 1 (cross-rank across-heads norm) is not implemented; CP covers the sequence")
    if head_dim != 128:
        raise ValueError(f"head_dim must be 128, got {head_dim}")
    L = _lib.load()
    if isinstance(packed_hidden, (tuple, list)):
        codes, row_scale = packed_hidden
        lead = tuple(codes.shape[:-1])
        H = codes.shape[-1]
        dev = codes.device
        codes = codes.contiguous()
        row_scale = row_scale.reshape(-1).float().contiguous()
    else:
        lead = tuple(packed_hidden.shape[:-1])
        H = packed_hidden.shape[-1] - 4
        dev = packed_hidden.device
        T0 = packed_hidden.numel() // (H + 4)
        codes = torch.empty(lead + (H,), dtype=torch.float8_e4m3fn, device=dev)
        row_scale = torch.empty(T0, dtype=torch.float32, device=dev)
        _lib.check(
            L.vomni_qkv_unpack_rows(packed_hidden.contiguous().data_ptr(), T0, H, codes.data_ptr(), row_scale.data_ptr(),
                                    torch.cuda.current_stream(dev).cuda_stream),
            "vomni_qkv_unpack_rows",
        )
    T = codes.numel() // H
    if weight.dim() == 3:
        weight = repack_mx_contiguous(weight)
    I = weight.shape[0]
    assert weight.shape[1] == H, f"weight contraction {weight.shape[1]} != activation width {H}"
    q_dim, kv_dim = num_heads * head_dim, num_kv_heads * head_dim
    assert q_dim + 2 * kv_dim == I, f"weight rows {I} != (num_heads + 2*num_kv_heads) * head_dim"
    chan = weight_scales.reshape(-1).float().contiguous()
    b = bias.reshape(-1).to(torch.bfloat16).contiguous() if bias is not None else None
    y = torch.empty(lead + (I,), dtype=torch.bfloat16, device=dev)
    norm = _wants_across_heads_norm(qk_norm_pre_rope)
    rope = bool(fused_rope)
    sumsq = None
    if norm or rope:
        sumsq = torch.empty(T, (q_dim + kv_dim) // head_dim, dtype=torch.float32, device=dev)
    st = torch.cuda.current_stream(dev).cuda_stream
    _lib.check(
        L.vomni_qkv_fp8_gemm(codes.data_ptr(), row_scale.data_ptr(), weight.contiguous().data_ptr(), chan.data_ptr(),
                             b.data_ptr() if b is not None else None, T, H, I, q_dim, kv_dim, y.data_ptr(),
                             sumsq.data_ptr() if sumsq is not None else None, st),
        "vomni_qkv_fp8_gemm",
    )
    if norm or rope:
        _apply_norm_rope(y, T, I, num_heads, num_kv_heads, head_dim, sumsq, norm, rope, qk_norm_pre_rope, norm_eps,
                         qk_norm_pre_rope_q_gamma, qk_norm_pre_rope_k_gamma, cos_cache, sin_cache, st)
    return y


def mx32_qkv_proj(
    x,
    w_codes: torch.Tensor,
    w_scales_packed: torch.Tensor,
    bias: torch.Tensor | None,
    *,
    num_heads: int,
    head_dim: int,
    num_kv_heads: int,
    fused_rope: bool = False,
    cos_cache: torch.Tensor | None = None,
    sin_cache: torch.Tensor | None = None,
    qk_norm_pre_rope=None,
    qk_norm_pre_rope_q_gamma: torch.Tensor | None = None,
    qk_norm_pre_rope_k_gamma: torch.Tensor | None = None,
    norm_eps: float = 1e-6,
) -> torch.Tensor:
    """MX-32 variant of :func:`row_mx_qkv_proj`: ``x = (codes [..., H] fp8, scales [..., H/32] u8)``
    from ``adaln_modulate(quant="mx32")``; weights from :func:`quantize_qkv_weight_mx32`. The GEMM is
    a tcgen05 block-scaled MMA (UE8M0 per 32 elements on both operands); the epilogue (bias, across-heads
    RMS norm, gamma, rotate-half RoPE) is the ROW path's."""
    if head_dim != 128:
        raise ValueError(f"head_dim must be 128, got {head_dim}")
    codes, scales = x
    lead = tuple(codes.shape[:-1])
    H = codes.shape[-1]
    dev = codes.device
    T = codes.numel() // H
    I = w_codes.shape[0]
    q_dim, kv_dim = num_heads * head_dim, num_kv_heads * head_dim
    assert q_dim + 2 * kv_dim == I and w_codes.shape[1] == H
    L = _lib.load()
    xs = pack_mx_scales(scales.reshape(T, H // 32))
    b = bias.reshape(-1).to(torch.bfloat16).contiguous() if bias is not None else None
    y = torch.empty(lead + (I,), dtype=torch.bfloat16, device=dev)
    norm = _wants_across_heads_norm(qk_norm_pre_rope)
    rope = bool(fused_rope)
    sumsq = torch.empty(T, (q_dim + kv_dim) // head_dim, dtype=torch.float32, device=dev) if (norm or rope) else None
    st = torch.cuda.current_stream(dev).cuda_stream
    _lib.check(
        L.vomni_qkv_mx32_gemm(codes.contiguous().data_ptr(), xs.data_ptr(), w_codes.contiguous().data_ptr(),
                              w_scales_packed.data_ptr(), b.data_ptr() if b is not None else None, T, H, I, q_dim,
                              kv_dim, y.data_ptr(), sumsq.data_ptr() if sumsq is not None else None, st),
        "vomni_qkv_mx32_gemm",
    )
    if norm or rope:
        _apply_norm_rope(y, T, I, num_heads, num_kv_heads, head_dim, sumsq, norm, rope, qk_norm_pre_rope, norm_eps,
                         qk_norm_pre_rope_q_gamma, qk_norm_pre_rope_k_gamma, cos_cache, sin_cache, st)
    return y
