"""CPU restatements of the reference's self-attention math (numpy, fp32 arithmetic).

Two algorithms:

* ``torch_attend``: exact non-causal attention, restating ``_torch_attend``
  (vllm_omni_neuron/diffusion/models/wan2_2/wan2_2_transformer.py:640-650):
  ``softmax(scale * Q @ K^T)`` in fp32, ``@ V`` in fp32, cast back to bf16.
  Layout ``[B, N, S, D]``.

* ``const_max_ring_attention``: the const-max ring kernel
  (vllm_omni_neuron/kernels/nkilib/experimental/attention/ring_attention_const_max_fwd.py
  and attention_const_max.py), restated step by step with the reference's rounding
  points:
    - per-token ||q_i||^2 and per-head max_j ||k_j||^2 in fp32 off the bf16 inputs
      (ring_attention_const_max_fwd.py:336-398);
    - global key max over the whole ring (all_reduce max, :1196-1205);
    - c_i = sqrt(scale^2 * kmax^2 * ||q_i||^2), stored bf16 (:559-642);
    - Q pre-scaled by softmax_scale and rounded to bf16 (attention_const_max.py:148-150);
    - scores = Q_s @ K^T accumulated in fp32 (trn2 PSUM) or rounded to bf16 (trn3 PSUM,
      attention_const_max.py:284), shifted = fp16(scores - c) (:311-327, 395-408),
      P = bf16(exp(shifted)) (:409-415);
    - O_aug = [sum P V | sum P] in fp32, pure-add across ring steps (:473-490;
      ring_attention_const_max_fwd.py:1328-1398); step s on rank r consumes the block
      that started on rank (r - s) mod N (collective_permute to the next rank, :130-144);
    - o = bf16(O / max(sum, 1e-37)); lse = c + log(max(sum, 1e-37)) in the
      [b, h, 128, ceil(S/128)] layout (:655-804).

Token-major ``[b, S_loc, h, d]`` in, head-major ``[b, h, S_loc, d]`` out, exactly
as the kernel. All arrays are float32 holding bf16-representable values.
"""

from __future__ import annotations

import numpy as np

from .numerics import bf16_round, fp16_round

SUM_CLAMP = 1e-37  # ring_attention_const_max_fwd.py:663


def torch_attend(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float, q_block: int = 1024) -> np.ndarray:
    """Exact attention, wan2_2_transformer.py:640-650. ``[B,N,S,D]`` -> ``[B,N,S,D]`` (bf16 values)."""
    q = np.asarray(q, np.float32)
    k = np.asarray(k, np.float32)
    v = np.asarray(v, np.float32)
    B, N, S, D = q.shape
    out = np.empty((B, N, S, v.shape[-1]), np.float32)
    for b in range(B):
        for n in range(N):
            kt = k[b, n].T
            for s0 in range(0, S, q_block):
                sc = (q[b, n, s0:s0 + q_block] * np.float32(scale)) @ kt
                sc = sc - sc.max(axis=-1, keepdims=True)
                p = np.exp(sc)
                p /= p.sum(axis=-1, keepdims=True)
                out[b, n, s0:s0 + q_block] = p @ v[b, n]
    return bf16_round(out)


def const_max_bounds(qs, ks, scale: float):
    """Per-rank per-token ||q||^2 and the ring-global per-head max ||k||^2.

    Returns (qn2 list of [b, h, S_loc] fp32, kmax2 [b, h] fp32, c list of [b, h, S_loc] bf16-valued).
    """
    qn2 = [np.einsum("bshd,bshd->bhs", q.astype(np.float32), q.astype(np.float32)) for q in qs]
    kmax_local = [np.einsum("bshd,bshd->bhs", k.astype(np.float32), k.astype(np.float32)).max(axis=-1) for k in ks]
    kmax2 = np.maximum.reduce(kmax_local)
    s2 = np.float32(scale) * np.float32(scale)
    cs = [bf16_round(np.sqrt(s2 * kmax2[:, :, None] * x)) for x in qn2]
    return qn2, kmax2, cs


def const_max_partial(q_tok, k_tok, v_tok, c, scale: float, scores_bf16: bool = False, q_block: int = 512):
    """One ring step / pass (attention_const_max.py:138-234): unnormalised ``[sum P V | sum P]`` of the
    query rows ``q_tok [b, Sq, h, d]`` against ``k_tok / v_tok [b, Sk, h, d]`` with the per-row bound
    ``c [b, h, Sq]``. Returns (acc [b, h, Sq, d] fp32, sums [b, h, Sq] fp32)."""
    qh = np.transpose(q_tok, (0, 2, 1, 3)).astype(np.float32)
    kh = np.transpose(k_tok, (0, 2, 1, 3)).astype(np.float32)
    vh = np.transpose(v_tok, (0, 2, 1, 3)).astype(np.float32)
    b, h, sq, d = qh.shape
    q_s = bf16_round(qh * np.float32(scale))
    acc = np.zeros((b, h, sq, vh.shape[-1]), np.float32)
    ssum = np.zeros((b, h, sq), np.float32)
    for bi in range(b):
        for hi in range(h):
            kt = kh[bi, hi].T
            for s0 in range(0, sq, q_block):
                sl = slice(s0, s0 + q_block)
                sc = q_s[bi, hi, sl] @ kt
                if scores_bf16:
                    sc = bf16_round(sc)
                shifted = fp16_round(sc - c[bi, hi, sl][:, None])
                p = bf16_round(np.exp(shifted))
                acc[bi, hi, sl] += p @ vh[bi, hi]
                ssum[bi, hi, sl] += p.sum(axis=-1)
    return acc, ssum


def const_max_normalize(acc, ssum, c=None, training: bool = False):
    """o = bf16(acc / max(sum, 1e-37)) and lse = c + log(max(sum, 1e-37)) in the [b, h, 128, groups]
    layout (ring_attention_const_max_fwd.py:655-804)."""
    clamped = np.maximum(ssum, np.float32(SUM_CLAMP))
    o = bf16_round(acc * (np.float32(1.0) / clamped)[..., None])
    if not training:
        return o
    b, h, s_loc = ssum.shape
    groups = -(-s_loc // 128)
    lse_tok = c + np.log(clamped)
    lse = np.zeros((b, h, 128, groups), np.float32)
    for g in range(groups):
        rows = min(128, s_loc - g * 128)
        lse[:, :, :rows, g] = lse_tok[:, :, g * 128:g * 128 + rows]
    return o, lse


def const_max_ring_attention(
    qs,
    ks,
    vs,
    softmax_scale: float | None = None,
    training: bool = False,
    scores_bf16: bool = False,
    q_block: int = 512,
):
    """Const-max ring attention over ``len(qs)`` ranks.

    ``qs/ks/vs``: per-rank lists of token-major ``[b, S_loc, h, d]`` float32 arrays (bf16 values).
    Returns the per-rank list of ``o [b, h, S_loc, d]`` (and ``lse [b, h, 128, ceil(S_loc/128)]``
    when ``training``).
    """
    n = len(qs)
    b, s_loc, h, d = qs[0].shape
    scale = float(softmax_scale) if softmax_scale else 1.0 / float(d) ** 0.5
    _, _, cs = const_max_bounds(qs, ks, scale)
    outs, lses = [], []
    for r in range(n):
        acc = np.zeros((b, h, s_loc, d), np.float32)
        ssum = np.zeros((b, h, s_loc), np.float32)
        for step in range(n):
            src = (r - step) % n
            a, sm = const_max_partial(qs[r], ks[src], vs[src], cs[r], scale, scores_bf16, q_block)
            acc += a
            ssum += sm
        res = const_max_normalize(acc, ssum, cs[r], training)
        if training:
            outs.append(res[0])
            lses.append(res[1])
        else:
            outs.append(res)
    if training:
        return outs, lses
    return outs


def wan_cp_self_attention_oracle(qs, ks, vs, scale):
    """What ``wan_cp_self_attention`` (wan2_2_transformer.py:806-847) returns on each CP rank:
    exact attention of the rank's query rows against the full (ring-gathered) K/V, d-major
    ``[B, N, D, S_loc]``. The fallback path (all-gather K/V + ``_torch_attend``) is the
    mathematical definition the ring kernel must reproduce.
    """
    kf = np.concatenate(ks, axis=1)
    vf = np.concatenate(vs, axis=1)
    kh = np.transpose(kf, (0, 2, 1, 3))
    vh = np.transpose(vf, (0, 2, 1, 3))
    outs = []
    for q in qs:
        qh = np.transpose(q, (0, 2, 1, 3))
        o = torch_attend(qh, kh, vh, scale)
        outs.append(np.ascontiguousarray(np.transpose(o, (0, 1, 3, 2))))
    return outs


def attention_flops(b: int, h: int, s_q: int, s_k: int, d: int) -> float:
    """Algorithmic FLOPs of one non-causal attention: 2 GEMMs of 2*S_q*S_k*d each, per head."""
    return 4.0 * b * h * s_q * s_k * d
