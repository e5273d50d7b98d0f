"""CPU oracle for the const-max ring attention / adaLN-quant / FP8 QKV hot path.

TEST INFRASTRUCTURE ONLY. Nothing in the product package imports this directory:
only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl
reference`` legs of ``bench.py`` use it, and only as the checker or as the timed
CPU stand-in for the reference's own PyTorch path.

Every function restates an algorithm of the reference (reecedantin/vllm-omni-neuron,
paths relative to the project root) and cites the file:line it follows. The
restatements are pinned against golden vectors produced by importing the
reference's own torch/numpy code in the build container (``tests/golden/``):

* ``adaln``: pinned bit-exactly against ``adaln_quant_torch_ref`` and
  ``_eager_adaln`` outputs.
* ``rope``: pinned against ``WanRotaryPosEmbed`` / ``apply_rotary_emb_wan`` /
  ``_rope_rotate_half_caches`` / the de-interleave loaders.
* ``attention``: the exact-attention restatement is pinned against
  ``_torch_attend``; the const-max restatement is checked against it within the
  north-star tolerance (the reference's own validation rule for the ring
  kernel: compare against exact attention, never against another device path).
* ``qkv``: the ROW_MX epilogue has no runnable reference (its kernel is NKI);
  its pieces (dequant, across-heads RMS, rotate-half RoPE) are built from the
  pinned adaln/rope pieces and the reference's bf16 path (``DistributedRMSNorm``
  + ``apply_rotary_emb_wan``), against which it is checked through the
  de-interleave identity.
"""
