"""Generate the golden vectors that pin the CPU oracle to the reference's own code.

Run where the reference checkout is available, with its root in ``VOMNI_REFERENCE``::

    VOMNI_REFERENCE=<reference checkout> python tests/golden/make_golden.py

Only the reference's dependency-light torch/numpy pieces are executed (the NKI kernels
cannot run without a Trainium toolchain):

* ``adaln_quant_torch_ref`` and ``_mx_dequant`` (kernels/nkilib/experimental/norm/
  adaln_quant_torch.py), loaded by file path;
* ``_eager_adaln`` (diffusion/quantization/adaln_kernels.py:51-84), loaded by file path;
* ``WanRotaryPosEmbed`` / ``apply_rotary_emb_wan`` (diffusion/layers/rope.py), by file path;
* ``_mlp_ref_standard`` (kernels/nkilib/core/mlp/mlp_torch.py:401-600) in ROW_MX CTE mode, for the
  ROW_MX MLP and, stopped after its up-projection, for the ROW_MX QKV dequant-matmul arithmetic;
* ``build_fp8_dequant_mappings`` (diffusion/quantization/comfy_fp8_checkpoint.py, imported by path:
  it needs only the standard library) and ``dequantize_to_bf16`` (dequant_loaders.py:38-52, by ``ast``);
* ``_torch_attend`` (diffusion/models/wan2_2/wan2_2_transformer.py:640-650), ``_wan_o_proj``
  (:246-254) and ``_wan_mlp`` (:389-410), the latter two on their torch path (the NKI kernels'
  capability checks are stubbed to False),
  ``DistributedRMSNorm`` (:855-893), ``_rope_rotate_half_caches``
  (diffusion/quantization/row_mx_modules.py:51-76) and the de-interleave loaders
  (diffusion/quantization/row_mx_loaders.py:26-71): their modules import the Neuron SDK at
  top level, so the function definitions are extracted from the source with ``ast`` and
  executed against plain torch.

Outputs ``*.npz`` next to this script. bf16 tensors are stored as their float32 values.
"""

from __future__ import annotations

import ast
import json
import math
import importlib.util
import os
import sys
import types
from pathlib import Path

import numpy as np
import torch

_REF_ROOT = os.environ.get("VOMNI_REFERENCE")
if not _REF_ROOT:
    raise SystemExit("set VOMNI_REFERENCE to the root of the reference checkout")
REF = Path(_REF_ROOT) / "vllm_omni_neuron"
OUT = Path(__file__).resolve().parent


def _load_file(name: str, path: Path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _extract(path: Path, names: list[str], env: dict) -> dict:
    """Exec only the named top-level defs/classes of a reference module against ``env``."""
    tree = ast.parse(path.read_text())
    body = [n for n in tree.body if isinstance(n, (ast.FunctionDef, ast.ClassDef)) and n.name in names]
    missing = set(names) - {n.name for n in body}
    if missing:
        raise RuntimeError(f"{path}: missing {missing}")
    mod = ast.Module(body=body, type_ignores=[])
    code = compile(mod, str(path), "exec")
    exec(code, env)
    return {n: env[n] for n in names}


def _bf16(t: torch.Tensor) -> np.ndarray:
    return t.to(torch.bfloat16).float().numpy()


def gen_adaln(rng: torch.Generator):
    adt = _load_file("ref_adaln_quant_torch", REF / "kernels/nkilib/experimental/norm/adaln_quant_torch.py")
    T, H = 12, 128
    hidden = torch.randn(T, H, generator=rng).to(torch.bfloat16)
    hidden[3, :] = 0.0  # an all-zero row exercises the 1e-6 scale floor
    mul = (1 + 0.1 * torch.randn(H, generator=rng)).to(torch.bfloat16)
    add = (0.1 * torch.randn(H, generator=rng)).to(torch.bfloat16)
    residual = torch.randn(T, H, generator=rng).to(torch.bfloat16)
    gate = 0.5 * torch.randn(H, generator=rng)
    out = {"hidden": _bf16(hidden), "mul": _bf16(mul), "add": _bf16(add), "residual": _bf16(residual), "gate": gate.numpy()}
    cases = []
    for norm in ("layer_norm", "rms_norm", "none"):
        for quant in ("none", "row", "mx"):
            for res_mode in ("plain", "residual", "gated"):
                for ocp in ((True, False) if quant == "row" else (True,)):
                    kw = dict(norm_type=norm, quant=quant, eps=1e-6, ocp=ocp)
                    if res_mode != "plain":
                        kw["residual"] = residual
                    if res_mode == "gated":
                        kw["gate"] = gate
                    r = adt.adaln_quant_torch_ref(hidden, mul, add, **kw)
                    key = f"{norm}|{quant}|{res_mode}|{int(ocp)}"
                    cases.append(key)
                    for f in ("y", "quant", "dequant_scale", "dequant"):
                        if r[f] is not None:
                            out[f"{key}|{f}"] = np.asarray(r[f], np.float32)
                    if r["residual_out"] is not None:
                        out[f"{res_mode}|residual_out"] = np.asarray(r["residual_out"], np.float32)
    out["cases"] = np.array(cases)
    np.savez_compressed(OUT / "adaln_ref.npz", **out)


def gen_eager_adaln(rng: torch.Generator):
    adk = _load_file("ref_adaln_kernels", REF / "diffusion/quantization/adaln_kernels.py")
    B, S, H = 2, 24, 128
    hidden = torch.randn(B, S, H, generator=rng).to(torch.bfloat16)
    mul = (1 + 0.1 * torch.randn(B, 1, H, generator=rng)).to(torch.bfloat16)
    add = (0.1 * torch.randn(B, 1, H, generator=rng)).to(torch.bfloat16)
    residual = torch.randn(B, S, H, generator=rng).to(torch.bfloat16)
    gate = 0.5 * torch.randn(B, 1, H, generator=rng)
    out = {"hidden": _bf16(hidden), "mul": _bf16(mul), "add": _bf16(add), "residual": _bf16(residual), "gate": gate.numpy()}
    for norm in ("layer_norm", "rms_norm", "none"):
        o = adk._eager_adaln(hidden, mul, add, eps=1e-6, norm_type=norm, quant="none")
        out[f"{norm}|plain|out"] = _bf16(o)
        ro, o = adk._eager_adaln(hidden, mul, add, eps=1e-6, norm_type=norm, quant="none", residual=residual, gate=gate)
        out[f"{norm}|gated|residual_out"] = _bf16(ro)
        out[f"{norm}|gated|out"] = _bf16(o)
    np.savez_compressed(OUT / "eager_adaln.npz", **out)


def gen_attention(rng: torch.Generator):
    wt = REF / "diffusion/models/wan2_2/wan2_2_transformer.py"
    fns = _extract(wt, ["_torch_attend"], {"torch": torch})
    out = {}
    for tag, (B, N, S, Sk) in {"a": (1, 2, 96, 96), "b": (2, 1, 130, 140)}.items():
        q = (0.5 * torch.randn(B, N, S, 128, generator=rng)).to(torch.bfloat16)
        k = (0.5 * torch.randn(B, N, Sk, 128, generator=rng)).to(torch.bfloat16)
        v = (0.5 * torch.randn(B, N, Sk, 128, generator=rng)).to(torch.bfloat16)
        scale = 1.0 / 128 ** 0.5
        o = fns["_torch_attend"](q, k, v, scale)
        out.update({f"{tag}|q": _bf16(q), f"{tag}|k": _bf16(k), f"{tag}|v": _bf16(v), f"{tag}|scale": np.float32(scale), f"{tag}|o": _bf16(o)})
    np.savez_compressed(OUT / "torch_attend.npz", **out)


def gen_rope_norm(rng: torch.Generator):
    rope = _load_file("ref_rope", REF / "diffusion/layers/rope.py")
    emb = rope.WanRotaryPosEmbed(128, (1, 2, 2), 1024)
    latent = torch.zeros(1, 16, 3, 6, 8)
    cos, sin = emb(latent)
    S = cos.shape[1]
    x = torch.randn(1, S, 2, 128, generator=rng).to(torch.bfloat16)
    xr = rope.apply_rotary_emb_wan(x, cos, sin)
    rmm = _extract(REF / "diffusion/quantization/row_mx_modules.py", ["_rope_rotate_half_caches"], {"torch": torch})
    cos_rh, sin_rh = rmm["_rope_rotate_half_caches"]((cos, sin), 1, 128)
    rml = _extract(
        REF / "diffusion/quantization/row_mx_loaders.py",
        ["deinterleave_perm", "_deinterleave_qk_columns", "deinterleave_gamma_row"],
        {"torch": torch},
    )
    w = torch.randn(4, 3 * 256, generator=rng)
    wd = rml["_deinterleave_qk_columns"](w, 256, 256, 128)
    gamma = torch.randn(256, generator=rng)
    gd = rml["deinterleave_gamma_row"](gamma, 128)

    # DistributedRMSNorm at TP=1: the class with its process-group helpers stubbed to TP=1.
    env = {
        "torch": torch,
        "nn": torch.nn,
        "dist": None,
        "get_tensor_model_parallel_world_size": lambda: 1,
        "get_tp_group": lambda: types.SimpleNamespace(device_group=None),
        "set_weight_loader": lambda *a, **k: None,
        "sharding_weight_loader": lambda *a, **k: None,
    }
    cls = _extract(REF / "diffusion/models/wan2_2/wan2_2_transformer.py", ["DistributedRMSNorm"], env)["DistributedRMSNorm"]
    norm = cls(256, eps=1e-6)
    with torch.no_grad():
        norm.weight.copy_(1 + 0.1 * torch.randn(256, generator=rng))
    xn = torch.randn(1, S, 256, generator=rng).to(torch.bfloat16)
    with torch.no_grad():
        yn = norm(xn)
    np.savez_compressed(
        OUT / "rope_norm.npz",
        cos=cos.numpy(), sin=sin.numpy(), x=_bf16(x), x_rope=_bf16(xr),
        cos_rh=cos_rh.numpy(), sin_rh=sin_rh.numpy(),
        w=w.numpy(), w_deint=wd.numpy(), gamma=gamma.numpy(), gamma_deint=gd.numpy(),
        norm_w=norm.weight.detach().numpy(), norm_x=_bf16(xn), norm_y=_bf16(yn),
        latent_fhw=np.array([3, 6, 8]),
    )


def gen_oproj():
    wt = REF / "diffusion/models/wan2_2/wan2_2_transformer.py"
    fns = _extract(wt, ["_wan_o_proj"], {"torch": torch, "_can_use_wan_o_proj_kernel": lambda *a: False})
    rng = torch.Generator().manual_seed(20261202)
    out = {}
    for tag, (B, N, S, H) in {"a": (1, 2, 96, 256), "b": (2, 1, 40, 512)}.items():
        active = torch.randn(B, N, 128, S, generator=rng).to(torch.bfloat16)  # d-major attention output
        w = (0.02 * torch.randn(N * 128, H, generator=rng)).to(torch.bfloat16)
        bias = (0.5 * torch.randn(1, H, generator=rng)).to(torch.bfloat16)
        y = fns["_wan_o_proj"](active, w, bias)
        out.update({f"{tag}|active": _bf16(active), f"{tag}|w": _bf16(w), f"{tag}|bias": _bf16(bias), f"{tag}|y": _bf16(y)})
    np.savez_compressed(OUT / "wan_o_proj.npz", **out)


def gen_mlp():
    wt = REF / "diffusion/models/wan2_2/wan2_2_transformer.py"
    fns = _extract(wt, ["_wan_mlp"], {"torch": torch, "F": torch.nn.functional,
                                      "_can_use_wan_mlp_kernel": lambda *a: False})
    rng = torch.Generator().manual_seed(20261203)
    out = {}
    for tag, (B, T, H, I) in {"a": (1, 64, 128, 256), "b": (2, 24, 128, 256)}.items():
        x = torch.randn(B, T, H, generator=rng).to(torch.bfloat16)
        wu = (0.05 * torch.randn(H, I, generator=rng)).to(torch.bfloat16)
        wd = (0.05 * torch.randn(I, H, generator=rng)).to(torch.bfloat16)
        bu = (0.5 * torch.randn(1, I, generator=rng)).to(torch.bfloat16)
        bd = (0.5 * torch.randn(1, H, generator=rng)).to(torch.bfloat16)
        y = fns["_wan_mlp"](x, wu, wd, bu, bd)
        out.update({f"{tag}|x": _bf16(x), f"{tag}|wu": _bf16(wu), f"{tag}|wd": _bf16(wd), f"{tag}|bu": _bf16(bu),
                    f"{tag}|bd": _bf16(bd), f"{tag}|y": _bf16(y)})
    np.savez_compressed(OUT / "wan_mlp.npz", **out)


def gen_mlp_row_mx():
    """The ROW_MX MLP of the FP8 FFN leaf through the reference's own PyTorch reference
    ``_mlp_ref_standard`` and ``_mx_quantize`` (kernels/nkilib/core/mlp/mlp_torch.py:252-271, 401-600),
    CTE mode (``force_cte_mode=True`` in row_mx_mlp), GELU-tanh, no gate projection. Executed from the
    source with stand-ins for what is not in the reference tree or needs the Neuron SDK:
    ``nl`` dtype tags, ``_fp8_round_trip`` (the e4m3fn round trip done with torch's float8_e4m3fn
    cast), ``get_float32_exp`` (the biased fp32 exponent field), ``get_mx_fp_max`` (448 for e4m3fn),
    the MX block ``_q_height * _q_width`` = 32, the weight-layout undo helpers (identity: the weights
    are given in the plain ``x @ W`` layout) and ``_extract_precomputed_row_scale`` (returns the codes
    and the fp32 scale of the packed ROW rows, which it decodes from the row bytes)."""
    ct_path = REF / "kernels/nkilib/core/utils/common_types.py"
    from enum import Enum
    from typing import Optional
    env = {"Enum": Enum, "Optional": Optional}
    enums = _extract(ct_path, ["ActFnType", "QuantizationType", "ComputationMode", "MLPGateUpWeightLayout"], env)
    nl = types.SimpleNamespace(float8_e4m3fn="e4m3fn", float8_e4m3="e4m3", float8_e4m3fn_x4="e4m3fn_x4",
                               float32=np.float32)
    held = {}

    def fp8_round_trip(tensor, quant_dtype=nl.float8_e4m3):
        assert quant_dtype == "e4m3fn", quant_dtype
        return tensor.to(torch.float8_e4m3fn).to(torch.float32)

    def extract_precomputed_row_scale(hidden_tensor, H):
        return hidden_tensor[..., :H], held["row_scale"].reshape(-1, 1)

    ident_w = lambda w, *a, **k: w  # noqa: E731
    env = {
        "torch": torch, "np": np, "math": math, "Optional": Optional, "nl": nl, **enums,
        "_fp8_round_trip": fp8_round_trip, "_extract_precomputed_row_scale": extract_precomputed_row_scale,
        "get_float32_exp": lambda x: ((np.ascontiguousarray(x, np.float32).view(np.uint32) >> 23) & 0xFF).astype(np.uint32),
        "get_mx_fp_max": lambda dtype: 448.0, "_q_height": 8, "_q_width": 4,
        "_undo_mx_gate_up_w_reshape": ident_w, "_undo_mx_down_w_reshape": ident_w,
        "_undo_mx_gate_up_bias_reshape": ident_w, "_FP8_E4M3_MAX": 240.0, "_FP8_E4M3FN_MAX": 448.0,
    }
    mt = REF / "kernels/nkilib/core/mlp/mlp_torch.py"
    fns = _extract(mt, ["_apply_activation", "_apply_clamp", "_row_quantize", "_mx_quantize", "_is_tkg",
                        "_mlp_ref_standard"], env)
    QT, AF, CM, LY = (enums[n] for n in ("QuantizationType", "ActFnType", "ComputationMode", "MLPGateUpWeightLayout"))
    rng = torch.Generator().manual_seed(20261205)
    out = {}
    for tag, (T, H, I) in {"a": (64, 128, 512), "b": (40, 256, 512)}.items():
        x = torch.randn(T, H, generator=rng)
        rs = torch.clamp(x.abs().amax(1) / 448.0, min=1e-6)  # the adaLN ROW output (codes + per-row scale)
        codes = (x * (1.0 / rs)[:, None]).to(torch.float8_e4m3fn)
        wu = torch.randn(H, I, generator=rng) * 0.02
        wd = torch.randn(I, H, generator=rng) * 0.02
        su, sd = float(wu.abs().max() / 448.0), float(wd.abs().max() / 448.0)
        uc, dc = (wu / su).to(torch.float8_e4m3fn), (wd / sd).to(torch.float8_e4m3fn)
        bu = (0.1 * torch.randn(I, generator=rng)).to(torch.bfloat16)
        bd = (0.1 * torch.randn(H, generator=rng)).to(torch.bfloat16)
        held["row_scale"] = rs
        hidden = torch.cat([codes.float(), torch.zeros(T, 4)], dim=1).unsqueeze(0)  # [1, T, H + 4]
        y = fns["_mlp_ref_standard"](
            hidden=hidden, gate_w=uc.float(), up_w=uc.float(), down_w=dc.float(), quantization_type=QT.ROW_MX,
            gate_w_scale=None, up_w_scale=torch.full((128, I // 512, 4), su), down_w_scale=torch.full((128, H), sd),
            gate_up_in_scale=None, down_in_scale=None, quant_clipping_bound=None, gate_proj_bias_tensor=None,
            up_proj_bias_tensor=bu.float().reshape(1, I), down_proj_bias_tensor=bd.float().reshape(1, H),
            skip_gate_proj=True, activation_fn=AF.GELU_Tanh_Approx, gate_clamp_upper_limit=None,
            gate_clamp_lower_limit=None, up_clamp_upper_limit=None, up_clamp_lower_limit=None,
            gate_up_w_layout=LY.H_X4_INNERMOST, mode=CM.PREFILL, fp8_max=448.0, fp8_round_trip_dtype=nl.float8_e4m3fn,
        )
        out.update({f"{tag}|codes": codes.view(torch.uint8).numpy(), f"{tag}|rs": rs.numpy(),
                    f"{tag}|uc": uc.view(torch.uint8).numpy(), f"{tag}|su": np.float32(su),
                    f"{tag}|dc": dc.view(torch.uint8).numpy(), f"{tag}|sd": np.float32(sd),
                    f"{tag}|bu": _bf16(bu), f"{tag}|bd": _bf16(bd), f"{tag}|y": _bf16(y)})
    # the reference's MX quantiser alone on GELU-shaped values, including tiny and zero blocks
    v = torch.nn.functional.gelu(3 * torch.randn(16, 256, generator=rng), approximate="tanh")
    v[2, :32] = 0.0
    v[3, 32:64] *= 1e-30
    q, sc = fns["_mx_quantize"](v)
    out["mxq|x"] = v.numpy()
    out["mxq|codes"] = fp8_round_trip(q, "e4m3fn").numpy()
    out["mxq|scale"] = sc.numpy()
    np.savez_compressed(OUT / "mlp_row_mx.npz", **out)


class _UpCaptured(Exception):
    """Raised by the activation stand-in to stop _mlp_ref_standard right after the up-projection."""

    def __init__(self, up):
        super().__init__("captured")
        self.up = up


def gen_qkv_row_mx():
    """The ROW_MX projection arithmetic on QKV-shaped operands, executed by the reference's own
    ``_mlp_ref_standard`` (kernels/nkilib/core/mlp/mlp_torch.py:401-600) in ROW_MX CTE mode: its
    up-projection ``(Xq * row_scale) @ (Wq * w_scale) + bias`` (fp32, :470-497 and :575-578) is the
    same dequant-matmul as the ROW_MX QKV kernel's ``_dequant_row_mx`` (qkv_cte.py:3996-4021). The
    activation stand-in captures ``up_out`` and stops the run there (the MLP's activation, MX
    quantisation and down-projection are not part of the QKV path). Per-tensor Q/K/V weight scales
    (row_mx_loaders.py:246-260) are passed through the ROW_MX ``[128, I/512, 4]`` scale layout that
    the function un-permutes (:493-495). Stand-ins as in ``gen_mlp_row_mx``."""
    ct_path = REF / "kernels/nkilib/core/utils/common_types.py"
    from enum import Enum
    from typing import Optional
    env = {"Enum": Enum, "Optional": Optional}
    enums = _extract(ct_path, ["ActFnType", "QuantizationType", "ComputationMode", "MLPGateUpWeightLayout"], env)
    nl = types.SimpleNamespace(float8_e4m3fn="e4m3fn", float8_e4m3="e4m3", float8_e4m3fn_x4="e4m3fn_x4",
                               float32=np.float32)
    held = {}

    def capture(x, fn):
        raise _UpCaptured(x)

    ident_w = lambda w, *a, **k: w  # noqa: E731
    env = {
        "torch": torch, "np": np, "math": math, "Optional": Optional, "nl": nl, **enums,
        "_fp8_round_trip": lambda t, quant_dtype=None: t.to(torch.float8_e4m3fn).to(torch.float32),
        "_extract_precomputed_row_scale": lambda hidden, H: (hidden[..., :H], held["row_scale"].reshape(-1, 1)),
        "_apply_activation": capture,
        "_undo_mx_gate_up_w_reshape": ident_w, "_undo_mx_down_w_reshape": ident_w,
        "_undo_mx_gate_up_bias_reshape": ident_w, "_FP8_E4M3_MAX": 240.0, "_FP8_E4M3FN_MAX": 448.0,
    }
    mt = REF / "kernels/nkilib/core/mlp/mlp_torch.py"
    fns = _extract(mt, ["_apply_clamp", "_is_tkg", "_mlp_ref_standard"], env)
    QT, AF, CM, LY = (enums[n] for n in ("QuantizationType", "ActFnType", "ComputationMode", "MLPGateUpWeightLayout"))
    rng = torch.Generator().manual_seed(20261206)
    out = {}
    # two shapes with 4 heads per segment (I = 1536, a multiple of the 512-column scale layout); the
    # full config-3 width is covered by the GPU tests against the oracle this fixture pins
    for tag, (T, H, heads) in {"a": (32, 1024, 4), "b": (40, 512, 4)}.items():
        I = 3 * heads * 128
        x = torch.randn(T, H, generator=rng)
        rs = torch.clamp(x.abs().amax(1) / 448.0, min=1e-6)  # the adaLN ROW output (codes + per-row scale)
        codes = (x * (1.0 / rs)[:, None]).to(torch.float8_e4m3fn)
        w = torch.randn(H, I, generator=rng) * 0.02
        seg = heads * 128
        cs = torch.empty(I)
        wc = torch.empty(H, I, dtype=torch.float8_e4m3fn)
        for lo in (0, seg, 2 * seg):  # per-tensor Q, K, V scales
            sc = float(w[:, lo:lo + seg].abs().max() / 448.0)
            cs[lo:lo + seg] = sc
            wc[:, lo:lo + seg] = (w[:, lo:lo + seg] / sc).to(torch.float8_e4m3fn)
        bias = (0.1 * torch.randn(I, generator=rng)).to(torch.bfloat16)
        held["row_scale"] = rs
        hidden = torch.cat([codes.float(), torch.zeros(T, 4)], dim=1).unsqueeze(0)  # [1, T, H + 4]
        up_scale = cs.reshape(I // 512, 128, 4).permute(1, 0, 2).contiguous()  # un-permuted by :493-495
        try:
            fns["_mlp_ref_standard"](
                hidden=hidden, gate_w=wc.float(), up_w=wc.float(), down_w=torch.zeros(I, H),
                quantization_type=QT.ROW_MX, gate_w_scale=None, up_w_scale=up_scale,
                down_w_scale=torch.ones(128, H), gate_up_in_scale=None, down_in_scale=None,
                quant_clipping_bound=None, gate_proj_bias_tensor=None,
                up_proj_bias_tensor=bias.float().reshape(1, I), down_proj_bias_tensor=None, skip_gate_proj=True,
                activation_fn=AF.GELU_Tanh_Approx, gate_clamp_upper_limit=None, gate_clamp_lower_limit=None,
                up_clamp_upper_limit=None, up_clamp_lower_limit=None, gate_up_w_layout=LY.H_X4_INNERMOST,
                mode=CM.PREFILL, fp8_max=448.0, fp8_round_trip_dtype=nl.float8_e4m3fn,
            )
            raise RuntimeError("the up-projection was not captured")
        except _UpCaptured as c:
            up = c.up
        out.update({f"{tag}|codes": codes.view(torch.uint8).numpy(), f"{tag}|rs": rs.numpy(),
                    f"{tag}|wc": wc.view(torch.uint8).numpy(), f"{tag}|cs": cs.numpy(), f"{tag}|bias": _bf16(bias),
                    f"{tag}|up": up.float().numpy()})
    np.savez_compressed(OUT / "qkv_row_mx.npz", **out)


def gen_checkpoint():
    comfy = _load_file("ref_comfy_fp8", REF / "diffusion/quantization/comfy_fp8_checkpoint.py")
    m = comfy.build_fp8_dequant_mappings(2)
    names = comfy.fp8_transformed_parameter_names(2)
    (OUT / "comfy_fp8_mapping.json").write_text(json.dumps({"mappings": m, "fp8_param_names": names}, indent=0, sort_keys=True))
    dq = _extract(REF / "diffusion/quantization/dequant_loaders.py", ["dequantize_to_bf16"], {"torch": torch})
    rng = torch.Generator().manual_seed(20261204)
    w = (torch.randn(48, 40, generator=rng) * 100).clamp(-448, 448).to(torch.float8_e4m3fn)
    s = torch.tensor(0.0123, dtype=torch.float32)
    y = dq["dequantize_to_bf16"](w, s)
    np.savez_compressed(OUT / "fp8_dequant.npz", codes=w.view(torch.uint8).numpy(), scale=s.numpy(), y=_bf16(y))


def main():
    if not REF.exists():
        sys.exit(f"reference checkout not found at {REF}")
    only = sys.argv[1:]
    if only:  # regenerate only the named fixtures, e.g. ``make_golden.py oproj``
        for name in only:
            globals()[f"gen_{name}"]()
        return
    rng = torch.Generator().manual_seed(20261201)
    gen_adaln(rng)
    gen_eager_adaln(rng)
    gen_attention(rng)
    gen_rope_norm(rng)
    gen_oproj()
    gen_mlp()
    gen_mlp_row_mx()
    gen_qkv_row_mx()
    gen_checkpoint()
    for p in sorted(OUT.glob("*.npz")):
        print(p.name, p.stat().st_size)


if __name__ == "__main__":
    main()
