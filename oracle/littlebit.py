"""LittleBitLinear and the runtime checkpoint layout restated (oracle; test
infrastructure only).

Reference: quantization/modules/littlebit.py (rank sizing :50-93, forward
:95-112, _compute_forward :114-121); convert_hf_to_runtime.py (convert_state_dict
:29-97, build_dummy_config :193-213, build_runtime_config :216-235);
littlespec_ref/littlebit_itq_spec.py:298-309 (shared-factor residual).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import numpy as np

from .packing import unpack_float


def estimate_split_dim(a: int, b: int, eff_bit, residual: bool):
    """littlebit.py:50-63."""
    if eff_bit is None or a * b == 0:
        return None
    base = a + b + 16
    if residual:
        num, den = a * b * eff_bit - 32 * (a + b), 2 * base
    else:
        num, den = a * b * eff_bit - 16 * (a + b), base
    return num / den if den else None


def finalize_split_dim(split_float, split_default: int, min_split_dim: int) -> int:
    """littlebit.py:65-80: round down to a multiple of 8, minimum fallback."""
    cand = split_float if split_float is not None else split_default
    cand = int(cand) if cand is not None else 0
    cand = (cand // 8) * 8
    if cand == 0:
        cand = min_split_dim
    return max(cand, min_split_dim)


def compute_eff_bits(a: int, b: int, s: int, residual: bool) -> float:
    """littlebit.py:82-93."""
    if a * b == 0:
        return float("inf")
    if residual:
        num = s * 2 * (a + b + 16) + 32 * (a + b)
    else:
        num = s * (a + b + 16) + 16 * (a + b)
    return num / (a * b)


def split_dim_for(in_f: int, out_f: int, eff_bit, residual=False, ratio_factor=1.0,
                  split_default=1024, min_split_dim=8) -> int:
    """The rank __quant_convert__ picks (littlebit.py:31-40)."""
    f = estimate_split_dim(in_f, out_f, eff_bit, residual)
    if f:
        f *= ratio_factor
    return finalize_split_dim(f, split_default, min_split_dim)


def compute_forward(x, V, U, v2, v1, u2, u1, dtype=np.float64):
    """littlebit.py:114-121: ((((x*v2) @ V^T) * (v1*u2)) @ U^T) * u1."""
    x, V, U = (np.asarray(a, dtype) for a in (x, V, U))
    v2, v1, u2, u1 = (np.asarray(a, dtype).reshape(1, -1) for a in (v2, v1, u2, u1))
    return ((((x * v2) @ V.T) * (v1 * u2)) @ U.T) * u1


@dataclass
class RtBranch:
    """One branch in runtime layout (convert_hf_to_runtime.py:47-57):
    v_sign [r, ceil(K/32)] int32 (None = shared with branch 0), v2 [K],
    mid [r] (= v1*u2), u_sign [N, ceil(r/32)] int32, u1 [N]."""
    v_sign: Optional[np.ndarray]
    v2: Optional[np.ndarray]
    mid: np.ndarray
    u_sign: np.ndarray
    u1: np.ndarray
    rank: int


def branch_forward(x: np.ndarray, br: RtBranch, in_f: int, out_f: int, main: RtBranch = None,
                   dtype=np.float64) -> np.ndarray:
    """y_b = u1 ⊙ U·(mid ⊙ V·(v2 ⊙ x)) from packed words (littlebit.py:114-121 with
    the runtime fusion mid = v1*u2, convert_hf_to_runtime.py:54-57).  A shared-V
    branch (v_sign None) uses ``main``'s V and v2 (littlebit_itq_spec.py:298-309)."""
    vsrc = br if br.v_sign is not None else main
    V = unpack_float(vsrc.v_sign, (br.rank, in_f), dtype)
    U = unpack_float(br.u_sign, (out_f, br.rank), dtype)
    x = np.asarray(x, dtype)
    t = (x * np.asarray(vsrc.v2, dtype).reshape(1, -1)) @ V.T
    t = t * np.asarray(br.mid, dtype).reshape(1, -1)
    return (t @ U.T) * np.asarray(br.u1, dtype).reshape(1, -1)


def linear_forward(x, branches, in_f: int, out_f: int, bias=None, dtype=np.float64):
    """LittleBitLinear.forward (littlebit.py:95-112): main + residual (+ bias)."""
    y = branch_forward(x, branches[0], in_f, out_f, dtype=dtype)
    for br in branches[1:]:
        y = y + branch_forward(x, br, in_f, out_f, main=branches[0], dtype=dtype)
    if bias is not None:
        y = y + np.asarray(bias, dtype).reshape(1, -1)
    return y


_DROP = ("._eff_bit_target", "._split_dim_final", "._eff_bit_actual", "._binarized")


def convert_state_dict(hf: dict) -> dict:
    """convert_hf_to_runtime.py:29-97 on a dict of numpy arrays."""
    out = {}
    prefixes = set()
    for k in hf:
        if k.endswith(".U_packed"):
            prefixes.add(k[: -len(".U_packed")])
        elif k.endswith(".U_R_packed"):
            prefixes.add(k[: -len(".U_R_packed")])
    used = set()
    for p in sorted(prefixes):
        if f"{p}.U_packed" in hf:
            out[f"{p}.u_sign_rt"] = hf[f"{p}.U_packed"]
            out[f"{p}.u_sign_rt_shape"] = hf[f"{p}.U_shape"]
            out[f"{p}.v_sign_rt"] = hf[f"{p}.V_packed"]
            out[f"{p}.v_sign_rt_shape"] = hf[f"{p}.V_shape"]
            out[f"{p}.u1"] = hf[f"{p}.u1"]
            out[f"{p}.v2"] = hf[f"{p}.v2"]
            out[f"{p}.mid"] = (hf[f"{p}.v1"].astype(np.float32) * hf[f"{p}.u2"].astype(np.float32))
            used.update(f"{p}.{s}" for s in ("U_packed", "U_shape", "V_packed", "V_shape",
                                             "u1", "u2", "v1", "v2"))
        if f"{p}.U_R_packed" in hf:
            out[f"{p}.u_sign_r_rt"] = hf[f"{p}.U_R_packed"]
            out[f"{p}.u_sign_r_rt_shape"] = hf[f"{p}.U_R_shape"]
            out[f"{p}.v_sign_r_rt"] = hf[f"{p}.V_R_packed"]
            out[f"{p}.v_sign_r_rt_shape"] = hf[f"{p}.V_R_shape"]
            out[f"{p}.u1_r"] = hf[f"{p}.u1_R"]
            out[f"{p}.v2_r"] = hf[f"{p}.v2_R"]
            out[f"{p}.mid_r"] = (hf[f"{p}.v1_R"].astype(np.float32) * hf[f"{p}.u2_R"].astype(np.float32))
            used.update(f"{p}.{s}" for s in ("U_R_packed", "U_R_shape", "V_R_packed", "V_R_shape",
                                             "u1_R", "u2_R", "v1_R", "v2_R"))
    for k, v in hf.items():
        if k in used or any(k.endswith(s) for s in _DROP):
            continue
        out[k] = v
    return out


def build_dummy_config(hf_cfg: dict, lb_cfg: dict) -> dict:
    """convert_hf_to_runtime.py:193-213."""
    return {
        "name": hf_cfg.get("_name_or_path", "llama"),
        "hidden_size": hf_cfg["hidden_size"],
        "intermediate_size": hf_cfg["intermediate_size"],
        "num_hidden_layers": hf_cfg["num_hidden_layers"],
        "num_attention_heads": hf_cfg["num_attention_heads"],
        "num_key_value_heads": hf_cfg.get("num_key_value_heads", hf_cfg["num_attention_heads"]),
        "vocab_size": hf_cfg["vocab_size"],
        "rms_norm_eps": hf_cfg.get("rms_norm_eps", 1e-6),
        "include_lm_head": False,
        "eff_bit": lb_cfg.get("eff_bit", 0.1),
        "residual": lb_cfg.get("residual", False),
    }


def build_runtime_config(hf_cfg: dict, lb_cfg: dict) -> dict:
    """convert_hf_to_runtime.py:216-235."""
    return {
        "format_version": 1,
        "checkpoint_format": "runtime",
        "sign_storage": "row_i1",
        "runtime_layout": "cpu_row_i1",
        "base_model_id": hf_cfg.get("_name_or_path", None),
        "model_type": hf_cfg.get("model_type", "llama"),
        "torch_dtype": "bfloat16",
        "quant_func": lb_cfg.get("quant_func", "STEBinary"),
        "eff_bit": lb_cfg.get("eff_bit", 0.1),
        "split_dim": lb_cfg.get("split_dim", None),
        "residual": lb_cfg.get("residual", False),
    }
