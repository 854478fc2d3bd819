"""The runtime checkpoint format (drop-in for convert_hf_to_runtime.py).

Same functions, key names and file set as the reference converter:
``convert_state_dict`` (convert_hf_to_runtime.py:29-97),
``convert_state_dict_canonical`` (:100-167), ``load_hf_state_dict`` (:170-190),
``build_dummy_config`` (:193-213), ``build_runtime_config`` (:216-235) and
``convert_hf_to_runtime`` (:238-290).  The key map has to be identical for
the checkpoints to be interchangeable, so the tables below follow the
reference one for one.
"""
from __future__ import annotations

import json
import shutil
from pathlib import Path
from typing import Dict

import torch

_DROP_SUFFIXES = ("._eff_bit_target", "._split_dim_final", "._eff_bit_actual", "._binarized")

# (HF suffix, runtime suffix, canonical suffix) for the main and residual branches
_MAIN = (("U_packed", "u_sign_rt", "u_sign_packed"), ("U_shape", "u_sign_rt_shape", "u_sign_shape"),
         ("V_packed", "v_sign_rt", "v_sign_packed"), ("V_shape", "v_sign_rt_shape", "v_sign_shape"),
         ("u1", "u1", "u1"), ("v2", "v2", "v2"))
_RES = (("U_R_packed", "u_sign_r_rt", "u_sign_r_packed"), ("U_R_shape", "u_sign_r_rt_shape", "u_sign_r_shape"),
        ("V_R_packed", "v_sign_r_rt", "v_sign_r_packed"), ("V_R_shape", "v_sign_r_rt_shape", "v_sign_r_shape"),
        ("u1_R", "u1_r", "u1_r"), ("v2_R", "v2_r", "v2_r"))


def _prefixes(hf: Dict[str, torch.Tensor]):
    out = set()
    for k in hf:
        if k.endswith(".U_packed"):
            out.add(k[: -len(".U_packed")])
        elif k.endswith(".U_R_packed"):
            out.add(k[: -len(".U_R_packed")])
    return sorted(out)


def _convert(hf: Dict[str, torch.Tensor], col: int) -> Dict[str, torch.Tensor]:
    out: Dict[str, torch.Tensor] = {}
    used = set()
    for p in _prefixes(hf):
        for table, v1k, u2k, midk in ((_MAIN, "v1", "u2", "mid"), (_RES, "v1_R", "u2_R", "mid_r")):
            if f"{p}.{table[0][0]}" not in hf:
                continue
            for row in table:
                out[f"{p}.{row[col]}"] = hf[f"{p}.{row[0]}"]
                used.add(f"{p}.{row[0]}")
            # the two middle scales fuse into one fp32 vector: mid = v1 * u2
            v1 = hf[f"{p}.{v1k}"].to(torch.float32)
            u2 = hf[f"{p}.{u2k}"].to(torch.float32)
            out[f"{p}.{midk}"] = (v1 * u2).contiguous()
            used.update((f"{p}.{v1k}", f"{p}.{u2k}"))
    for k, v in hf.items():
        if k in used or k.endswith(_DROP_SUFFIXES):
            continue
        out[k] = v
    return out


def convert_state_dict(hf_state: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
    """HF LittleBit state dict -> runtime keys (convert_hf_to_runtime.py:29-97)."""
    return _convert(hf_state, 1)


def convert_state_dict_canonical(hf_state: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
    """HF LittleBit state dict -> canonical keys (convert_hf_to_runtime.py:100-167)."""
    return _convert(hf_state, 2)


def load_hf_state_dict(model_path) -> Dict[str, torch.Tensor]:
    from safetensors.torch import load_file

    p = Path(model_path)
    idx, single = p / "model.safetensors.index.json", p / "model.safetensors"
    if idx.exists():
        shards = set(json.loads(idx.read_text())["weight_map"].values())
        sd = {}
        for s in shards:
            sd.update(load_file(str(p / s)))
        return sd
    if single.exists():
        return load_file(str(single))
    raise FileNotFoundError(f"No safetensors files found in {p}")


def _json_or_dict(v) -> dict:
    """A config given as a JSON file path (the reference's argument) or as a dict."""
    if isinstance(v, dict):
        return v
    return json.loads(Path(v).read_text())


def build_dummy_config(hf_config, lb_config) -> dict:
    """dummy_llama3_config.json (convert_hf_to_runtime.py:193-213).  Takes the
    paths of config.json and littlebit_config.json, as the reference does, or
    the two configs as dicts."""
    hf_config, lb_config = _json_or_dict(hf_config), _json_or_dict(lb_config)
    return {
        "name": hf_config.get("_name_or_path", "llama"),
        "hidden_size": hf_config["hidden_size"],
        "intermediate_size": hf_config["intermediate_size"],
        "num_hidden_layers": hf_config["num_hidden_layers"],
        "num_attention_heads": hf_config["num_attention_heads"],
        "num_key_value_heads": hf_config.get("num_key_value_heads", hf_config["num_attention_heads"]),
        "vocab_size": hf_config["vocab_size"],
        "rms_norm_eps": hf_config.get("rms_norm_eps", 1e-6),
        "include_lm_head": False,
        "eff_bit": lb_config.get("eff_bit", 0.1),
        "residual": lb_config.get("residual", False),
    }


def build_runtime_config(hf_config, lb_config) -> dict:
    """littlebit_runtime_config.json (convert_hf_to_runtime.py:216-235); arguments
    as for :func:`build_dummy_config`."""
    hf_config, lb_config = _json_or_dict(hf_config), _json_or_dict(lb_config)
    return {
        "format_version": 1,
        "checkpoint_format": "runtime",
        "sign_storage": "row_i1",
        "runtime_layout": "cpu_row_i1",
        "base_model_id": hf_config.get("_name_or_path", None),
        "model_type": hf_config.get("model_type", "llama"),
        "torch_dtype": "bfloat16",
        "quant_func": lb_config.get("quant_func", "STEBinary"),
        "eff_bit": lb_config.get("eff_bit", 0.1),
        "split_dim": lb_config.get("split_dim", None),
        "residual": lb_config.get("residual", False),
    }


def convert_hf_to_runtime(input_path, output_path, fmt: str = "runtime") -> str:
    """Directory-level conversion (convert_hf_to_runtime.py:238-290)."""
    from safetensors.torch import save_file

    src, dst = Path(input_path), Path(output_path)
    dst.mkdir(parents=True, exist_ok=True)
    hf = load_hf_state_dict(src)
    if fmt == "canonical":
        conv = convert_state_dict_canonical(hf)
        target = dst / "model.safetensors"
    else:
        conv = convert_state_dict(hf)
        target = dst / "littlebit_runtime.safetensors"
    save_file({k: v.contiguous() for k, v in conv.items()}, str(target))
    hf_cfg_p, lb_cfg_p = src / "config.json", src / "littlebit_config.json"
    if hf_cfg_p.exists() and lb_cfg_p.exists():
        hf_cfg = json.loads(hf_cfg_p.read_text())
        lb_cfg = json.loads(lb_cfg_p.read_text())
        (dst / "littlebit_runtime_config.json").write_text(json.dumps(build_runtime_config(hf_cfg, lb_cfg), indent=2))
        (dst / "dummy_llama3_config.json").write_text(json.dumps(build_dummy_config(hf_cfg, lb_cfg), indent=2))
        if fmt == "canonical":
            shutil.copy2(hf_cfg_p, dst / "config.json")
            shutil.copy2(lb_cfg_p, dst / "littlebit_config.json")
            for pat in ("tokenizer*", "special_tokens*"):
                for f in src.glob(pat):
                    shutil.copy2(f, dst / f.name)
    return str(dst)


def load_runtime_checkpoint(runtime_path, device="cpu"):
    """(state dict, runtime config) of a runtime directory — the loader the CPU
    adapters import from lb_kernels (cpu_draft_model.py:31-39, 158-162)."""
    from safetensors.torch import load_file

    p = Path(runtime_path)
    state = load_file(str(p / "littlebit_runtime.safetensors"), device=str(device))
    cfg = {}
    if (p / "littlebit_runtime_config.json").exists():
        cfg = json.loads((p / "littlebit_runtime_config.json").read_text())
    return state, cfg
