"""LittleBitLinear — drop-in module for quantization/modules/littlebit.py.

Same conversion entry point (``__quant_convert__``, applied to an nn.Linear by
a ``__class__`` swap as quant_util.patch_inst does, quant_util.py:66-76), same
rank sizing (littlebit.py:50-93), parameter names (U, V, u1, u2, v1, v2 and the
``_R`` residual set, :144-173), buffers (``_eff_bit_target``,
``_split_dim_final``, ``_eff_bit_actual``) and packed ``state_dict``
(:307-345: ``{U,V}{,_R}_packed`` + ``_shape``, float factors dropped).

The forward is different by design: instead of multiplying unpacked bf16 ±1
matrices (littlebit.py:114-121 on cuBLAS), it runs the sm_100a kernels on the
packed sign words.  Latent float factors are packed on first use (sign with
0 -> +1, functions/binary.py:7-10); packed checkpoints load without ever
being unpacked.  CUDA tensors only.
"""
from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn as nn

from . import ops


class LittleBitLinear(nn.Module):
    # ---- construction (littlebit.py:9-48) ----------------------------------
    def __quant_convert__(self, do_train: bool, quant_func=None, *, split_dim: int = 1024,
                          eff_bit: Optional[float] = None, residual: bool = False,
                          ratio_factor: float = 1.0, min_split_dim: int = 8, **kwargs):
        self.do_train = do_train
        self.quant_func = quant_func
        self.residual = residual
        self._binarized = False
        a, b = self.in_features, self.out_features
        f = self._estimate_split_dim(a, b, eff_bit, residual)
        if f:
            f *= ratio_factor
        s = self._finalize_split_dim(f, split_dim, min_split_dim)
        self.split_dim = s
        eff = self._compute_eff_bits(a, b, s, residual)
        self.register_buffer("_eff_bit_target", torch.tensor(-1.0 if eff_bit is None else float(eff_bit)))
        self.register_buffer("_split_dim_final", torch.tensor(s))
        self.register_buffer("_eff_bit_actual", torch.tensor(eff))
        if do_train:
            raise NotImplementedError(
                "LittleBitLinear(do_train=True): the SVD initialisation for quantisation-aware "
                "training is not part of the B200 inference runtime")
        self._initialize_empty_parameters()
        self._packed: Optional[ops.PackedLinear] = None

    @staticmethod
    def _estimate_split_dim(a, b, eff_bit_target, residual):
        if eff_bit_target is None or a * b == 0:
            return None
        base = a + b + 16
        if residual:
            num, den = a * b * eff_bit_target - 32 * (a + b), 2 * base
        else:
            num, den = a * b * eff_bit_target - 16 * (a + b), base
        return num / den if den else None

    @staticmethod
    def _finalize_split_dim(split_float, split_default, min_split_dim):
        cand = split_float if split_float is not None else split_default
        cand = int(cand) if cand is not None else 0
        cand = (cand // 8) * 8
        if cand == 0:
            cand = min_split_dim
        return max(cand, min_split_dim)

    @staticmethod
    def _compute_eff_bits(a, b, s, residual):
        if a * b == 0:
            return float("inf")
        if residual:
            return (s * 2 * (a + b + 16) + 32 * (a + b)) / (a * b)
        return (s * (a + b + 16) + 16 * (a + b)) / (a * b)

    def _initialize_empty_parameters(self):
        def mk(*shape):
            return nn.Parameter(torch.empty(*shape, device="meta", dtype=torch.bfloat16),
                                requires_grad=False)
        o, i, s = self.out_features, self.in_features, self.split_dim
        for suf in ([""] + (["_R"] if self.residual else [])):
            setattr(self, "U" + suf, mk(o, s))
            setattr(self, "V" + suf, mk(s, i))
            setattr(self, "u1" + suf, mk(1, o))
            setattr(self, "u2" + suf, mk(1, s))
            setattr(self, "v1" + suf, mk(1, s))
            setattr(self, "v2" + suf, mk(1, i))
        if hasattr(self, "weight"):
            del self.weight
        self.register_parameter("weight", None)

    # ---- packing (littlebit.py:307-345) ------------------------------------
    def quantize(self, x):
        if self._binarized:
            return x
        return self.quant_func(x) if self.quant_func is not None else torch.where(x < 0, -1.0, 1.0).to(x.dtype)

    def _sign_words(self, name: str) -> torch.Tensor:
        if name in self._packed_src:
            return self._packed_src[name]
        p = getattr(self, name)
        if p is None or p.device.type == "meta":
            raise RuntimeError(f"LittleBitLinear.{name} is not loaded")
        return ops.pack_signs_from_float(p.data.contiguous())

    def pack_weights(self, *args, **kwargs):
        out = {}
        for nm in ("U", "V") + (("U_R", "V_R") if self.residual else ()):
            out[f"{nm}_packed"] = self._sign_words(nm)
            p = getattr(self, nm)
            shp = p.shape if p is not None else self._packed_shape[nm]
            out[f"{nm}_shape"] = torch.tensor(tuple(shp), dtype=torch.long)
        return out

    def state_dict(self, *args, **kwargs):
        prefix = kwargs.get("prefix", "")
        st = super().state_dict(*args, **kwargs)
        for k in [k for k in st if k.startswith(prefix + "U") or k.startswith(prefix + "V")]:
            del st[k]
        for k, v in self.pack_weights().items():
            st[prefix + k] = v
        return st

    @property
    def _packed_src(self):
        return self.__dict__.setdefault("_packed_words", {})

    @property
    def _packed_shape(self):
        return self.__dict__.setdefault("_packed_shapes", {})

    def _load_from_state_dict(self, state_dict, prefix, local_metadata, strict, missing_keys,
                              unexpected_keys, error_msgs):
        # packed sign words load as-is (no unpacking); float scales as parameters
        names = ("U", "V") + (("U_R", "V_R") if self.residual else ())
        for nm in names:
            pk, sk = prefix + f"{nm}_packed", prefix + f"{nm}_shape"
            if pk in state_dict:
                self._packed_src[nm] = state_dict.pop(pk).to(torch.int32)
                shp = tuple(int(v) for v in state_dict.pop(sk)) if sk in state_dict else None
                self._packed_shape[nm] = shp
                setattr(self, nm, None)
        for nm in [n for n, _ in self.named_parameters(recurse=False)]:
            k = prefix + nm
            if k in state_dict:
                v = state_dict.pop(k)
                setattr(self, nm, nn.Parameter(v.detach().clone(), requires_grad=False))
        for nm in ("_eff_bit_target", "_split_dim_final", "_eff_bit_actual"):
            k = prefix + nm
            if k in state_dict:
                self._buffers[nm] = state_dict.pop(k).clone()
        self._packed = None
        self._binarized = True

    # ---- forward -----------------------------------------------------------
    def _device_layer(self, device) -> ops.PackedLinear:
        if self._packed is not None and self._packed.device == device:
            return self._packed
        f32 = lambda t: t.detach().reshape(-1).to(device=device, dtype=torch.float32).contiguous()
        brs = []
        for suf in ([""] + (["_R"] if self.residual else [])):
            v = self._sign_words("V" + suf).to(device)
            u = self._sign_words("U" + suf).to(device)
            r = int(v.shape[0])
            mid = (getattr(self, "v1" + suf).detach().float() * getattr(self, "u2" + suf).detach().float())
            brs.append(ops.Branch(v.contiguous(), f32(getattr(self, "v2" + suf)), f32(mid), u.contiguous(),
                                  f32(getattr(self, "u1" + suf)), r))
        bias = None if self.bias is None else f32(self.bias)
        self._packed = ops.PackedLinear(self.in_features, self.out_features, brs, bias)
        return self._packed

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if not x.is_cuda:
            raise RuntimeError("LittleBitLinear (B200) runs on CUDA tensors only")
        lay = self._device_layer(x.device)
        out_dtype = x.dtype if x.dtype in (torch.float32, torch.bfloat16) else torch.float32
        xin = x if x.dtype in (torch.float32, torch.bfloat16) else x.float()
        return ops.lb_linear(lay, xin, out_dtype=out_dtype)

    # ---- reporting (littlebit.py:123-140, 347-362) --------------------------
    @property
    def eff_bit_target(self):
        v = float(self._eff_bit_target)
        return None if v < 0 else v

    @property
    def eff_bit_actual(self):
        return float(self._eff_bit_actual)

    @property
    def total_bit_usage(self):
        return self.eff_bit_actual * self.in_features * self.out_features

    def extra_repr(self):
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"bias={self.bias is not None}, split_dim={int(self._split_dim_final)}, "
                f"eff_bit_actual={self.eff_bit_actual:.4f}, residual={self.residual}")


def patch_linear(mod: nn.Linear, **convert_kwargs) -> LittleBitLinear:
    """nn.Linear -> LittleBitLinear in place (quant_util.py:66-76)."""
    mod.__class__ = LittleBitLinear
    mod.__quant_convert__(**convert_kwargs)
    return mod
