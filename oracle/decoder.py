"""LittleBit Llama decoder restated in numpy (oracle; test infrastructure only).

Semantics follow HF Llama (transformers LlamaForCausalLM: RMSNorm, rotate_half
RoPE, GQA attention, SiLU MLP) with every q/k/v/o/gate/up/down replaced by
LittleBitLinear (quantization/utils/quant_util.py:36-79 patching,
littlebit.py:95-121 forward).  The KV-cached step mirrors the CPU runtime's
layer order (patches/littlebit_cpu_optimized.cpp:1627-1835) and its batch
verify (cpp:1846-2079), plus rotary positions and tree masks
(tree_utils.py:72-175, speculative_decoding.py:454-617).

``kv_bf16=True`` rounds cached keys/values to bfloat16 (the B200 cache
precision); with False the cache is exact, as in HF's fp32 path.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional, Sequence

import numpy as np

from .littlebit import RtBranch, linear_forward

PROJ_NAMES = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even to bfloat16, returned as float32."""
    f = np.ascontiguousarray(x, dtype=np.float32)
    u = f.view(np.uint32).astype(np.uint64)
    u = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return u.astype(np.uint32).view(np.float32)


@dataclass
class DecoderConfig:
    n_layers: int
    hidden: int
    intermediate: int
    heads: int
    kv_heads: int
    vocab: int
    rms_eps: float = 1e-6
    rope_theta: float = 10000.0
    max_seq: int = 1024

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads


@dataclass
class OracleLayer:
    ln1: np.ndarray
    ln2: np.ndarray
    projs: List[List[RtBranch]]  # 7 projections, each 1-2 branches


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """HF LlamaRMSNorm / cpp:998-1052: x * rsqrt(mean(x^2) + eps) * w."""
    var = np.mean(x * x, axis=-1, keepdims=True)
    return x / np.sqrt(var + eps) * w


def rope(x: np.ndarray, pos: np.ndarray, theta: float) -> np.ndarray:
    """HF rotate_half RoPE on x [n, heads, d] at positions pos [n] (float64 angles).
    theta <= 0 applies no rotation, as the reference's CPU runtime does
    (patches/littlebit_cpu_optimized.cpp:1522-2079 has no rotary step)."""
    if not theta > 0:
        return x
    d = x.shape[-1]
    half = d // 2
    inv = theta ** (-2.0 * np.arange(half, dtype=np.float64) / d)
    ang = pos.astype(np.float64)[:, None] * inv[None, :]
    c, s = np.cos(ang)[:, None, :], np.sin(ang)[:, None, :]
    x1, x2 = x[..., :half], x[..., half:]
    return np.concatenate([x1 * c - x2 * s, x2 * c + x1 * s], axis=-1)


def silu(x: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        return x / (1.0 + np.exp(-x))


class OracleDecoder:
    def __init__(self, cfg: DecoderConfig, embed: np.ndarray, final_norm: np.ndarray,
                 lm_head: Optional[np.ndarray], layers: Sequence[OracleLayer],
                 kv_bf16: bool = True, dtype=np.float64):
        self.cfg = cfg
        self.embed = np.asarray(embed, np.float64)
        self.final_norm = np.asarray(final_norm, np.float64)
        self.lm_head = None if lm_head is None else np.asarray(lm_head, np.float64)
        self.layers = list(layers)
        self.kv_bf16 = kv_bf16
        self.dtype = dtype
        self.reset()

    def reset(self):
        c = self.cfg
        shp = (c.n_layers, c.kv_heads, c.max_seq, c.head_dim)
        self.kc = np.zeros(shp, np.float64)
        self.vc = np.zeros(shp, np.float64)

    def _lin(self, x, li, p, in_f, out_f):
        return linear_forward(x, self.layers[li].projs[p], in_f, out_f, dtype=self.dtype)

    def forward(self, tokens: Sequence[int], start: int, pos: Optional[Sequence[int]] = None,
                tree_mask: Optional[Sequence[int]] = None):
        """Process n tokens at cache slots start..start+n-1; returns the pre-norm
        residual stream [n, hidden] (apply final_hidden / logits on it)."""
        c = self.cfg
        n = len(tokens)
        d, H, KVH = c.head_dim, c.heads, c.kv_heads
        rep = H // KVH
        pos = np.arange(start, start + n) if pos is None else np.asarray(pos)
        x = self.embed[np.asarray(tokens)].astype(np.float64)
        for li, ly in enumerate(self.layers):
            h = rms_norm(x, ly.ln1, c.rms_eps)
            q = self._lin(h, li, 0, c.hidden, H * d).reshape(n, H, d)
            k = self._lin(h, li, 1, c.hidden, KVH * d).reshape(n, KVH, d)
            v = self._lin(h, li, 2, c.hidden, KVH * d).reshape(n, KVH, d)
            q = rope(q, pos, c.rope_theta)
            k = rope(k, pos, c.rope_theta)
            if self.kv_bf16:
                k = bf16_round(k).astype(np.float64)
                v = bf16_round(v).astype(np.float64)
            for i in range(n):
                self.kc[li, :, start + i] = k[i]
                self.vc[li, :, start + i] = v[i]
            att = np.zeros((n, H, d))
            for i in range(n):
                vis = list(range(start))
                for j in range(n):
                    ok = ((tree_mask[i] >> j) & 1) if tree_mask is not None else j <= i
                    if ok:
                        vis.append(start + j)
                vis = np.asarray(vis)
                for hh in range(H):
                    kv = hh // rep
                    s = (self.kc[li, kv, vis] @ q[i, hh]) / np.sqrt(d)
                    s = s - s.max()
                    p = np.exp(s)
                    p /= p.sum()
                    att[i, hh] = p @ self.vc[li, kv, vis]
            x = x + self._lin(att.reshape(n, H * d), li, 3, H * d, c.hidden)
            h2 = rms_norm(x, ly.ln2, c.rms_eps)
            g = self._lin(h2, li, 4, c.hidden, c.intermediate)
            u = self._lin(h2, li, 5, c.hidden, c.intermediate)
            x = x + self._lin(silu(g) * u, li, 6, c.intermediate, c.hidden)
        return x

    def final_hidden(self, x: np.ndarray) -> np.ndarray:
        return rms_norm(x, self.final_norm, self.cfg.rms_eps)

    def logits(self, x: np.ndarray) -> np.ndarray:
        return self.final_hidden(x) @ self.lm_head.T


def _np(t):
    """torch tensor or array -> numpy (bf16 tensors widen to float32 exactly)."""
    if hasattr(t, "detach"):
        t = t.detach().cpu()
        return t.float().numpy() if t.is_floating_point() else t.numpy()
    return np.asarray(t)


def _proj_prefix(layer: int, name: str) -> str:
    grp = "self_attn" if name in ("q_proj", "k_proj", "v_proj", "o_proj") else "mlp"
    return f"model.layers.{layer}.{grp}.{name}"


def from_runtime_state(state, n_layers: int, hidden: int, intermediate: int, heads: int,
                       kv_heads: int, vocab: int, rms_eps: float = 1e-6, rope_theta: float = 10000.0,
                       max_seq: int = 256, include_residual: bool = True,
                       kv_bf16: bool = True) -> "OracleDecoder":
    """OracleDecoder over a state dict in the runtime checkpoint layout
    (convert_hf_to_runtime.py:47-77 keys: ``*.v_sign_rt``, ``*.u_sign_rt``, ``v2``,
    ``mid``, ``u1`` and the ``_r`` residual set; a residual without its own
    ``v_sign_r_rt`` shares the main branch's V)."""
    layers = []
    for i in range(n_layers):
        projs = []
        for nm in PROJ_NAMES:
            p = _proj_prefix(i, nm)
            r = int(_np(state[f"{p}.v_sign_rt_shape"])[0])
            br = [RtBranch(_np(state[f"{p}.v_sign_rt"]), _np(state[f"{p}.v2"]).reshape(-1),
                           _np(state[f"{p}.mid"]).reshape(-1), _np(state[f"{p}.u_sign_rt"]),
                           _np(state[f"{p}.u1"]).reshape(-1), r)]
            if include_residual and f"{p}.u_sign_r_rt" in state:
                rr = int(_np(state[f"{p}.u_sign_r_rt_shape"])[1])
                shared = f"{p}.v_sign_r_rt" not in state
                br.append(RtBranch(None if shared else _np(state[f"{p}.v_sign_r_rt"]),
                                   None if shared else _np(state[f"{p}.v2_r"]).reshape(-1),
                                   _np(state[f"{p}.mid_r"]).reshape(-1), _np(state[f"{p}.u_sign_r_rt"]),
                                   _np(state[f"{p}.u1_r"]).reshape(-1), rr))
            projs.append(br)
        layers.append(OracleLayer(_np(state[f"model.layers.{i}.input_layernorm.weight"]),
                                  _np(state[f"model.layers.{i}.post_attention_layernorm.weight"]), projs))
    cfg = DecoderConfig(n_layers, hidden, intermediate, heads, kv_heads, vocab, rms_eps, rope_theta, max_seq)
    return OracleDecoder(cfg, _np(state["model.embed_tokens.weight"]), _np(state["model.norm.weight"]),
                         _np(state["lm_head.weight"]) if "lm_head.weight" in state else None, layers,
                         kv_bf16=kv_bf16)
