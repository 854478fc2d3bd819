"""Device-resident LittleBit Llama decoder driven by the native step runner.

The weights come in the reference's runtime checkpoint layout
(convert_hf_to_runtime.py:29-97): per projection
``{prefix}.u_sign_rt / v_sign_rt (+ _shape) / u1 / v2 / mid`` and, for a
residual branch, ``u_sign_r_rt / v_sign_r_rt / u1_r / v2_r / mid_r``; plus
``model.embed_tokens.weight``, ``model.layers.{i}.{input,post_attention}_layernorm.weight``,
``model.norm.weight`` and ``lm_head.weight``.  Packed words stay exactly as
stored (the HBM layout is the checkpoint layout); scales become fp32; the
embedding and lm_head are bf16.

The KV cache of layer l is [kv_heads, max_seq, head_dim] bf16, the layout of
the reference's per-layer cache (cpu_draft_model.py:213-225 passes
``layer_cache.key / .value`` of shape [kvh, max_seq, d] to full_forward,
patches/littlebit_cpu_optimized.cpp:1183-1187) at half the width.

One ``step`` = ``lbx_forward`` (include/lbx.h): a native C++ runner launching
embedding -> L x (q/k/v with fused RMSNorm, attention with RoPE and KV write,
o + residual, gate/up with fused RMSNorm, down with fused SiLU·mul + residual)
-> final RMSNorm + lm_head + argmax, all on one stream with programmatic
dependent launch.
"""
from __future__ import annotations

import ctypes
import json
import math
from dataclasses import asdict, dataclass
from pathlib import Path
from typing import Dict, List, Optional, Sequence

import torch

from . import _lib as L
from .ops import Branch, PackedLinear, _p, _stream, lib

PROJ_NAMES = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")


def proj_prefix(layer: int, name: str) -> str:
    grp = "self_attn" if name in ("q_proj", "k_proj", "v_proj", "o_proj") else "mlp"
    return f"model.layers.{layer}.{grp}.{name}"


@dataclass
class DecoderShape:
    """dummy_llama3_config.json fields (convert_hf_to_runtime.py:193-213) plus RoPE."""
    num_hidden_layers: int
    hidden_size: int
    intermediate_size: int
    num_attention_heads: int
    num_key_value_heads: int
    vocab_size: int
    rms_norm_eps: float = 1e-6
    rope_theta: float = 10000.0
    name: str = "littlebit-llama"

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_attention_heads

    @classmethod
    def from_json(cls, d: dict) -> "DecoderShape":
        keys = {k for k in cls.__dataclass_fields__}
        return cls(**{k: v for k, v in d.items() if k in keys})


LLAMA2_7B = DecoderShape(32, 4096, 11008, 32, 32, 32000, 1e-6, 10000.0, "llama-2-7b-shape")
LLAMA2_70B = DecoderShape(80, 8192, 28672, 64, 8, 32000, 1e-5, 10000.0, "llama-2-70b-shape")


def _f32(t: torch.Tensor, device) -> torch.Tensor:
    return t.reshape(-1).to(device=device, dtype=torch.float32).contiguous()


def _words(t: torch.Tensor, device) -> torch.Tensor:
    return t.to(device=device, dtype=torch.int32).contiguous()


def branches_from_runtime(state: Dict[str, torch.Tensor], prefix: str, device,
                          include_residual: bool = True) -> List[Branch]:
    """Runtime keys of one projection -> device branches (main [+ residual])."""
    vs = state[f"{prefix}.v_sign_rt_shape"]
    rank = int(vs[0])
    br = [Branch(_words(state[f"{prefix}.v_sign_rt"], device), _f32(state[f"{prefix}.v2"], device),
                 _f32(state[f"{prefix}.mid"], device), _words(state[f"{prefix}.u_sign_rt"], device),
                 _f32(state[f"{prefix}.u1"], device), rank)]
    if include_residual and f"{prefix}.u_sign_r_rt" in state:
        rr = int(state[f"{prefix}.u_sign_r_rt_shape"][1])
        if f"{prefix}.v_sign_r_rt" in state:
            br.append(Branch(_words(state[f"{prefix}.v_sign_r_rt"], device),
                             _f32(state[f"{prefix}.v2_r"], device), _f32(state[f"{prefix}.mid_r"], device),
                             _words(state[f"{prefix}.u_sign_r_rt"], device),
                             _f32(state[f"{prefix}.u1_r"], device), rr))
        else:  # shared-factor residual: reuses the main V and v2 (littlebit_itq_spec.py:298-309)
            br.append(Branch(None, None, _f32(state[f"{prefix}.mid_r"], device),
                             _words(state[f"{prefix}.u_sign_r_rt"], device),
                             _f32(state[f"{prefix}.u1_r"], device), rr))
    return br


class LittleBitDecoder:
    """A LittleBit Llama decoder resident on one GPU, with its own KV cache."""

    def __init__(self, shape: DecoderShape, state: Dict[str, torch.Tensor], device="cuda",
                 max_seq: int = 4096, include_residual: bool = True, use_pdl: bool = True,
                 lm_head: Optional[torch.Tensor] = None, embed: Optional[torch.Tensor] = None,
                 exec_mode: int = L.LBX_EXEC_AUTO):
        """``exec_mode``: LBX_EXEC_AUTO / LBX_EXEC_KERNELS launch one grid per
        op; LBX_EXEC_PROGRAM runs a step of up to 16 tokens as one persistent
        cooperative program (same numerics)."""
        self.shape = shape
        self.device = torch.device(device)
        self.max_seq = int(max_seq)
        self.use_pdl = use_pdl
        self.exec_mode = exec_mode
        dev = self.device
        H = shape.hidden_size
        emb = embed if embed is not None else state["model.embed_tokens.weight"]
        self.embed = emb.to(device=dev, dtype=torch.bfloat16).contiguous()
        head = lm_head if lm_head is not None else state.get("lm_head.weight")
        self.lm_head = None if head is None else head.to(device=dev, dtype=torch.bfloat16).contiguous()
        self.final_norm = _f32(state["model.norm.weight"], dev)
        self.layers = []
        for i in range(shape.num_hidden_layers):
            pre = f"model.layers.{i}"
            projs = []
            for nm in PROJ_NAMES:
                in_f = H if nm not in ("down_proj",) else shape.intermediate_size
                if nm == "o_proj":
                    in_f = shape.num_attention_heads * shape.head_dim
                out_f = {"q_proj": shape.num_attention_heads * shape.head_dim,
                         "k_proj": shape.num_key_value_heads * shape.head_dim,
                         "v_proj": shape.num_key_value_heads * shape.head_dim,
                         "o_proj": H, "gate_proj": shape.intermediate_size,
                         "up_proj": shape.intermediate_size, "down_proj": H}[nm]
                projs.append(PackedLinear(in_f, out_f, branches_from_runtime(
                    state, proj_prefix(i, nm), dev, include_residual)))
            self.layers.append({
                "ln1": _f32(state[f"{pre}.input_layernorm.weight"], dev),
                "ln2": _f32(state[f"{pre}.post_attention_layernorm.weight"], dev),
                "projs": projs,
            })
        kvs = (shape.num_key_value_heads, self.max_seq, shape.head_dim)
        self.k_cache = [torch.zeros(kvs, dtype=torch.bfloat16, device=dev) for _ in self.layers]
        self.v_cache = [torch.zeros(kvs, dtype=torch.bfloat16, device=dev) for _ in self.layers]
        self._build_struct()
        self._ws = torch.zeros(0, dtype=torch.uint8, device=dev)
        self._ws_n = 0

    # ---- native descriptors -------------------------------------------------
    def _build_struct(self):
        s = self.shape
        self._layer_arr = (L.Layer * len(self.layers))()
        for i, ly in enumerate(self.layers):
            c = self._layer_arr[i]
            c.ln1 = _p(ly["ln1"])
            c.ln2 = _p(ly["ln2"])
            for j, pr in enumerate(ly["projs"]):
                c.proj[j] = pr.proj
            c.k_cache = _p(self.k_cache[i])
            c.v_cache = _p(self.v_cache[i])
        m = L.Model()
        m.n_layers = len(self.layers)
        m.hidden = s.hidden_size
        m.intermediate = s.intermediate_size
        m.heads = s.num_attention_heads
        m.kv_heads = s.num_key_value_heads
        m.head_dim = s.head_dim
        m.vocab = s.vocab_size
        m.max_seq = self.max_seq
        m.rms_eps = s.rms_norm_eps
        m.rope_theta = s.rope_theta
        m.attn_scale = 1.0 / math.sqrt(s.head_dim)
        m.use_pdl = 1 if self.use_pdl else 0
        m.exec_mode = int(getattr(self, "exec_mode", L.LBX_EXEC_AUTO))
        m.embed = _p(self.embed)
        m.final_norm = _p(self.final_norm)
        m.lm_head = _p(self.lm_head)
        m.layers = ctypes.cast(self._layer_arr, ctypes.POINTER(L.Layer))
        self._model = m

    def workspace(self, n: int) -> torch.Tensor:
        if n > self._ws_n:
            need = int(lib().lbx_forward_workspace_size(ctypes.byref(self._model), n))
            if need > self._ws.numel():
                self._ws = torch.zeros(need, dtype=torch.uint8, device=self.device)
            self._ws_n = n
        return self._ws

    def packed_bytes(self) -> int:
        return sum(p.packed_bytes() for ly in self.layers for p in ly["projs"])

    def scale_bytes(self) -> int:
        return sum(p.scale_bytes() for ly in self.layers for p in ly["projs"]) + \
            4 * self.shape.hidden_size * (2 * len(self.layers) + 1)

    # ---- one step ----------------------------------------------------------
    def step(self, tokens: torch.Tensor, start: int, *, pos: Optional[torch.Tensor] = None,
             tree_mask: Optional[torch.Tensor] = None, logits: Optional[torch.Tensor] = None,
             argmax: Optional[torch.Tensor] = None, hidden: Optional[torch.Tensor] = None,
             start_dev: Optional[torch.Tensor] = None) -> None:
        """Run n tokens (device int64 [n]) at cache slots start..start+n-1.
        Writes into the given output tensors (any of logits [n,V] fp32, argmax [n]
        int64, hidden [n,H] fp32 final-norm output).  With ``start_dev`` (device
        int32 [1]) the slot offset is read on the device and ``start`` is an upper
        bound, so the launch sequence can be captured once and replayed."""
        n = int(tokens.numel())
        if start + n > self.max_seq:
            raise RuntimeError(f"KV cache full: {start}+{n} > max_seq {self.max_seq}")
        ws = self.workspace(n)
        L.check(lib().lbx_forward(ctypes.byref(self._model), _p(tokens), n, int(start), _p(start_dev),
                                  _p(pos), _p(tree_mask), _p(hidden), _p(logits), _p(argmax), _p(ws),
                                  ws.numel(), _stream(self.device)), "lbx_forward")

    def forward_tokens(self, tokens, start: int, *, pos=None, tree_mask=None, want_logits=True,
                       want_argmax=True, want_hidden=False):
        """Convenience: allocate outputs and run ``step``; returns a dict."""
        dev = self.device
        tok = torch.as_tensor(tokens, dtype=torch.int64).reshape(-1).to(dev)
        n = tok.numel()
        out = {}
        lg = torch.empty(n, self.shape.vocab_size, dtype=torch.float32, device=dev) if want_logits else None
        am = torch.empty(n, dtype=torch.int64, device=dev) if want_argmax else None
        hd = torch.empty(n, self.shape.hidden_size, dtype=torch.float32, device=dev) if want_hidden else None
        p = None if pos is None else torch.as_tensor(pos, dtype=torch.int32).reshape(-1).to(dev)
        tm = None if tree_mask is None else torch.as_tensor(tree_mask, dtype=torch.int64).reshape(-1).to(dev)
        if (want_logits or want_argmax) and self.lm_head is None:
            raise RuntimeError("this model has no lm_head")
        self.step(tok, start, pos=p, tree_mask=tm, logits=lg, argmax=am, hidden=hd)
        out["logits"], out["argmax"], out["hidden"] = lg, am, hd
        return out


# ---------------------------------------------------------------------------
# synthetic weights in the runtime layout (BASELINE distributions)
# ---------------------------------------------------------------------------
def synthetic_runtime_state(shape: DecoderShape, ranks: Dict[str, Sequence[int]], seed: int = 0,
                            shared_residual: bool = False, device="cpu",
                            with_embed: bool = True, unit_gain: bool = False) -> Dict[str, torch.Tensor]:
    """Random LittleBit Llama in runtime layout.  ``ranks[name]`` lists the rank of
    the main branch and optionally of the residual branch of each projection.
    Signs Bernoulli(0.5) (uniform random words, pad bits cleared), scales
    |N(1,0.1)|, norms |N(1,0.1)|, embed / lm_head bf16 N(0, 0.02).

    With |N(1,0.1)| scales a projection has gain about sqrt(in_features * rank),
    so activations grow by orders of magnitude per layer and attention turns
    one-hot on scores of 1e5 and more, where one bf16 ulp of a cached key moves
    the output.  ``unit_gain`` divides mid by sqrt(in_features) and u1 by
    sqrt(rank), which keeps every projection near unit gain (the regime of
    trained checkpoints) for comparisons against a float64 oracle."""
    g = torch.Generator(device=device).manual_seed(seed)
    dev = torch.device(device)

    def words(rows, cols):
        w = torch.randint(-(2 ** 31), 2 ** 31, (rows, (cols + 31) // 32), generator=g, device=dev,
                          dtype=torch.int64)
        if cols % 32:
            w[:, -1] &= (1 << (cols % 32)) - 1
        return w.to(torch.int32)

    def sc(*shp):
        return (1 + 0.1 * torch.randn(*shp, generator=g, device=dev)).abs()

    H, I = shape.hidden_size, shape.intermediate_size
    qd = shape.num_attention_heads * shape.head_dim
    kvd = shape.num_key_value_heads * shape.head_dim
    dims = {"q_proj": (H, qd), "k_proj": (H, kvd), "v_proj": (H, kvd), "o_proj": (qd, H),
            "gate_proj": (H, I), "up_proj": (H, I), "down_proj": (I, H)}
    st: Dict[str, torch.Tensor] = {}
    if with_embed:
        st["model.embed_tokens.weight"] = (0.02 * torch.randn(shape.vocab_size, H, generator=g, device=dev)).bfloat16()
        st["lm_head.weight"] = (0.02 * torch.randn(shape.vocab_size, H, generator=g, device=dev)).bfloat16()
    st["model.norm.weight"] = sc(H)
    for i in range(shape.num_hidden_layers):
        st[f"model.layers.{i}.input_layernorm.weight"] = sc(H)
        st[f"model.layers.{i}.post_attention_layernorm.weight"] = sc(H)
        for nm in PROJ_NAMES:
            in_f, out_f = dims[nm]
            pre = proj_prefix(i, nm)
            rk = list(ranks[nm])
            r = rk[0]
            st[f"{pre}.v_sign_rt"] = words(r, in_f)
            st[f"{pre}.v_sign_rt_shape"] = torch.tensor([r, in_f], dtype=torch.int64)
            st[f"{pre}.u_sign_rt"] = words(out_f, r)
            st[f"{pre}.u_sign_rt_shape"] = torch.tensor([out_f, r], dtype=torch.int64)
            st[f"{pre}.v2"] = sc(1, in_f)
            g_mid = 1.0 / math.sqrt(in_f) if unit_gain else 1.0
            st[f"{pre}.mid"] = sc(1, r) * g_mid
            st[f"{pre}.u1"] = sc(1, out_f) * (1.0 / math.sqrt(r) if unit_gain else 1.0)
            if len(rk) > 1:
                rr = rk[1]
                if not shared_residual:
                    st[f"{pre}.v_sign_r_rt"] = words(rr, in_f)
                    st[f"{pre}.v_sign_r_rt_shape"] = torch.tensor([rr, in_f], dtype=torch.int64)
                    st[f"{pre}.v2_r"] = sc(1, in_f)
                st[f"{pre}.u_sign_r_rt"] = words(out_f, rr)
                st[f"{pre}.u_sign_r_rt_shape"] = torch.tensor([out_f, rr], dtype=torch.int64)
                st[f"{pre}.mid_r"] = sc(1, rr) * g_mid
                st[f"{pre}.u1_r"] = sc(1, out_f) * (1.0 / math.sqrt(rr) if unit_gain else 1.0)
    return st


def draft_ranks(shape: DecoderShape, eff_bit: float = 0.1) -> Dict[str, List[int]]:
    """Ranks LittleBitLinear picks at ``eff_bit`` (littlebit.py:50-80)."""
    from .littlebit import LittleBitLinear

    H, I = shape.hidden_size, shape.intermediate_size
    qd = shape.num_attention_heads * shape.head_dim
    kvd = shape.num_key_value_heads * shape.head_dim
    dims = {"q_proj": (H, qd), "k_proj": (H, kvd), "v_proj": (H, kvd), "o_proj": (qd, H),
            "gate_proj": (H, I), "up_proj": (H, I), "down_proj": (I, H)}
    out = {}
    for nm, (a, b) in dims.items():
        f = LittleBitLinear._estimate_split_dim(a, b, eff_bit, False)
        out[nm] = [LittleBitLinear._finalize_split_dim(f, 1024, 8)]
    return out


def save_runtime(path, state: Dict[str, torch.Tensor], shape: DecoderShape, eff_bit: float = 0.1,
                 residual: bool = False) -> Path:
    """Write littlebit_runtime.safetensors + littlebit_runtime_config.json +
    dummy_llama3_config.json (convert_hf_to_runtime.py:260-281 file set)."""
    from safetensors.torch import save_file

    from .runtime import build_dummy_config, build_runtime_config

    p = Path(path)
    p.mkdir(parents=True, exist_ok=True)
    save_file({k: v.contiguous().cpu() for k, v in state.items()}, str(p / "littlebit_runtime.safetensors"))
    hf_cfg = {"_name_or_path": shape.name, "hidden_size": shape.hidden_size,
              "intermediate_size": shape.intermediate_size,
              "num_hidden_layers": shape.num_hidden_layers,
              "num_attention_heads": shape.num_attention_heads,
              "num_key_value_heads": shape.num_key_value_heads, "vocab_size": shape.vocab_size,
              "rms_norm_eps": shape.rms_norm_eps, "model_type": "llama"}
    lb_cfg = {"eff_bit": eff_bit, "residual": residual, "quant_func": "STEBinary"}
    (p / "littlebit_runtime_config.json").write_text(json.dumps(build_runtime_config(hf_cfg, lb_cfg), indent=2))
    dummy = build_dummy_config(hf_cfg, lb_cfg)
    dummy["rope_theta"] = shape.rope_theta
    (p / "dummy_llama3_config.json").write_text(json.dumps(dummy, indent=2))
    return p


def load_runtime(path, device="cpu"):
    """Read a runtime checkpoint directory -> (state dict, DecoderShape, runtime config)."""
    from safetensors.torch import load_file

    p = Path(path)
    state = load_file(str(p / "littlebit_runtime.safetensors"), device=str(device))
    dummy = json.loads((p / "dummy_llama3_config.json").read_text())
    rt = {}
    if (p / "littlebit_runtime_config.json").exists():
        rt = json.loads((p / "littlebit_runtime_config.json").read_text())
    return state, DecoderShape.from_json(dummy), rt
