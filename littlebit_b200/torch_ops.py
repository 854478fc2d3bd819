"""torch.ops.littlebit_cuda_ops: the B200 library under schemas parallel to the
reference's torch.ops.littlebit_cpu_ops (patches/littlebit_cpu_optimized.cpp:2321-2377).

Importing this module registers the namespace (CUDA tensors only; there is no
CPU kernel, so a CPU tensor raises the dispatcher's "no kernel" error).  The
schemas keep the reference's argument names and order; the differences are in
the data the arguments carry:

* sign tensors are the runtime int32 row words (``v_sign_rt`` / ``u_sign_rt``,
  convert_hf_to_runtime.py:47-57) where the reference's full_forward family
  takes its lossy i2 repack (``repack_signs_to_i2``, cpp:712-870);
* KV caches are bf16 ``[kv_heads, max_seq, head_dim]`` (the reference: fp32,
  same order);
* ``generate_token`` takes the bf16 lm_head where the reference takes its Q4_0
  blocks (``quantize_lm_head_q4``), and returns the exact argmax;
* like the reference CPU runtime, fused_attention / full_forward* / generate_token
  apply no rotary embedding (the model adapters in ``cuda_models`` do).

Op list: littlebit_linear, embedding_lookup, rms_norm, dense_gemv_f32, silu_mul,
fused_attention, full_forward, full_forward_batch, generate_token.
"""
from __future__ import annotations

import ctypes
from typing import Dict, Tuple

import torch

from . import _lib as L
from . import ops
from .ops import Branch, PackedLinear, _p, _stream, lib

NS = "littlebit_cuda_ops"

SCHEMAS = {
    "littlebit_linear": "littlebit_linear(Tensor input, Tensor v2, Tensor v_sign, int v_cols, "
                        "Tensor mid, Tensor u_sign, int u_cols, Tensor u1) -> Tensor",
    "embedding_lookup": "embedding_lookup(Tensor weight, Tensor indices) -> Tensor",
    "rms_norm": "rms_norm(Tensor input, Tensor weight, float eps) -> Tensor",
    "dense_gemv_f32": "dense_gemv_f32(Tensor input, Tensor weight) -> Tensor",
    "silu_mul": "silu_mul(Tensor gate, Tensor up) -> Tensor",
    "fused_attention": "fused_attention(Tensor q, Tensor(a!) k_cache, Tensor(b!) v_cache, Tensor k_new, "
                       "Tensor v_new, int position, int num_kv_heads, int kv_repeat, int head_dim, "
                       "float attn_scale) -> Tensor",
    "full_forward": "full_forward(int token_id, Tensor embed_weight, Tensor final_norm_weight, "
                    "Tensor[] layer_tensors, Tensor(a!)[] kv_caches, int[] layer_dims, int num_layers, "
                    "int hidden_size, int num_kv_heads, int kv_repeat, int head_dim, int max_seq_len, "
                    "int position, float attn_scale, float rms_eps) -> Tensor",
    "full_forward_batch": "full_forward_batch(Tensor token_ids, Tensor embed_weight, "
                          "Tensor final_norm_weight, Tensor[] layer_tensors, Tensor(a!)[] kv_caches, "
                          "int[] layer_dims, int num_layers, int hidden_size, int num_kv_heads, "
                          "int kv_repeat, int head_dim, int max_seq_len, int start_position, "
                          "float attn_scale, float rms_eps) -> Tensor",
    "generate_token": "generate_token(int token_id, Tensor embed_weight, Tensor final_norm_weight, "
                      "Tensor[] layer_tensors, Tensor(a!)[] kv_caches, int[] layer_dims, "
                      "Tensor lm_head_q4, int vocab_size, int num_layers, int hidden_size, "
                      "int num_kv_heads, int kv_repeat, int head_dim, int max_seq_len, int position, "
                      "float attn_scale, float rms_eps) -> int",
}

TENSORS_PER_LAYER = 37  # ln1, ln2, then (v2, v_sign, mid, u_sign, u1) x 7 (cpu_draft_model.py:233-262)
DIMS_PER_LAYER = 28     # (v_cols, rank, u_cols, out_features) x 7


# ---------------------------------------------------------------------------
# decoder descriptors built from the reference's flat argument lists
# ---------------------------------------------------------------------------
class _FlatModel:
    """ctypes lbx_model over caller-owned tensors (kept alive here)."""

    def __init__(self, embed, final_norm, layer_tensors, kv_caches, layer_dims, num_layers, hidden,
                 num_kv_heads, kv_repeat, head_dim, max_seq_len, attn_scale, rms_eps, lm_head=None):
        if len(layer_tensors) != TENSORS_PER_LAYER * num_layers:
            raise RuntimeError(f"layer_tensors: expected {TENSORS_PER_LAYER * num_layers} tensors "
                               f"({TENSORS_PER_LAYER} per layer), got {len(layer_tensors)}")
        if len(layer_dims) != DIMS_PER_LAYER * num_layers:
            raise RuntimeError(f"layer_dims: expected {DIMS_PER_LAYER * num_layers} ints, got {len(layer_dims)}")
        if len(kv_caches) != 2 * num_layers:
            raise RuntimeError(f"kv_caches: expected {2 * num_layers} tensors (k, v per layer)")
        dev = embed.device
        self.device = dev
        self.embed = _bf16_exact(embed, "embed_weight")
        self.lm_head = None if lm_head is None else _bf16_exact(lm_head, "lm_head")
        self.final_norm = final_norm.to(torch.float32).contiguous()
        for t in kv_caches:
            if t.dtype != torch.bfloat16 or not t.is_cuda or tuple(t.shape) != (num_kv_heads, max_seq_len, head_dim):
                raise RuntimeError("kv_caches: bf16 CUDA tensors [num_kv_heads, max_seq_len, head_dim] expected")
        self.keep = [self.embed, self.final_norm, self.lm_head]
        self.layers = (L.Layer * num_layers)()
        inter = 0
        for li in range(num_layers):
            base = li * TENSORS_PER_LAYER
            ly = self.layers[li]
            ln1 = layer_tensors[base].to(torch.float32).contiguous().reshape(-1)
            ln2 = layer_tensors[base + 1].to(torch.float32).contiguous().reshape(-1)
            self.keep += [ln1, ln2]
            ly.ln1, ly.ln2 = _p(ln1), _p(ln2)
            for p in range(7):
                t = layer_tensors[base + 2 + 5 * p: base + 7 + 5 * p]
                v_cols, rank, u_cols, out_f = layer_dims[li * DIMS_PER_LAYER + 4 * p: li * DIMS_PER_LAYER + 4 * p + 4]
                if u_cols != rank:
                    raise RuntimeError(f"layer {li} proj {p}: u_cols {u_cols} != rank {rank}")
                v2, vs, mid, us, u1 = (x.contiguous() for x in t)
                v2, mid, u1 = (x.to(torch.float32).reshape(-1) for x in (v2, mid, u1))
                if vs.dtype != torch.int32 or us.dtype != torch.int32:
                    raise RuntimeError("sign tensors must be int32 runtime row words (v_sign_rt / u_sign_rt)")
                pl = PackedLinear(int(v_cols), int(out_f), [Branch(vs, v2, mid, us, u1, int(rank))])
                self.keep.append(pl)
                ly.proj[p] = pl.proj
                if p == 4:
                    inter = int(out_f)
            ly.k_cache, ly.v_cache = _p(kv_caches[2 * li]), _p(kv_caches[2 * li + 1])
        m = L.Model()
        m.n_layers, m.hidden, m.intermediate = num_layers, hidden, inter
        m.heads, m.kv_heads, m.head_dim = num_kv_heads * kv_repeat, num_kv_heads, head_dim
        m.vocab = self.embed.shape[0]
        m.max_seq = max_seq_len
        m.rms_eps, m.rope_theta, m.attn_scale = float(rms_eps), 0.0, float(attn_scale)
        m.use_pdl = 1
        m.embed, m.final_norm = _p(self.embed), _p(self.final_norm)
        m.lm_head = _p(self.lm_head)
        m.layers = ctypes.cast(self.layers, ctypes.POINTER(L.Layer))
        self.model = m
        self.hidden = hidden
        self.ws = torch.zeros(0, dtype=torch.uint8, device=dev)

    def run(self, ids: torch.Tensor, start: int, hidden=None, argmax=None):
        n = ids.numel()
        need = int(lib().lbx_forward_workspace_size(ctypes.byref(self.model), n))
        if need > self.ws.numel():
            self.ws = torch.zeros(need, dtype=torch.uint8, device=self.device)
        L.check(lib().lbx_forward(ctypes.byref(self.model), _p(ids), n, int(start), None, None, None,
                                  _p(hidden), None, _p(argmax), _p(self.ws), self.ws.numel(),
                                  _stream(self.device)), "full_forward")


_BF16_CACHE: Dict[Tuple[int, Tuple[int, ...]], torch.Tensor] = {}


def _bf16_exact(t: torch.Tensor, name: str) -> torch.Tensor:
    """bf16 view of an embedding / lm_head table.  An fp32 table (the reference
    passes one) is converted once and must hold bf16-representable values, as it
    does when it was widened from a bf16 checkpoint."""
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor")
    if t.dtype == torch.bfloat16:
        return t.contiguous()
    key = (t.data_ptr(), tuple(t.shape))
    b = _BF16_CACHE.get(key)
    if b is None:
        b = t.to(torch.bfloat16).contiguous()
        if not torch.equal(b.float(), t.float()):
            raise RuntimeError(f"{name}: values are not bf16-representable (the B200 tables are bf16)")
        _BF16_CACHE[key] = b
    return b


_MODELS: Dict[tuple, _FlatModel] = {}


def _flat_model(embed, final_norm, layer_tensors, kv_caches, layer_dims, num_layers, hidden, num_kv_heads,
                kv_repeat, head_dim, max_seq_len, attn_scale, rms_eps, lm_head=None) -> _FlatModel:
    key = (embed.data_ptr(), final_norm.data_ptr(), tuple(t.data_ptr() for t in layer_tensors),
           tuple(t.data_ptr() for t in kv_caches), tuple(int(d) for d in layer_dims), num_layers, hidden,
           num_kv_heads, kv_repeat, head_dim, max_seq_len, float(attn_scale), float(rms_eps),
           None if lm_head is None else lm_head.data_ptr())
    m = _MODELS.get(key)
    if m is None:
        m = _FlatModel(embed, final_norm, layer_tensors, kv_caches, layer_dims, num_layers, hidden,
                       num_kv_heads, kv_repeat, head_dim, max_seq_len, attn_scale, rms_eps, lm_head)
        _MODELS[key] = m
    return m


# ---------------------------------------------------------------------------
# op implementations
# ---------------------------------------------------------------------------
def _fused_attention(q, k_cache, v_cache, k_new, v_new, position, num_kv_heads, kv_repeat, head_dim,
                     attn_scale):
    """fused_attention (cpp:1172-1301): write k_new/v_new at ``position`` and
    attend over slots 0..position (no rotary embedding, like the reference)."""
    heads = num_kv_heads * kv_repeat
    qf = q.reshape(1, heads * head_dim).to(torch.float32).contiguous()
    kf = k_new.reshape(1, num_kv_heads * head_dim).to(torch.float32).contiguous()
    vf = v_new.reshape(1, num_kv_heads * head_dim).to(torch.float32).contiguous()
    pos = torch.tensor([position], dtype=torch.int32, device=q.device)
    out = ops.attention(qf, kf, vf, pos, k_cache, v_cache, int(position), heads, num_kv_heads, head_dim,
                        float(attn_scale), 0.0)
    return out.reshape(q.shape[:-1] + (heads * head_dim,)) if q.dim() > 1 else out.reshape(-1)


def _full_forward(token_id, embed_weight, final_norm_weight, layer_tensors, kv_caches, layer_dims,
                  num_layers, hidden_size, num_kv_heads, kv_repeat, head_dim, max_seq_len, position,
                  attn_scale, rms_eps):
    m = _flat_model(embed_weight, final_norm_weight, layer_tensors, kv_caches, layer_dims, num_layers,
                    hidden_size, num_kv_heads, kv_repeat, head_dim, max_seq_len, attn_scale, rms_eps)
    ids = torch.tensor([int(token_id)], dtype=torch.int64, device=m.device)
    out = torch.empty(1, hidden_size, dtype=torch.float32, device=m.device)
    m.run(ids, position, hidden=out)
    return out


def _full_forward_batch(token_ids, embed_weight, final_norm_weight, layer_tensors, kv_caches, layer_dims,
                        num_layers, hidden_size, num_kv_heads, kv_repeat, head_dim, max_seq_len,
                        start_position, attn_scale, rms_eps):
    m = _flat_model(embed_weight, final_norm_weight, layer_tensors, kv_caches, layer_dims, num_layers,
                    hidden_size, num_kv_heads, kv_repeat, head_dim, max_seq_len, attn_scale, rms_eps)
    ids = token_ids.reshape(-1).to(device=m.device, dtype=torch.int64).contiguous()
    n = ids.numel()
    out = torch.empty(n, hidden_size, dtype=torch.float32, device=m.device)
    for a in range(0, n, L.LBX_MAX_TOKENS):
        b = min(n, a + L.LBX_MAX_TOKENS)
        m.run(ids[a:b], start_position + a, hidden=out[a:b])
    return out


def _generate_token(token_id, embed_weight, final_norm_weight, layer_tensors, kv_caches, layer_dims,
                    lm_head_q4, vocab_size, num_layers, hidden_size, num_kv_heads, kv_repeat, head_dim,
                    max_seq_len, position, attn_scale, rms_eps):
    if lm_head_q4.dtype not in (torch.bfloat16, torch.float32) or lm_head_q4.shape[0] != vocab_size:
        raise RuntimeError("generate_token: lm_head must be the bf16 (or bf16-valued fp32) "
                           "[vocab_size, hidden] table on the B200 path")
    m = _flat_model(embed_weight, final_norm_weight, layer_tensors, kv_caches, layer_dims, num_layers,
                    hidden_size, num_kv_heads, kv_repeat, head_dim, max_seq_len, attn_scale, rms_eps,
                    lm_head=lm_head_q4)
    ids = torch.tensor([int(token_id)], dtype=torch.int64, device=m.device)
    am = torch.empty(1, dtype=torch.int64, device=m.device)
    m.run(ids, position, argmax=am)
    return int(am.item())


IMPLS = {
    "littlebit_linear": ops.littlebit_linear,
    "embedding_lookup": ops.embedding_lookup,
    "rms_norm": ops.rms_norm,
    "dense_gemv_f32": ops.dense_gemv_f32,
    "silu_mul": ops.silu_mul,
    "fused_attention": _fused_attention,
    "full_forward": _full_forward,
    "full_forward_batch": _full_forward_batch,
    "generate_token": _generate_token,
}

_LIB = None


def register() -> None:
    """Define torch.ops.littlebit_cuda_ops.* (idempotent)."""
    global _LIB
    if _LIB is not None:
        return
    lib_ = torch.library.Library(NS, "DEF")
    for name, schema in SCHEMAS.items():
        lib_.define(schema)
        lib_.impl(name, IMPLS[name], "CUDA")
    _LIB = lib_


register()
