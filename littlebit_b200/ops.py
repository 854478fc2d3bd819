"""Torch-facing wrappers of the sm_100a kernels (C ABI in include/lbx.h).

These mirror the reference's native op library
(patches/littlebit_cpu_optimized.cpp, ``torch.ops.littlebit_cpu_ops.*``,
schemas at :2321-2377) on CUDA tensors: same argument meaning, same shape
checks, RuntimeError on bad input.  There is no CPU path — CPU tensors are
rejected, and a missing kernel library raises at import of ``_lib``.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import Optional, Sequence

import torch

from . import _lib as L


# ---------------------------------------------------------------------------
# plumbing
# ---------------------------------------------------------------------------
def lib():
    return L.load()


def _stream(device: torch.device | None = None) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _p(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _cuda(name: str, t: torch.Tensor) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a tensor")
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor (the B200 library has no CPU path)")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")


def _dt(t: torch.Tensor) -> int:
    if t.dtype == torch.float32:
        return L.LBX_F32
    if t.dtype == torch.bfloat16:
        return L.LBX_BF16
    raise RuntimeError(f"unsupported activation dtype {t.dtype} (float32 or bfloat16)")


class Workspace:
    """A growable device scratch buffer (one per device and purpose).

    Zero-filled when (re)allocated: the kernels keep small bookkeeping words in
    the workspace that must start at zero and are left at zero by every call."""

    def __init__(self, device: torch.device):
        self.device = device
        self.buf = torch.zeros(0, dtype=torch.uint8, device=device)

    def get(self, nbytes: int) -> torch.Tensor:
        if self.buf.numel() < nbytes:
            self.buf = torch.zeros(max(nbytes, 2 * self.buf.numel()), dtype=torch.uint8,
                                   device=self.device)
        return self.buf


_WS: dict = {}


def workspace(device: torch.device, tag: str = "op") -> Workspace:
    key = (torch.device(device).index or 0, tag)
    if key not in _WS:
        _WS[key] = Workspace(torch.device(device))
    return _WS[key]


def device_error(device=None) -> int:
    v = ctypes.c_int32(0)
    L.check(lib().lbx_device_error(ctypes.byref(v), _stream(device)), "lbx_device_error")
    return v.value


def clear_device_error(device=None) -> None:
    L.check(lib().lbx_clear_device_error(_stream(device)), "lbx_clear_device_error")


# ---------------------------------------------------------------------------
# bit packing (quantization/utils/binary_packer.py)
# ---------------------------------------------------------------------------
def binary_packer(tensor: torch.Tensor) -> torch.Tensor:
    """±1 int8 [rows, cols] -> int32 [rows, ceil(cols/32)], LSB-first, bit 1 <=> -1
    (binary_packer.py:4-50).  Raises TypeError for non-int8 input like the reference."""
    if tensor.dtype != torch.int8:
        raise TypeError("Input tensor must be int8.")
    _cuda("tensor", tensor)
    if tensor.dim() != 2:
        raise ValueError("binary_packer expects a 2-D tensor")
    rows, cols = tensor.shape
    out = torch.empty(rows, (cols + 31) // 32, dtype=torch.int32, device=tensor.device)
    L.check(lib().lbx_pack_signs(_p(tensor), rows, cols, _p(out), None, _stream(tensor.device)),
            "binary_packer")
    return out


def binary_unpacker(packed_tensor: torch.Tensor, original_shape) -> torch.Tensor:
    """int32 words -> ±1 int8 of ``original_shape`` (binary_packer.py:53-97)."""
    _cuda("packed_tensor", packed_tensor)
    if packed_tensor.dim() == 2:
        n_rows, n_cols = (int(v) for v in original_shape)
        if tuple(packed_tensor.shape) == (n_rows, (n_cols + 31) // 32):
            if packed_tensor.dtype != torch.int32:
                raise TypeError("packed tensor must be int32")
            out = torch.empty(n_rows, n_cols, dtype=torch.int8, device=packed_tensor.device)
            L.check(lib().lbx_unpack_signs(_p(packed_tensor), n_rows, n_cols, _p(out),
                                           _stream(packed_tensor.device)), "binary_unpacker")
            return out
    raise ValueError(f"Unsupported packed tensor format. Expected 2D tensor with shape "
                     f"(n_rows, words_per_row), got {packed_tensor.shape} with "
                     f"{packed_tensor.dim()} dimensions.")


def pack_signs_from_float(w: torch.Tensor) -> torch.Tensor:
    """sign(w) (0 -> +1) packed straight from a float/bf16 latent factor
    (littlebit.py:313-317 pack_param: quantize -> int8 -> binary_packer)."""
    _cuda("w", w)
    rows, cols = w.shape
    out = torch.empty(rows, (cols + 31) // 32, dtype=torch.int32, device=w.device)
    L.check(lib().lbx_pack_signs_from_float(_p(w), _dt(w), rows, cols, _p(out), _stream(w.device)),
            "pack_signs_from_float")
    return out


# ---------------------------------------------------------------------------
# LittleBit linear
# ---------------------------------------------------------------------------
@dataclass
class Branch:
    """One LittleBit factorisation on device.  ``v_sign is None`` means the
    branch reuses branch 0's V-stage (shared-factor residual)."""
    v_sign: Optional[torch.Tensor]  # int32 [rank, ceil(in/32)]
    v2: Optional[torch.Tensor]      # fp32 [in]
    mid: torch.Tensor               # fp32 [rank]
    u_sign: torch.Tensor            # int32 [out, ceil(rank/32)]
    u1: torch.Tensor                # fp32 [out]
    rank: int


class PackedLinear:
    """Device-resident LittleBitLinear (main + optional residual branch + bias)
    with its C descriptor built once."""

    def __init__(self, in_features: int, out_features: int, branches: Sequence[Branch],
                 bias: Optional[torch.Tensor] = None):
        if not 1 <= len(branches) <= 2:
            raise ValueError("1 or 2 branches")
        self.in_features = int(in_features)
        self.out_features = int(out_features)
        self.branches = list(branches)
        self.bias = bias
        for i, b in enumerate(self.branches):
            for nm in ("mid", "u_sign", "u1"):
                _cuda(f"branch{i}.{nm}", getattr(b, nm))
            if b.v_sign is not None:
                _cuda(f"branch{i}.v_sign", b.v_sign)
                _cuda(f"branch{i}.v2", b.v2)
                if tuple(b.v_sign.shape) != (b.rank, (self.in_features + 31) // 32):
                    raise RuntimeError(f"v_sign shape {tuple(b.v_sign.shape)} != "
                                       f"({b.rank}, {(self.in_features + 31) // 32})")
            if tuple(b.u_sign.shape) != (self.out_features, (b.rank + 31) // 32):
                raise RuntimeError(f"u_sign shape {tuple(b.u_sign.shape)} != "
                                   f"({self.out_features}, {(b.rank + 31) // 32})")
        self.device = self.branches[0].u_sign.device
        self.proj = self._build()

    def _build(self) -> L.Proj:
        pr = L.Proj()
        pr.in_features = self.in_features
        pr.out_features = self.out_features
        pr.n_branches = len(self.branches)
        for i, b in enumerate(self.branches):
            br = pr.br[i]
            br.v_sign = _p(b.v_sign)
            br.v2 = _p(b.v2)
            br.mid = _p(b.mid)
            br.u_sign = _p(b.u_sign)
            br.u1 = _p(b.u1)
            br.rank = int(b.rank)
        pr.bias = _p(self.bias)
        return pr

    def packed_bytes(self) -> int:
        """Algorithmic packed-sign bytes (no word padding)."""
        tot = 0
        for b in self.branches:
            if b.v_sign is not None:
                tot += (b.rank * self.in_features + 7) // 8
            tot += (self.out_features * b.rank + 7) // 8
        return tot

    def scale_bytes(self) -> int:
        tot = 0
        for b in self.branches:
            if b.v_sign is not None:
                tot += 4 * self.in_features
            tot += 4 * (b.rank + self.out_features)
        return tot + (4 * self.out_features if self.bias is not None else 0)


def projs_array(projs: Sequence[PackedLinear]):
    arr = (L.Proj * len(projs))()
    for i, p in enumerate(projs):
        arr[i] = p.proj
    return arr


def linear_chain(layers: Sequence[PackedLinear], acts: Sequence[torch.Tensor],
                 ws: Optional[torch.Tensor] = None, arr=None, ptrs=None) -> None:
    """acts[i+1] = layers[i](acts[i]) for every layer, as one persistent program
    (lbx_linear_chain).  All activations [k, features] share one dtype."""
    n = len(layers)
    if len(acts) != n + 1:
        raise ValueError("need len(layers) + 1 activation buffers")
    for i, t in enumerate(acts):
        _cuda(f"acts[{i}]", t)
    k = acts[0].shape[0]
    if arr is None:
        arr = projs_array(layers)
    if ptrs is None:
        ptrs = (ctypes.c_void_p * (n + 1))(*[t.data_ptr() for t in acts])
    need = int(lib().lbx_linear_chain_workspace_size(arr, n, k))
    if ws is None:
        ws = workspace(acts[0].device, "chain").get(need)
    L.check(lib().lbx_linear_chain(arr, n, k, _dt(acts[0]), ptrs, _p(ws), ws.numel(),
                                   _stream(acts[0].device)), "linear_chain")


class FusedChain:
    """A chain of single-projection layers run by the fused chain executor
    (lbx_chain_fused): layer i's U-stage and layer i+1's V-stage partials in
    one launch, bit-identical to running the layers one by one.  The sign
    words are copied once into the executor's layout (lbx_chain_prepare)."""

    def __init__(self, layers: Sequence[PackedLinear]):
        self.layers = list(layers)
        self.arr = projs_array(self.layers)
        n = len(self.layers)
        nb = int(lib().lbx_chain_prepare_size(self.arr, n))
        if nb == 0:
            raise RuntimeError(f"layer chain does not fit the fused chain executor: {L.last_error()}")
        dev = self.layers[0].device
        self.blob = torch.empty(nb // 4, dtype=torch.int32, device=dev)
        L.check(lib().lbx_chain_prepare(self.arr, n, _p(self.blob), nb, _stream(dev)), "chain_prepare")
        self._ws = {}

    def workspace(self, k: int) -> torch.Tensor:
        if k not in self._ws:
            nb = int(lib().lbx_chain_fused_workspace_size(self.arr, len(self.layers), k))
            if nb == 0:
                raise RuntimeError(f"fused chain: {k} tokens unsupported: {L.last_error()}")
            self._ws[k] = torch.empty(nb, dtype=torch.uint8, device=self.layers[0].device)
        return self._ws[k]

    def run(self, acts: Sequence[torch.Tensor], ptrs=None, stream=None) -> None:
        """acts[i+1] = layers[i](acts[i]); all activations [k, features] of one dtype."""
        n = len(self.layers)
        if len(acts) != n + 1:
            raise ValueError("need len(layers) + 1 activation buffers")
        for i, t in enumerate(acts):
            _cuda(f"acts[{i}]", t)
        k = acts[0].shape[0]
        ws = self.workspace(k)
        if ptrs is None:
            ptrs = (ctypes.c_void_p * (n + 1))(*[t.data_ptr() for t in acts])
        st = _stream(acts[0].device) if stream is None else ctypes.c_void_p(stream.cuda_stream)
        L.check(lib().lbx_chain_fused(self.arr, n, k, _dt(acts[0]), ptrs, _p(self.blob), self.blob.numel() * 4,
                                      _p(ws), ws.numel(), st), "chain_fused")


def linear_workspace_bytes(projs: Sequence[PackedLinear], n_tokens: int) -> int:
    return int(lib().lbx_linear_workspace_size(projs_array(projs), len(projs), n_tokens))


def linear_args(projs: Sequence[PackedLinear], x: torch.Tensor, outs: Sequence[torch.Tensor], *,
                prologue: int = L.LBX_PRO_NONE, norm_w: Optional[torch.Tensor] = None,
                eps: float = 1e-6, x2: Optional[torch.Tensor] = None,
                epilogue: int = L.LBX_EPI_STORE, use_pdl: bool = True,
                exec_mode: int = L.LBX_EXEC_AUTO) -> L.LinearArgs:
    """The lbx_linear_args of a call (checked shapes), for callers that issue the
    C-ABI call themselves, e.g. many times over fixed buffers."""
    _cuda("x", x)
    k = x.shape[0]
    a = L.LinearArgs()
    a.n_proj = len(projs)
    a.n_tokens = k
    a.x_dtype = _dt(x)
    a.y_dtype = _dt(outs[0])
    a.prologue = prologue
    a.epilogue = epilogue
    a.eps = float(eps)
    a.use_pdl = 1 if use_pdl else 0
    a.exec = exec_mode
    a.x = _p(x)
    a.x2 = _p(x2)
    a.norm_w = _p(norm_w)
    for i, o in enumerate(outs):
        _cuda(f"out{i}", o)
        if o.shape[0] != k or o.shape[-1] != projs[i].out_features:
            raise RuntimeError(f"out{i} has shape {tuple(o.shape)}, expected ({k}, {projs[i].out_features})")
        a.y[i] = _p(o)
        a.y_ld[i] = o.stride(0)
    return a


def linear_group(projs: Sequence[PackedLinear], x: torch.Tensor, outs: Sequence[torch.Tensor], *,
                 prologue: int = L.LBX_PRO_NONE, norm_w: Optional[torch.Tensor] = None,
                 eps: float = 1e-6, x2: Optional[torch.Tensor] = None,
                 epilogue: int = L.LBX_EPI_STORE, use_pdl: bool = True,
                 ws: Optional[torch.Tensor] = None, arr=None,
                 exec_mode: int = L.LBX_EXEC_AUTO) -> None:
    """Run 1..3 LittleBit projections that share the input x [k, in].

    ``exec_mode``: LBX_EXEC_AUTO (one cluster launch when the call fits it,
    else the two stage grids), LBX_EXEC_KERNELS or LBX_EXEC_CLUSTER; all give
    the same bits."""
    a = linear_args(projs, x, outs, prologue=prologue, norm_w=norm_w, eps=eps, x2=x2, epilogue=epilogue,
                    use_pdl=use_pdl, exec_mode=exec_mode)
    k = x.shape[0]
    if arr is None:
        arr = projs_array(projs)
    need = int(lib().lbx_linear_workspace_size(arr, len(projs), k))
    if ws is None:
        ws = workspace(x.device, "linear").get(need)
    L.check(lib().lbx_linear_verify(arr, ctypes.byref(a), _p(ws), ws.numel(), _stream(x.device)),
            "littlebit_linear")


def lb_linear(layer: PackedLinear, x: torch.Tensor, out: Optional[torch.Tensor] = None,
              out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """y = LittleBitLinear(x) for x [..., in] (float32 or bfloat16)."""
    shp = x.shape
    x2d = x.reshape(-1, shp[-1]).contiguous()
    if out is None:
        out = torch.empty(x2d.shape[0], layer.out_features, dtype=out_dtype, device=x.device)
    linear_group([layer], x2d, [out])
    return out.reshape(*shp[:-1], layer.out_features)


def littlebit_linear(input: torch.Tensor, v2: torch.Tensor, v_sign: torch.Tensor, v_cols: int,
                     mid: torch.Tensor, u_sign: torch.Tensor, u_cols: int, u1: torch.Tensor) -> torch.Tensor:
    """CUDA counterpart of littlebit_cpu_ops.littlebit_linear (cpp:598-701), same
    argument checks, fp32 [M, N] output; no int8 activation quantisation."""
    for nm, t in (("input", input), ("v2", v2), ("mid", mid), ("u1", u1)):
        _cuda(nm, t)
        if t.dtype != torch.float32:
            raise RuntimeError(f"{nm} must be float32")
    for nm, t in (("v_sign", v_sign), ("u_sign", u_sign)):
        _cuda(nm, t)
        if t.dtype != torch.int32:
            raise RuntimeError(f"{nm} must be int32")
    if input.dim() != 2:
        raise RuntimeError("input must have shape [M, K]")
    if not (v2.dim() == 2 and v2.shape[0] == 1):
        raise RuntimeError("v2 must have shape [1, K]")
    if not (mid.dim() == 2 and mid.shape[0] == 1):
        raise RuntimeError("mid must have shape [1, R]")
    if not (u1.dim() == 2 and u1.shape[0] == 1):
        raise RuntimeError("u1 must have shape [1, N]")
    if input.shape[1] != v_cols or v2.shape[1] != v_cols:
        raise RuntimeError("input K must match v_cols")
    if v_sign.dim() != 2 or u_sign.dim() != 2:
        raise RuntimeError("v_sign / u_sign must be 2-D")
    if v_sign.shape[0] != mid.shape[1] or mid.shape[1] != u_cols:
        raise RuntimeError("mid rank must match v_sign rows and u_cols")
    if u_sign.shape[0] != u1.shape[1]:
        raise RuntimeError("u1 out_features must match u_sign rows")
    if v_sign.shape[1] != (v_cols + 31) // 32 or u_sign.shape[1] != (u_cols + 31) // 32:
        raise RuntimeError("packed word counts must equal ceil(cols / 32)")
    layer = PackedLinear(v_cols, u_sign.shape[0],
                         [Branch(v_sign, v2.reshape(-1), mid.reshape(-1), u_sign, u1.reshape(-1), u_cols)])
    out = torch.empty(input.shape[0], layer.out_features, dtype=torch.float32, device=input.device)
    linear_group([layer], input, [out])
    return out


# ---------------------------------------------------------------------------
# decoder pieces (CUDA counterparts of the CPU ops at cpp:973-1301)
# ---------------------------------------------------------------------------
def embedding_lookup(weight: torch.Tensor, indices: torch.Tensor) -> torch.Tensor:
    """weight [vocab, hidden] bf16 (or fp32, converted once), indices [N] or [1, N]
    -> fp32 [N, hidden]  (cpp:973-996)."""
    _cuda("weight", weight)
    if weight.dtype != torch.bfloat16:
        weight = weight.to(torch.bfloat16)
    idx = indices.reshape(-1).to(device=weight.device, dtype=torch.int64).contiguous()
    out = torch.empty(idx.numel(), weight.shape[1], dtype=torch.float32, device=weight.device)
    L.check(lib().lbx_embed(_p(weight), _p(idx), idx.numel(), weight.shape[1], weight.shape[0],
                            _p(out), _stream(weight.device)), "embedding_lookup")
    return out


def rms_norm(input: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """x * rsqrt(mean(x^2) + eps) * w over the last dim; any number of rows
    (the CPU op accepts one row, cpp:998-1052)."""
    _cuda("input", input)
    _cuda("weight", weight)
    h = weight.numel()
    x = input.reshape(-1, h)
    out = torch.empty_like(x, dtype=torch.float32)
    L.check(lib().lbx_rmsnorm(_p(x), _p(weight), x.shape[0], h, float(eps), _p(out),
                              _stream(input.device)), "rms_norm")
    return out


def silu_mul(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """SiLU(gate) * up (cpp:1117-1170), exact exp."""
    _cuda("gate", gate)
    _cuda("up", up)
    if gate.shape != up.shape:
        raise RuntimeError("gate and up must have same shape")
    out = torch.empty_like(gate)
    L.check(lib().lbx_silu_mul(_p(gate), _p(up), gate.numel(), _p(out), _stream(gate.device)),
            "silu_mul")
    return out


def rope_(x: torch.Tensor, pos: torch.Tensor, heads: int, head_dim: int, theta: float) -> torch.Tensor:
    """In-place HF-Llama rotary embedding on x [n, heads*head_dim] at positions pos [n]."""
    _cuda("x", x)
    p = pos.to(device=x.device, dtype=torch.int32).contiguous()
    L.check(lib().lbx_rope(_p(x), _p(p), x.shape[0], heads, head_dim, float(theta),
                           _stream(x.device)), "rope")
    return x


def dense_gemv_f32(input: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """lm_head GEMV (cpp:1054-1115): input [n, K] fp32, weight [N, K] bf16 -> fp32 [n, N]."""
    _cuda("input", input)
    _cuda("weight", weight)
    if weight.dtype != torch.bfloat16:
        raise RuntimeError("weight must be bfloat16 on the B200 path")
    if input.shape[-1] != weight.shape[1]:
        raise RuntimeError("input K must match weight K")
    x = input.reshape(-1, weight.shape[1]).to(torch.float32).contiguous()
    out = torch.empty(x.shape[0], weight.shape[0], dtype=torch.float32, device=x.device)
    ws = workspace(x.device, "lm").get(int(lib().lbx_lmhead_workspace_size(x.shape[0], weight.shape[0])))
    L.check(lib().lbx_lmhead_argmax(_p(x), None, 0.0, x.shape[0], weight.shape[1], _p(weight),
                                    weight.shape[0], _p(out), None, _p(ws), ws.numel(), 0,
                                    _stream(x.device)), "dense_gemv_f32")
    return out


def lmhead_argmax(x: torch.Tensor, weight: torch.Tensor, norm_w: Optional[torch.Tensor] = None,
                  eps: float = 1e-6, want_logits: bool = True):
    """Fused final RMSNorm + lm_head + argmax.  Returns (logits or None, argmax int64 [n])."""
    _cuda("x", x)
    _cuda("weight", weight)
    n = x.shape[0]
    logits = (torch.empty(n, weight.shape[0], dtype=torch.float32, device=x.device)
              if want_logits else None)
    am = torch.empty(n, dtype=torch.int64, device=x.device)
    ws = workspace(x.device, "lm").get(int(lib().lbx_lmhead_workspace_size(n, weight.shape[0])))
    L.check(lib().lbx_lmhead_argmax(_p(x), _p(norm_w), float(eps), n, weight.shape[1], _p(weight),
                                    weight.shape[0], _p(logits), _p(am), _p(ws), ws.numel(), 0,
                                    _stream(x.device)), "lmhead_argmax")
    return logits, am


def attention(q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor, pos: torch.Tensor,
              k_cache: torch.Tensor, v_cache: torch.Tensor, prefix_len: int, heads: int,
              kv_heads: int, head_dim: int, scale: float, theta: float,
              tree_mask: Optional[torch.Tensor] = None,
              rope_cs: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Attention for n new tokens (RoPE + bf16 KV write + causal/tree mask).
    ``rope_cs``: the (cos, sin) table of ``pos`` from :func:`rope_table` (the
    kernel evaluates the same values itself when it is None)."""
    for nm, t in (("q", q), ("k_new", k_new), ("v_new", v_new), ("k_cache", k_cache),
                  ("v_cache", v_cache)):
        _cuda(nm, t)
    n = q.shape[0]
    a = L.AttnArgs()
    a.n = n
    a.heads, a.kv_heads, a.head_dim = heads, kv_heads, head_dim
    a.max_seq = k_cache.shape[1]
    a.prefix_len = int(prefix_len)
    a.scale, a.theta = float(scale), float(theta)
    a.use_pdl = 0
    p32 = pos.to(device=q.device, dtype=torch.int32).contiguous()
    a.q, a.q_ld = _p(q), q.stride(0)
    a.k_new, a.v_new, a.kv_ld = _p(k_new), _p(v_new), k_new.stride(0)
    a.pos = _p(p32)
    tm = None
    if tree_mask is not None:
        tm = tree_mask.to(device=q.device, dtype=torch.int64).contiguous()
    a.tree_mask = _p(tm)
    a.k_cache, a.v_cache = _p(k_cache), _p(v_cache)
    if rope_cs is not None:
        _cuda("rope_cs", rope_cs)
        if rope_cs.dtype != torch.float32 or rope_cs.numel() != n * head_dim or not rope_cs.is_contiguous():
            raise RuntimeError("rope_cs must be a contiguous float32 [n, head_dim] table from rope_table")
        a.rope_cs = _p(rope_cs)
    out = torch.empty(n, heads * head_dim, dtype=torch.float32, device=q.device)
    a.out = _p(out)
    ws = workspace(q.device, "attn").get(int(lib().lbx_attn_workspace_size(ctypes.byref(a))))
    L.check(lib().lbx_attn_decode(ctypes.byref(a), _p(ws), ws.numel(), _stream(q.device)),
            "attention")
    return out


def rope_table(pos: torch.Tensor, head_dim: int, theta: float) -> torch.Tensor:
    """(cos, sin) of pos[i] * theta^(-2j/head_dim) for j < head_dim/2 as a float32
    [n, head_dim] table (pairs), for :func:`attention`'s ``rope_cs``."""
    _cuda("pos", pos)
    p32 = pos.to(dtype=torch.int32).contiguous()
    n = p32.numel()
    out = torch.empty(n, head_dim, dtype=torch.float32, device=pos.device)
    L.check(lib().lbx_rope_table(_p(p32), n, head_dim, float(theta), _p(out), _stream(pos.device)),
            "rope_table")
    return out


def accept_greedy_chain(draft: torch.Tensor, target_argmax: torch.Tensor) -> torch.Tensor:
    """-> int64 [2] = (accepted count, next token) on device."""
    out = torch.empty(2, dtype=torch.int64, device=target_argmax.device)
    L.check(lib().lbx_accept_greedy_chain(_p(draft), _p(target_argmax), draft.numel(), _p(out),
                                          _stream(out.device)), "accept_greedy_chain")
    return out


def accept_greedy_tree(cand: torch.Tensor, node_argmax: torch.Tensor,
                       retrieve: torch.Tensor) -> torch.Tensor:
    """-> int64 [3 + D] = (best row, accept length, bonus token, accepted node ids...)."""
    L_, D1 = retrieve.shape
    out = torch.empty(3 + D1 - 1, dtype=torch.int64, device=cand.device)
    L.check(lib().lbx_accept_greedy_tree(_p(cand), _p(node_argmax), _p(retrieve), L_, D1, _p(out),
                                         _stream(out.device)), "accept_greedy_tree")
    return out
