"""ctypes binding of the C ABI in include/lbx.h (liblbx.so, built in-tree).

There is no CPU fallback: importing the ops without the built library, or
calling them without a CUDA device, raises.
"""
from __future__ import annotations

import ctypes
from ctypes import POINTER, c_char_p, c_float, c_int, c_int32, c_int64, c_size_t, c_uint64, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "liblbx.so"

LBX_OK, LBX_EINVAL, LBX_EUNSUPPORTED, LBX_ECUDA = 0, 1, 2, 3
LBX_F32, LBX_BF16 = 0, 1
LBX_MAX_TOKENS = 16
LBX_MAX_PROJ = 3
LBX_PRO_NONE, LBX_PRO_RMSNORM, LBX_PRO_SILU_MUL, LBX_PRO_MUL = 0, 1, 2, 3
LBX_EPI_STORE, LBX_EPI_ADD, LBX_EPI_SILU0 = 0, 1, 2
LBX_EXEC_AUTO, LBX_EXEC_KERNELS, LBX_EXEC_PROGRAM, LBX_EXEC_CLUSTER = 0, 1, 2, 3
LBX_EXEC_KERNELS_ONE_CTA_V = 4
LBX_EXEC_TC, LBX_EXEC_NO_TC = 5, 6


class Branch(ctypes.Structure):
    _fields_ = [
        ("v_sign", c_void_p), ("v2", c_void_p), ("mid", c_void_p),
        ("u_sign", c_void_p), ("u1", c_void_p), ("rank", c_int32),
    ]


class Proj(ctypes.Structure):
    _fields_ = [
        ("in_features", c_int32), ("out_features", c_int32), ("n_branches", c_int32),
        ("_pad", c_int32), ("br", Branch * 2), ("bias", c_void_p),
    ]


class LinearArgs(ctypes.Structure):
    _fields_ = [
        ("n_proj", c_int32), ("n_tokens", c_int32), ("x_dtype", c_int32), ("y_dtype", c_int32),
        ("prologue", c_int32), ("epilogue", c_int32), ("eps", c_float), ("use_pdl", c_int32),
        ("x", c_void_p), ("x2", c_void_p), ("norm_w", c_void_p),
        ("y", c_void_p * LBX_MAX_PROJ), ("y_ld", c_int64 * LBX_MAX_PROJ),
        ("exec", c_int32), ("_pad", c_int32),
    ]


class AttnArgs(ctypes.Structure):
    _fields_ = [
        ("n", c_int32), ("heads", c_int32), ("kv_heads", c_int32), ("head_dim", c_int32),
        ("max_seq", c_int32), ("prefix_len", c_int32), ("scale", c_float), ("theta", c_float),
        ("use_pdl", c_int32), ("prefix_dev", c_void_p),
        ("q", c_void_p), ("q_ld", c_int64),
        ("k_new", c_void_p), ("v_new", c_void_p), ("kv_ld", c_int64),
        ("pos", c_void_p), ("tree_mask", c_void_p),
        ("k_cache", c_void_p), ("v_cache", c_void_p), ("out", c_void_p),
        ("rope_cs", c_void_p),
        ("n_seq", c_int32), ("_pad", c_int32), ("cache_seq_stride", c_int64), ("prefix_seq", c_void_p),
    ]


class Layer(ctypes.Structure):
    _fields_ = [
        ("ln1", c_void_p), ("ln2", c_void_p), ("proj", Proj * 7),
        ("k_cache", c_void_p), ("v_cache", c_void_p),
    ]


class Model(ctypes.Structure):
    _fields_ = [
        ("n_layers", c_int32), ("hidden", c_int32), ("intermediate", c_int32),
        ("heads", c_int32), ("kv_heads", c_int32), ("head_dim", c_int32),
        ("vocab", c_int32), ("max_seq", c_int32),
        ("rms_eps", c_float), ("rope_theta", c_float), ("attn_scale", c_float),
        ("use_pdl", c_int32),
        ("embed", c_void_p), ("final_norm", c_void_p), ("lm_head", c_void_p),
        ("layers", POINTER(Layer)),
        ("exec_mode", c_int32), ("_pad2", c_int32),
    ]


_SIGNATURES = {
    "lbx_linear_workspace_size": (c_size_t, [POINTER(Proj), c_int32, c_int32]),
    "lbx_linear": (c_int, [POINTER(Proj), POINTER(LinearArgs), c_void_p, c_size_t, c_void_p]),
    "lbx_linear_verify": (c_int, [POINTER(Proj), POINTER(LinearArgs), c_void_p, c_size_t, c_void_p]),
    "lbx_linear_noalloc": (c_int, [POINTER(Proj), POINTER(LinearArgs), c_void_p]),
    "lbx_linear_floor": (c_int, [POINTER(Proj), POINTER(LinearArgs), c_int32, c_void_p, c_size_t, c_void_p]),
    "lbx_linear_noalloc_max_bytes": (c_size_t, []),
    "lbx_pack_signs": (c_int, [c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_void_p]),
    "lbx_unpack_signs": (c_int, [c_void_p, c_int64, c_int64, c_void_p, c_void_p]),
    "lbx_pack_signs_from_float": (c_int, [c_void_p, c_int32, c_int64, c_int64, c_void_p, c_void_p]),
    "lbx_embed": (c_int, [c_void_p, c_void_p, c_int32, c_int32, c_int32, c_void_p, c_void_p]),
    "lbx_rmsnorm": (c_int, [c_void_p, c_void_p, c_int32, c_int32, c_float, c_void_p, c_void_p]),
    "lbx_silu_mul": (c_int, [c_void_p, c_void_p, c_int64, c_void_p, c_void_p]),
    "lbx_rope": (c_int, [c_void_p, c_void_p, c_int32, c_int32, c_int32, c_float, c_void_p]),
    "lbx_attn_workspace_size": (c_size_t, [POINTER(AttnArgs)]),
    "lbx_attn_decode": (c_int, [POINTER(AttnArgs), c_void_p, c_size_t, c_void_p]),
    "lbx_rope_table": (c_int, [c_void_p, c_int32, c_int32, c_float, c_void_p, c_void_p]),
    "lbx_lmhead_workspace_size": (c_size_t, [c_int32, c_int32]),
    "lbx_lmhead_argmax": (c_int, [c_void_p, c_void_p, c_float, c_int32, c_int32, c_void_p,
                                  c_int32, c_void_p, c_void_p, c_void_p, c_size_t, c_int32,
                                  c_void_p]),
    "lbx_accept_greedy_chain": (c_int, [c_void_p, c_void_p, c_int32, c_void_p, c_void_p]),
    "lbx_accept_greedy_tree": (c_int, [c_void_p, c_void_p, c_void_p, c_int32, c_int32,
                                       c_void_p, c_void_p]),
    "lbx_linear_chain_workspace_size": (c_size_t, [POINTER(Proj), c_int32, c_int32]),
    "lbx_linear_chain": (c_int, [POINTER(Proj), c_int32, c_int32, c_int32, POINTER(c_void_p), c_void_p,
                                 c_size_t, c_void_p]),
    "lbx_chain_prepare_size": (c_size_t, [POINTER(Proj), c_int32]),
    "lbx_chain_prepare": (c_int, [POINTER(Proj), c_int32, c_void_p, c_size_t, c_void_p]),
    "lbx_chain_fused_workspace_size": (c_size_t, [POINTER(Proj), c_int32, c_int32]),
    "lbx_chain_fused": (c_int, [POINTER(Proj), c_int32, c_int32, c_int32, POINTER(c_void_p), c_void_p, c_size_t,
                                c_void_p, c_size_t, c_void_p]),
    "lbx_linear_allgather": (c_int, [POINTER(Proj), POINTER(LinearArgs), c_int32, POINTER(c_void_p),
                                     c_int64, c_int32, c_int64, c_void_p, c_void_p, c_size_t, c_void_p]),
    "lbx_allgather_unpack": (c_int, [c_void_p, c_int64, c_int32, c_int32, c_int64, c_void_p, c_int64,
                                     c_void_p, c_int32, c_void_p]),
    "lbx_forward_workspace_size": (c_size_t, [POINTER(Model), c_int32]),
    "lbx_forward": (c_int, [POINTER(Model), c_void_p, c_int32, c_int32, c_void_p, c_void_p,
                            c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    "lbx_forward_multi_workspace_size": (c_size_t, [POINTER(Model), c_int32, c_int32]),
    "lbx_forward_multi": (c_int, [POINTER(Model), c_void_p, c_int32, c_int32, c_int32, c_void_p, c_int64,
                                  c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t,
                                  c_void_p]),
    "lbx_kv_move": (c_int, [c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int32, c_void_p,
                            c_void_p, c_int32, c_void_p]),
    "lbx_last_error": (c_int, [c_char_p, c_size_t]),
    "lbx_device_error": (c_int, [POINTER(c_int32), c_void_p]),
    "lbx_clear_device_error": (c_int, [c_void_p]),
    "lbx_version": (c_char_p, []),
}

# every symbol include/lbx.h declares (checked by the CPU test suite)
EXPORTED = tuple(_SIGNATURES)

_lib = None


def load(path: Path | None = None) -> ctypes.CDLL:
    """Load liblbx.so (once).  Raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise ImportError(
            f"{p} is missing: build the sm_100a kernels with `python -m littlebit_b200.build` "
            "(there is no CPU fallback)")
    lib = ctypes.CDLL(str(p))
    for name, (res, args) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(512)
    load().lbx_last_error(buf, 512)
    return buf.value.decode(errors="replace")


def check(rc: int, what: str = "lbx") -> None:
    if rc != LBX_OK:
        kind = {LBX_EINVAL: "invalid argument", LBX_EUNSUPPORTED: "unsupported",
                LBX_ECUDA: "CUDA error"}.get(rc, f"status {rc}")
        raise RuntimeError(f"{what}: {kind}: {last_error()}")
