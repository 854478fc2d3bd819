"""Small, fixed launch sequences of every kernel family, for profiler captures.

    python -m littlebit_b200.profile_cases [all|c2|vsplit|70b|fused|decode|allgather|tc|c5]

Each case builds seeded random layers (Bernoulli(0.5) signs, |N(1,0.1)|
scales) on cuda:0 and launches each kernel a few times in a known order, so a
capture (for instance ``ncu --metrics gpu__time_duration.sum,dram__bytes_read.sum
--clock-control none python -m littlebit_b200.profile_cases all``) lists
every kernel of the library with a small device footprint (about 0.3 GB).

  c2      the C2 layer (4096 -> 4096, ranks 208 + 1840, bf16) on the two
          stage grids at k = 1, 5 and 8 tokens
  vsplit  the 7B draft down projection (11008 -> 4096, rank 280, x * x2
          prologue): the pass-split V-stage
  70b     the 70B gate/up target call (8192 -> 2 x 28672, ranks 616 + 5736,
          RMSNorm prologue, silu(gate) epilogue) at k = 1 and 5
  fused   a chain of 8 unit-gain C2 layers on the fused chain executor, k = 1
  decode  two multi-sequence decoder steps (4 sequences) of a small model:
          attention with the sequence dimension, embedding, lm_head
  allgather  the row-sharded 8192 -> 28672 layer with the all-gather fused
          into its U-stage, two shards emulated on one GPU in stream order
  tc      the tensor-core executor (LBX_EXEC_TC) on the 70B down projection
          (28672 -> 8192, ranks 616 + 5712, x * x2 prologue) at 64 tokens,
          twice: x staging, tcgen05 V-stage, tcgen05 U-stage
  c5      two decode steps of a 2-layer Llama-2-70B-shaped target (0.1 + 0.9 bit
          ranks) for 64 sequences at 511 cached slots: the linears on the
          tensor-core executor, attention with the sequence dimension, the lm_head
          and argmax (not part of "all": ~2 GB on the device)
"""
from __future__ import annotations

import sys

import torch

from . import _lib as L
from . import ops, synthetic


def _layer(K, N, ranks, g, dev):
    return synthetic.to_packed_linear(K, N, synthetic.layer(K, N, ranks, g), dev)


def case_c2(dev, g):
    c2 = _layer(4096, 4096, [208, 1840], g, dev)
    for k in (1, 5, 8):
        x = torch.randn(k, 4096, generator=g).to(dev, torch.bfloat16)
        y = torch.empty(k, 4096, device=dev, dtype=torch.bfloat16)
        ops.linear_group([c2], x, [y], exec_mode=L.LBX_EXEC_KERNELS)


def case_vsplit(dev, g):
    dn = _layer(11008, 4096, [280], g, dev)
    x = torch.randn(1, 11008, generator=g).to(dev)
    x2 = torch.randn(1, 11008, generator=g).to(dev)
    y = torch.empty(1, 4096, device=dev)
    ops.linear_group([dn], x, [y], prologue=L.LBX_PRO_MUL, x2=x2, exec_mode=L.LBX_EXEC_KERNELS)


def case_70b(dev, g):
    gate, up = _layer(8192, 28672, [616, 5736], g, dev), _layer(8192, 28672, [616, 5736], g, dev)
    w = torch.ones(8192, device=dev)
    for k in (1, 5):
        x = torch.randn(k, 8192, generator=g).to(dev)
        ys = [torch.empty(k, 28672, device=dev) for _ in range(2)]
        ops.linear_group([gate, up], x, ys, prologue=L.LBX_PRO_RMSNORM, norm_w=w, epilogue=L.LBX_EPI_SILU0,
                         exec_mode=L.LBX_EXEC_KERNELS)


def case_fused(dev, g):
    layers = []
    for _ in range(8):
        brs = synthetic.layer(4096, 4096, [208, 1840], g)
        for b in brs:  # unit gain: the chain's activations stay finite
            b["mid"] = b["mid"] / 64.0
            b["u1"] = b["u1"] / (2 * b["rank"]) ** 0.5
        layers.append(synthetic.to_packed_linear(4096, 4096, brs, dev))
    fc = ops.FusedChain(layers)
    acts = [torch.randn(1, 4096, generator=g).to(dev, torch.bfloat16)] + \
        [torch.empty(1, 4096, device=dev, dtype=torch.bfloat16) for _ in layers]
    fc.run(acts)


def case_decode(dev, g):
    from .batch_decode import BatchDecoder
    from .model import DecoderShape, LittleBitDecoder, synthetic_runtime_state

    shape = DecoderShape(2, 512, 1024, 8, 2, 2048)
    ranks = {"q_proj": [64, 64], "k_proj": [32, 32], "v_proj": [32, 32], "o_proj": [64, 64],
             "gate_proj": [96, 96], "up_proj": [96, 96], "down_proj": [96, 96]}
    st = synthetic_runtime_state(shape, ranks, seed=1, unit_gain=True)
    dec = LittleBitDecoder(shape, st, device=dev, max_seq=16)
    bd = BatchDecoder(dec, 4, max_seq=256)
    bd.fill_synthetic_prefix(127, seed=2)
    tok = torch.randint(0, shape.vocab_size, (4,), generator=g).to(dev)
    am = torch.empty(4, dtype=torch.int64, device=dev)
    for i in range(2):
        bd.step(tok, torch.full((4,), 127 + i, dtype=torch.int32, device=dev), 127 + i, 1, argmax=am)
        tok = am.clone()


def case_allgather(dev, g):
    """The row-sharded 8192 -> 28672 layer (rank 616) with its all-gather fused
    into the U-stage, two shards emulated on one GPU in stream order (every word
    is written before the unpack that reads it starts)."""
    import ctypes

    from .sharded import RowShardedLinear

    K, N, G, k = 8192, 28672, 2, 1
    full = _layer(K, N, [616], g, dev)
    shards = [RowShardedLinear(full, G, r) for r in range(G)]
    half = k * N
    xbufs = [torch.zeros(2 * half, dtype=torch.int64, device=dev) for _ in range(G)]
    states = [torch.zeros(2, dtype=torch.int32, device=dev) for _ in range(G)]
    peers = (ctypes.c_void_p * G)(*[b.data_ptr() for b in xbufs])
    wss = [torch.zeros(ops.linear_workspace_bytes([s.local], k), dtype=torch.uint8, device=dev) for s in shards]
    lib = ops.lib()
    st = torch.cuda.current_stream().cuda_stream
    x = torch.randn(k, K, generator=g).to(dev)
    for rank, sh in enumerate(shards):
        a = L.LinearArgs()
        a.n_proj, a.n_tokens, a.x_dtype, a.y_dtype = 1, k, L.LBX_F32, L.LBX_F32
        a.epilogue, a.use_pdl, a.x = L.LBX_EPI_STORE, 0, x.data_ptr()
        L.check(lib.lbx_linear_allgather(ops.projs_array([sh.local]), ctypes.byref(a), G, peers, half, sh.lo, N,
                                         states[rank].data_ptr(), wss[rank].data_ptr(), wss[rank].numel(), st),
                "allgather")
    ys = [torch.empty(k, N, device=dev) for _ in range(G)]
    for rank in range(G):
        L.check(lib.lbx_allgather_unpack(xbufs[rank].data_ptr(), half, k, N, N, ys[rank].data_ptr(), N,
                                         states[rank].data_ptr(), 0, st), "unpack")


def case_tc(dev, g):
    dn = _layer(28672, 8192, [616, 5712], g, dev)
    k = 64
    x = torch.randn(k, 28672, generator=g).to(dev, torch.bfloat16)
    x2 = torch.randn(k, 28672, generator=g).to(dev, torch.bfloat16)
    y = torch.empty(k, 8192, device=dev, dtype=torch.bfloat16)
    ws = torch.zeros(ops.linear_workspace_bytes([dn], k), dtype=torch.uint8, device=dev)
    for _ in range(2):
        ops.linear_group([dn], x, [y], ws=ws, x2=x2, prologue=L.LBX_PRO_MUL, exec_mode=L.LBX_EXEC_TC)


def case_c5(dev, g):
    import dataclasses

    from .batch_decode import BatchDecoder
    from .littlebit import LittleBitLinear
    from .model import LLAMA2_70B, LittleBitDecoder, synthetic_runtime_state

    shape = dataclasses.replace(LLAMA2_70B, num_hidden_layers=2)
    H, I = shape.hidden_size, shape.intermediate_size
    qd, kvd = shape.num_attention_heads * shape.head_dim, shape.num_key_value_heads * shape.head_dim
    dims = {"q_proj": (H, qd), "k_proj": (H, kvd), "v_proj": (H, kvd), "o_proj": (qd, H),
            "gate_proj": (H, I), "up_proj": (H, I), "down_proj": (I, H)}
    rk = lambda b: {nm: LittleBitLinear._finalize_split_dim(LittleBitLinear._estimate_split_dim(a, o, b, False),
                                                              1024, 8) for nm, (a, o) in dims.items()}
    rd, rr = rk(0.1), rk(0.9)
    st = synthetic_runtime_state(shape, {nm: [rd[nm], rr[nm]] for nm in dims}, seed=91, device=dev,
                                 unit_gain=True)
    dec = LittleBitDecoder(shape, st, device=dev, max_seq=16)
    del st
    S = 64
    bd = BatchDecoder(dec, S, 640)
    bd.fill_synthetic_prefix(511, seed=3)
    tok = torch.randint(0, shape.vocab_size, (S,), generator=g).to(dev)
    am = torch.empty(S, dtype=torch.int64, device=dev)
    st = torch.full((S,), 511, dtype=torch.int32, device=dev)
    for _ in range(2):
        bd.step(tok, st, 511, 1, argmax=am)


CASES = {"c2": case_c2, "vsplit": case_vsplit, "70b": case_70b, "fused": case_fused, "decode": case_decode,
         "allgather": case_allgather, "tc": case_tc, "c5": case_c5}
ALL_SKIPS = ("c5",)


def main(argv):
    which = argv[1] if len(argv) > 1 else "all"
    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(0)
    for name, fn in CASES.items():
        if which == name or (which == "all" and name not in ALL_SKIPS):
            fn(dev, g)
    torch.cuda.synchronize()
    print("ok", which)


if __name__ == "__main__":
    main(sys.argv)
