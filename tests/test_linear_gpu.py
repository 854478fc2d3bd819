"""CUDA LittleBitLinear and bit packing vs the CPU oracle (seeded inputs).

Bars: packed words bit-exact; per-layer outputs within rtol 1e-3 of the fp64
restatement of LittleBitLinear._compute_forward (abs floor 1e-4 x max|y|);
a token's output bit-identical whatever verify batch it is computed in.
"""
import numpy as np
import pytest
import torch

from helpers import assert_linear_close, oracle_branches, rel_err
from oracle import littlebit as olb
from oracle import packing as opk

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def ops():
    from littlebit_b200 import ops as o

    o.clear_device_error()
    yield o
    torch.cuda.synchronize()
    assert o.device_error() == 0


def _gen(seed):
    return torch.Generator().manual_seed(seed)


@pytest.mark.parametrize("shape", [(2, 40), (5, 33), (3, 1), (16, 1840), (4096, 208), (208, 4096),
                                   (7, 64), (0, 5)])
def test_pack_bitexact(ops, shape):
    g = _gen(1)
    s = (torch.randint(0, 2, shape, generator=g, dtype=torch.int8) * 2 - 1)
    p = ops.binary_packer(s.to(DEV)).cpu().numpy()
    ref = opk.binary_packer(s.numpy()) if shape[0] else np.zeros((0, (shape[1] + 31) // 32), np.int32)
    assert np.array_equal(p, ref)
    u = ops.binary_unpacker(torch.from_numpy(ref).to(DEV), shape).cpu().numpy()
    assert np.array_equal(u, s.numpy())


def test_pack_golden(ops, golden):
    gd = golden("packing")
    for n in sorted({k.rsplit("_", 1)[0] for k in gd.files}):
        s = torch.from_numpy(gd[f"{n}_signs"]).to(DEV)
        assert np.array_equal(ops.binary_packer(s).cpu().numpy(), gd[f"{n}_packed"]), n


def test_pack_from_float_sign_convention(ops):
    w = torch.tensor([[0.0, -0.0, -1.5, 2.0, -1e-30] + [1.0] * 30], device=DEV)
    p = ops.pack_signs_from_float(w).cpu().numpy()
    ref = opk.binary_packer(opk.sign(w.cpu().numpy()).astype(np.int8))
    assert np.array_equal(p, ref)
    pb = ops.pack_signs_from_float(w.bfloat16()).cpu().numpy()
    assert np.array_equal(pb, ref)


def test_pack_rejects(ops):
    with pytest.raises(TypeError):
        ops.binary_packer(torch.ones(2, 3, dtype=torch.int32, device=DEV))
    with pytest.raises(RuntimeError):
        ops.binary_packer(torch.ones(2, 3, dtype=torch.int8))  # CPU tensor: no CPU path


def _layer(ops, in_f, out_f, ranks, seed, shared=False, bias=False):
    from littlebit_b200 import synthetic as syn

    g = _gen(seed)
    brs = syn.layer(in_f, out_f, ranks, g, shared_residual=shared)
    b = torch.randn(out_f, generator=g) if bias else None
    return brs, b, syn.to_packed_linear(in_f, out_f, brs, DEV, bias=b)


def _ref(x, brs, in_f, out_f, bias=None):
    return olb.linear_forward(x.double().numpy(), oracle_branches(brs), in_f, out_f,
                              bias=None if bias is None else bias.numpy())


@pytest.mark.parametrize("case", [
    ("c1", 4096, 4096, [208], 1, torch.float32),
    ("c2_k1", 4096, 4096, [208, 1840], 1, torch.bfloat16),
    ("c2_k5", 4096, 4096, [208, 1840], 5, torch.bfloat16),
    ("c2_k8", 4096, 4096, [208, 1840], 8, torch.bfloat16),
    ("down", 11008, 4096, [280], 3, torch.float32),
    ("gate", 4096, 11008, [280], 2, torch.float32),
    ("odd_rank", 256, 128, [40, 8], 4, torch.float32),
    ("k9", 512, 256, [184, 96], 9, torch.float32),
    ("k12", 1024, 512, [64, 40], 12, torch.bfloat16),
    ("k16", 512, 256, [184], 16, torch.float32),
    ("k20", 512, 256, [96], 20, torch.float32),
    ("tiny", 128, 16, [8], 1, torch.float32),
])
def test_linear_matches_oracle(ops, case):
    name, in_f, out_f, ranks, k, dt = case
    brs, _, lay = _layer(ops, in_f, out_f, ranks, seed=sum(map(ord, name)))
    x = torch.randn(k, in_f, generator=_gen(7)).to(dt)
    y = ops.lb_linear(lay, x.to(DEV)).cpu()
    ref = _ref(x.float(), brs, in_f, out_f)
    assert_linear_close(y.numpy(), ref)
    assert rel_err(y.numpy(), ref) < 2e-4


def test_linear_shared_residual_and_bias(ops):
    brs, b, lay = _layer(ops, 1024, 512, [96, 96], seed=3, shared=True, bias=True)
    x = torch.randn(3, 1024, generator=_gen(8))
    y = ops.lb_linear(lay, x.to(DEV)).cpu().numpy()
    assert_linear_close(y, _ref(x, brs, 1024, 512, bias=b))


def test_verify_batch_bit_identical_to_batch1(ops):
    brs, _, lay = _layer(ops, 4096, 4096, [208, 1840], seed=4)
    x = torch.randn(8, 4096, generator=_gen(9)).bfloat16().to(DEV)
    yk = ops.lb_linear(lay, x)
    for i in range(8):
        y1 = ops.lb_linear(lay, x[i:i + 1])
        assert torch.equal(y1[0], yk[i]), i
    y5 = ops.lb_linear(lay, x[2:7])
    assert torch.equal(y5, yk[2:7])


def test_prologues_epilogues_groups(ops):
    from littlebit_b200 import _lib as L

    g = _gen(12)
    H, I, k = 512, 768, 3
    layers = [_layer(ops, H, o, [64], seed=20 + i) for i, o in enumerate((H, 256, 256))]
    x = torch.randn(k, H, generator=g)
    w = (1 + 0.1 * torch.randn(H, generator=g)).abs()
    outs = [torch.empty(k, l[2].out_features, device=DEV) for l in layers]
    ops.linear_group([l[2] for l in layers], x.to(DEV), outs, prologue=L.LBX_PRO_RMSNORM,
                     norm_w=w.to(DEV), eps=1e-6)
    xn = x.double() / torch.sqrt((x.double() ** 2).mean(-1, keepdim=True) + 1e-6) * w.double()
    for (brs, _, lay), o in zip(layers, outs):
        assert_linear_close(o.cpu().numpy(), _ref(xn, brs, H, lay.out_features))
    # SiLU-mul prologue + residual-add epilogue (the down projection)
    brs, _, dn = _layer(ops, I, H, [80], seed=30)
    gt, up = torch.randn(k, I, generator=g), torch.randn(k, I, generator=g)
    res = torch.randn(k, H, generator=g)
    y = res.clone().to(DEV)
    ops.linear_group([dn], gt.to(DEV), [y], prologue=L.LBX_PRO_SILU_MUL, x2=up.to(DEV),
                     epilogue=L.LBX_EPI_ADD)
    a = torch.nn.functional.silu(gt.double()) * up.double()
    assert_linear_close(y.cpu().numpy() - res.numpy(), _ref(a, brs, I, H), atol_frac=2e-4)


def test_reference_schema_littlebit_linear(ops):
    from littlebit_b200 import synthetic as syn

    g = _gen(13)
    b = syn.branch(256, 384, 40, g)
    x = torch.randn(2, 256, generator=g)
    y = ops.littlebit_linear(x.to(DEV), b["v2"][None].to(DEV), b["v_sign"].to(DEV), 256,
                             b["mid"][None].to(DEV), b["u_sign"].to(DEV), 40, b["u1"][None].to(DEV))
    assert_linear_close(y.cpu().numpy(), _ref(x, [b], 256, 384))
    with pytest.raises(RuntimeError):  # shape checks as cpp:608-634
        ops.littlebit_linear(x.to(DEV), b["v2"][None].to(DEV), b["v_sign"].to(DEV), 255,
                             b["mid"][None].to(DEV), b["u_sign"].to(DEV), 40, b["u1"][None].to(DEV))


def test_unsupported_shapes_raise(ops):
    from littlebit_b200 import synthetic as syn

    brs = syn.layer(96, 64, [16], _gen(1))  # in_features not a multiple of 128
    lay = syn.to_packed_linear(96, 64, brs, DEV)
    with pytest.raises(RuntimeError, match="unsupported"):
        ops.lb_linear(lay, torch.randn(1, 96, device=DEV))


def test_pdl_chain_matches_unchained(ops):
    # a chain of layers launched back to back with programmatic dependent launch
    # must equal the same layers run one at a time
    layers = [_layer(ops, 1024, 1024, [96, 256], seed=40 + i)[2] for i in range(6)]
    x0 = torch.randn(3, 1024, generator=_gen(41)).bfloat16().to(DEV)
    acts = [x0] + [torch.empty(3, 1024, dtype=torch.bfloat16, device=DEV) for _ in layers]
    for i, l in enumerate(layers):
        ops.linear_group([l], acts[i], [acts[i + 1]], use_pdl=True)
    y = x0
    for i, l in enumerate(layers):
        y2 = torch.empty_like(y)
        ops.linear_group([l], y, [y2], use_pdl=False)
        torch.cuda.synchronize()
        assert torch.equal(y2, acts[i + 1]), i
        y = y2


def test_c2_k16(ops):
    brs, _, lay = _layer(ops, 4096, 4096, [208, 1840], seed=77)
    x = torch.randn(16, 4096, generator=_gen(78)).bfloat16()
    y = ops.lb_linear(lay, x.to(DEV)).cpu()
    assert_linear_close(y.numpy(), _ref(x.float(), brs, 4096, 4096))
    y1 = ops.lb_linear(lay, x[5:6].to(DEV)).cpu()
    assert torch.equal(y1[0], y[5])


def test_linear_chain_program_matches_layer_calls():
    """lbx_linear_chain (all layers in one persistent program) equals calling
    lbx_linear layer by layer, bit for bit, for k = 1, 5 and 12 bf16 tokens."""
    from littlebit_b200 import ops, synthetic

    g = torch.Generator().manual_seed(77)
    layers = []
    for i in range(6):
        ranks = [208, 1840] if i % 2 == 0 else [96]
        layers.append(synthetic.to_packed_linear(4096, 4096, synthetic.layer(4096, 4096, ranks, g), "cuda"))
    for k in (1, 5, 12):
        x = torch.randn(k, 4096, generator=g).bfloat16().cuda()
        acts = [x] + [torch.empty(k, 4096, dtype=torch.bfloat16, device="cuda") for _ in layers]
        ops.linear_chain(layers, acts)
        ref = x
        for lay in layers:
            y = torch.empty(k, 4096, dtype=torch.bfloat16, device="cuda")
            ops.linear_group([lay], ref, [y])
            ref = y
        torch.cuda.synchronize()
        assert torch.equal(acts[-1], ref), k
        assert ops.device_error() == 0


def test_allgather_exchange_two_shards_one_gpu():
    """lbx_linear_allgather + lbx_allgather_unpack with two row shards emulated
    on one GPU: both shards' tagged words go into two exchange buffers, each
    unpack yields the unsharded layer's y bit for bit, over alternating buffer
    halves and ragged token counts.  The calls run in stream order (every
    word is written before the unpack that reads it starts), so no launch
    waits on a concurrent one."""
    import ctypes

    from littlebit_b200 import _lib as L
    from littlebit_b200 import ops, synthetic
    from littlebit_b200.sharded import RowShardedLinear

    K, N, r, G, kmax = 4096, 2048, 208, 2, 8
    g = torch.Generator().manual_seed(91)
    full = synthetic.to_packed_linear(K, N, synthetic.layer(K, N, [r, 96], g), DEV)
    shards = [RowShardedLinear(full, G, rank) for rank in range(G)]
    half = kmax * N
    xbufs = [torch.zeros(2 * half, dtype=torch.int64, device=DEV) for _ in range(G)]
    states = [torch.zeros(2, dtype=torch.int32, device=DEV) for _ in range(G)]
    peers = (ctypes.c_void_p * G)(*[b.data_ptr() for b in xbufs])
    arrs = [ops.projs_array([s.local]) for s in shards]
    wss = [torch.zeros(ops.linear_workspace_bytes([s.local], kmax), dtype=torch.uint8, device=DEV)
           for s in shards]
    lib = ops.lib()
    st = torch.cuda.current_stream().cuda_stream
    for k in (1, 3, 8, 1, 2):
        x = torch.randn(k, K, generator=g).cuda()
        for rank, s in enumerate(shards):
            a = L.LinearArgs()
            a.n_proj, a.n_tokens, a.x_dtype, a.y_dtype = 1, k, L.LBX_F32, L.LBX_F32
            a.epilogue, a.use_pdl, a.x = L.LBX_EPI_STORE, 1, x.data_ptr()
            L.check(lib.lbx_linear_allgather(arrs[rank], ctypes.byref(a), G, peers, half, s.lo, N,
                                             states[rank].data_ptr(), wss[rank].data_ptr(),
                                             wss[rank].numel(), st), "allgather")
        ys = [torch.empty(k, N, device=DEV) for _ in range(G)]
        for rank in range(G):
            L.check(lib.lbx_allgather_unpack(xbufs[rank].data_ptr(), half, k, N, N, ys[rank].data_ptr(),
                                             N, states[rank].data_ptr(), 1, st), "unpack")
        ref = ops.lb_linear(full, x)
        torch.cuda.synchronize()
        assert ops.device_error() == 0
        for rank in range(G):
            assert torch.equal(ys[rank], ref), (k, rank)
    assert [int(s[0]) for s in states] == [5, 5] and [int(s[1]) for s in states] == [0, 0]


def test_allgather_unpack_bounded_wait_reports_missing_shard():
    """The unpack kernel's wait is bounded: when one (emulated) shard never
    delivers its words, each unpack gives up after 1 s, records device error
    0x601, writes NaN for the missing columns and returns with the GPU context
    intact.  After the error word is cleared, the next call of both shards
    exchanges normally and matches the unsharded layer bit for bit.  Only the
    waiting kernel is launched; nothing the wait depends on is in flight."""
    import ctypes

    from littlebit_b200 import _lib as L
    from littlebit_b200 import ops, synthetic
    from littlebit_b200.sharded import RowShardedLinear

    K, N, r, G, k = 4096, 1024, 208, 2, 2
    g = torch.Generator().manual_seed(93)
    full = synthetic.to_packed_linear(K, N, synthetic.layer(K, N, [r], g), DEV)
    shards = [RowShardedLinear(full, G, rank) for rank in range(G)]
    half = k * N
    xbufs = [torch.zeros(2 * half, dtype=torch.int64, device=DEV) for _ in range(G)]
    states = [torch.zeros(2, dtype=torch.int32, device=DEV) for _ in range(G)]
    peers = (ctypes.c_void_p * G)(*[b.data_ptr() for b in xbufs])
    arrs = [ops.projs_array([s.local]) for s in shards]
    wss = [torch.zeros(ops.linear_workspace_bytes([s.local], k), dtype=torch.uint8, device=DEV) for s in shards]
    lib = ops.lib()
    st = torch.cuda.current_stream().cuda_stream

    def send(rank, x):
        a = L.LinearArgs()
        a.n_proj, a.n_tokens, a.x_dtype, a.y_dtype = 1, k, L.LBX_F32, L.LBX_F32
        a.epilogue, a.use_pdl, a.x = L.LBX_EPI_STORE, 0, x.data_ptr()
        L.check(lib.lbx_linear_allgather(arrs[rank], ctypes.byref(a), G, peers, half, shards[rank].lo, N,
                                         states[rank].data_ptr(), wss[rank].data_ptr(), wss[rank].numel(), st),
                "allgather")

    def unpack_all():
        ys = [torch.empty(k, N, device=DEV) for _ in range(G)]
        for rank in range(G):
            L.check(lib.lbx_allgather_unpack(xbufs[rank].data_ptr(), half, k, N, N, ys[rank].data_ptr(), N,
                                             states[rank].data_ptr(), 0, st), "unpack")
        return ys

    ops.clear_device_error()
    x = torch.randn(k, K, generator=g).cuda()
    ref = ops.lb_linear(full, x)
    send(0, x)  # shard 1 never delivers call 1
    torch.cuda.synchronize()
    import time

    t0 = time.perf_counter()
    ys = unpack_all()
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert ops.device_error() == 0x601
    assert 1.5 < waited < 30.0, waited  # two unpacks, each bounded at 1 s
    lo1 = shards[1].lo
    for y in ys:
        assert torch.equal(y[:, :lo1], ref[:, :lo1])  # shard 0's columns arrived
        assert torch.isnan(y[:, lo1:]).all()          # shard 1's are reported missing
    assert [int(s[0]) for s in states] == [1, 1] and [int(s[1]) for s in states] == [0, 0]
    # recovery: clear the error word; the next call of both shards is exact
    ops.clear_device_error()
    x = torch.randn(k, K, generator=g).cuda()
    for rank in range(G):
        send(rank, x)
    ys = unpack_all()
    ref = ops.lb_linear(full, x)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    for y in ys:
        assert torch.equal(y, ref)


def _run_both(ops, projs, x, out_shapes, dt=torch.float32, y_init=None, **kw):
    """The same call on the cluster executor and on the two stage grids."""
    from littlebit_b200 import _lib as L

    res = []
    for mode in (L.LBX_EXEC_CLUSTER, L.LBX_EXEC_KERNELS):
        outs = [torch.zeros(s, dtype=dt, device=DEV) for s in out_shapes]
        for o, i0 in zip(outs, y_init or []):
            o.copy_(i0)
        ops.linear_group(projs, x, outs, exec_mode=mode, **kw)
        res.append(outs)
    torch.cuda.synchronize()
    return res


@pytest.mark.parametrize("case", [
    ("c2", 4096, 4096, [208, 1840], (1, 2, 3, 4), torch.bfloat16, False, False),
    ("c1", 4096, 4096, [208], (1, 3), torch.float32, False, False),
    ("shared_bias", 1024, 512, [96, 96], (1, 3, 4), torch.float32, True, True),
    ("shared_big", 4096, 4096, [1840, 1840], (1, 2), torch.bfloat16, True, False),
    ("odd_rank", 256, 128, [40, 8], (1, 4), torch.float32, False, False),
    ("gate", 4096, 11008, [280], (1, 2), torch.float32, False, False),
    ("narrow_k", 2048, 1024, [136, 24], (1, 4), torch.bfloat16, False, True),
    ("tiny", 128, 16, [8], (1,), torch.float32, False, False),
])
def test_cluster_executor_matches_two_stage_bitwise(ops, case):
    """The split-rank cluster executor (one launch: each cluster's share of z in
    distributed shared memory, exact group sums combined by the last CTA of
    each output range) computes the same bits as the V-stage + U-stage grids:
    shared-V and independent residuals, bias, ranks that are not multiples of
    16 or 128, inputs narrower than 4096, k = 1..4, repeated calls."""
    name, in_f, out_f, ranks, ks, dt, shared, bias = case
    _, _, lay = _layer(ops, in_f, out_f, ranks, seed=sum(map(ord, name)) + 5, shared=shared, bias=bias)
    for rep in range(2):
        for k in ks:
            x = torch.randn(k, in_f, generator=_gen(k + 40 + rep)).to(dt).to(DEV)
            (yc,), (yk,) = _run_both(ops, [lay], x, [(k, out_f)], dt=dt)
            assert torch.equal(yc, yk), (name, k, float((yc.float() - yk.float()).abs().max()))


def test_cluster_executor_prologues_epilogues_groups(ops):
    """q/k/v-style groups with the RMSNorm prologue, and the SiLU-mul prologue
    with the residual-add epilogue: cluster executor == two stage grids."""
    from littlebit_b200 import _lib as L

    g = _gen(61)
    H, I = 1024, 1536
    layers = [_layer(ops, H, o, r, seed=70 + i)[2] for i, (o, r) in
              enumerate(((H, [64, 32]), (256, [48]), (256, [48, 48])))]
    w = (1 + 0.1 * torch.randn(H, generator=g)).abs().to(DEV)
    dn = _layer(ops, I, H, [80, 40], seed=80)[2]
    for k in (1, 3, 4):
        x = torch.randn(k, H, generator=g).to(DEV)
        yc, yk = _run_both(ops, layers, x, [(k, l.out_features) for l in layers],
                           prologue=L.LBX_PRO_RMSNORM, norm_w=w, eps=1e-6)
        for a, b in zip(yc, yk):
            assert torch.equal(a, b), k
        gt, up = torch.randn(k, I, generator=g).to(DEV), torch.randn(k, I, generator=g).to(DEV)
        res = torch.randn(k, H, generator=g).to(DEV)
        (ac,), (ak,) = _run_both(ops, [dn], gt, [(k, H)], prologue=L.LBX_PRO_SILU_MUL, x2=up,
                                 epilogue=L.LBX_EPI_ADD, y_init=[res])
        assert torch.equal(ac, ak), k


def test_cluster_executor_rejects_what_it_cannot_take(ops):
    """LBX_EXEC_CLUSTER refuses calls outside the executor (k > 4, K > 4096);
    LBX_EXEC_AUTO runs them."""
    from littlebit_b200 import _lib as L

    _, _, lay = _layer(ops, 8192, 512, [64], seed=91)
    x = torch.randn(1, 8192, generator=_gen(92)).to(DEV)
    y = torch.empty(1, 512, device=DEV)
    with pytest.raises(RuntimeError, match="unsupported"):
        ops.linear_group([lay], x, [y], exec_mode=L.LBX_EXEC_CLUSTER)
    ops.linear_group([lay], x, [y], exec_mode=L.LBX_EXEC_AUTO)
    _, _, lay2 = _layer(ops, 512, 256, [64], seed=93)
    x5 = torch.randn(5, 512, generator=_gen(94)).to(DEV)
    y5 = torch.empty(5, 256, device=DEV)
    with pytest.raises(RuntimeError, match="unsupported"):
        ops.linear_group([lay2], x5, [y5], exec_mode=L.LBX_EXEC_CLUSTER)
    torch.cuda.synchronize()


def test_two_tile_v_units_match_one_tile(ops):
    """A q/k/v call of the 7B shape (375 V tiles, more than two CTAs per SM hold)
    runs two 16-row tiles per V unit; each projection alone (125 tiles) runs one.
    Both give the same bits, for k = 1, 3, 5 and with the RMSNorm prologue."""
    from littlebit_b200 import _lib as L

    layers = [_layer(ops, 4096, 4096, [184, 1816], seed=300 + i)[2] for i in range(3)]
    w = (1 + 0.1 * torch.randn(4096, generator=_gen(301))).abs().to(DEV)
    for k in (1, 3, 5):
        x = torch.randn(k, 4096, generator=_gen(310 + k)).to(DEV)
        grouped = [torch.empty(k, 4096, device=DEV) for _ in layers]
        ops.linear_group(layers, x, grouped, prologue=L.LBX_PRO_RMSNORM, norm_w=w,
                         exec_mode=L.LBX_EXEC_KERNELS)
        for lay, yg in zip(layers, grouped):
            y1 = torch.empty(k, 4096, device=DEV)
            ops.linear_group([lay], x, [y1], prologue=L.LBX_PRO_RMSNORM, norm_w=w,
                             exec_mode=L.LBX_EXEC_KERNELS)
            torch.cuda.synchronize()
            assert torch.equal(yg, y1), k


def test_silu_epilogue_then_mul_prologue_equals_silu_mul_prologue(ops):
    """gate/up with LBX_EPI_SILU0 (gate stored as silu(gate)) followed by down
    with LBX_PRO_MUL computes the same bits as gate/up stored plainly followed
    by down with LBX_PRO_SILU_MUL (fp32), on both executors."""
    from littlebit_b200 import _lib as L

    H, I = 1024, 2816
    gate, up = (_layer(ops, H, I, [96, 80], seed=400 + i)[2] for i in range(2))
    down = _layer(ops, I, H, [96, 80], seed=402)[2]
    w = (1 + 0.1 * torch.randn(H, generator=_gen(403))).abs().to(DEV)
    for k in (1, 4, 7):
        x = torch.randn(k, H, generator=_gen(410 + k)).to(DEV)
        res = torch.randn(k, H, generator=_gen(420 + k)).to(DEV)
        outs = {}
        for fused in (False, True):
            for mode in (L.LBX_EXEC_KERNELS, L.LBX_EXEC_CLUSTER):
                if mode == L.LBX_EXEC_CLUSTER and k > 4:
                    continue
                g_ = torch.empty(k, I, device=DEV)
                u_ = torch.empty(k, I, device=DEV)
                ops.linear_group([gate, up], x, [g_, u_], prologue=L.LBX_PRO_RMSNORM, norm_w=w,
                                 epilogue=L.LBX_EPI_SILU0 if fused else L.LBX_EPI_STORE, exec_mode=mode)
                y = res.clone()
                ops.linear_group([down], g_, [y], prologue=L.LBX_PRO_MUL if fused else L.LBX_PRO_SILU_MUL,
                                 x2=u_, epilogue=L.LBX_EPI_ADD, exec_mode=L.LBX_EXEC_KERNELS)
                outs[(fused, mode)] = y
        torch.cuda.synchronize()
        ref = outs[(False, L.LBX_EXEC_KERNELS)]
        for key, y in outs.items():
            assert torch.equal(y, ref), (k, key)


def test_large_rank_splits_token_batches_bitwise(ops):
    """A rank where 16 tokens' digits do not fit in shared memory (the 70B
    0.9-bit residual size): the call runs in smaller token batches and every
    token keeps the bits of a one-token call."""
    _, _, lay = _layer(ops, 8192, 2048, [5736], seed=500)
    x = torch.randn(16, 8192, generator=_gen(501)).to(DEV)
    y = ops.lb_linear(lay, x)
    for i in (0, 7, 8, 15):
        assert torch.equal(ops.lb_linear(lay, x[i:i + 1])[0], y[i]), i
    torch.cuda.synchronize()


@pytest.mark.parametrize("k", [1, 5])
def test_pass_split_v_stage_matches_one_cta_passes(ops, k):
    """Inputs wider than one 4096-column staging pass (8192 and 11008 columns) run
    the pass-split V-stage: a cluster of one CTA per pass, rank 0 adding the
    partial sums in the one-CTA order.  The persistent program runs every unit's
    passes in one CTA; both give the same bits."""
    from littlebit_b200 import synthetic

    g = _gen(800 + k)
    # draft-sized single branches take the pass-split form (at most two CTAs per
    # SM for the whole split grid); the two-branch targets keep one CTA per unit
    for K, N, ranks in ((8192, 1024, [392]), (11008, 4096, [280]), (8192, 1024, [392, 3664]),
                        (11008, 4096, [280, 2664])):
        lay = synthetic.to_packed_linear(K, N, synthetic.layer(K, N, ranks, g), DEV)
        x = torch.randn(k, K, generator=g).to(DEV)
        y = torch.empty(k, N, device=DEV)
        ops.linear_group([lay], x, [y], exec_mode=ops.L.LBX_EXEC_KERNELS)
        acts = [x.clone(), torch.empty(k, N, device=DEV)]
        ops.linear_chain([lay], acts)
        assert torch.equal(y.view(torch.int32), acts[1].view(torch.int32)), (K, N)


@pytest.mark.parametrize("k", [1, 5])
@pytest.mark.parametrize("prologue", ["rmsnorm", "silu_mul", "mul"])
def test_pass_split_v_stage_prologues_bitwise(ops, k, prologue):
    """The pass-split V-stage with each fused prologue: RMSNorm (rank 0 adds the
    other ranks' sums of squares over distributed shared memory), SiLU-mul and
    mul (the draft down projection).  Bit-identical to the same call with every
    V unit's passes in one CTA."""
    from littlebit_b200 import synthetic

    L_ = ops.L
    pro = {"rmsnorm": L_.LBX_PRO_RMSNORM, "silu_mul": L_.LBX_PRO_SILU_MUL, "mul": L_.LBX_PRO_MUL}[prologue]
    g = _gen(830 + k)
    for K, N, ranks in ((8192, 1024, [392]), (11008, 4096, [280]), (11008, 4096, [280, 280])):
        lay = synthetic.to_packed_linear(K, N, synthetic.layer(K, N, ranks, g), DEV)
        x = torch.randn(k, K, generator=g).to(DEV)
        x2 = torch.randn(k, K, generator=g).to(DEV)
        w = (1 + 0.1 * torch.randn(K, generator=g)).abs().to(DEV)
        kw = dict(prologue=pro)
        if pro == L_.LBX_PRO_RMSNORM:
            kw["norm_w"] = w
        else:
            kw["x2"] = x2
        ys = []
        for mode in (L_.LBX_EXEC_KERNELS, L_.LBX_EXEC_KERNELS_ONE_CTA_V):
            y = torch.empty(k, N, device=DEV)
            ops.linear_group([lay], x, [y], exec_mode=mode, **kw)
            ys.append(y)
        torch.cuda.synchronize()
        assert torch.isfinite(ys[0]).all()
        assert torch.equal(ys[0].view(torch.int32), ys[1].view(torch.int32)), (K, N, prologue)
