"""The fused chain executor (lbx_chain_fused): layer i's U-stage and layer
i+1's V-stage partial sums in one launch.  Every activation of the chain must
equal, bit for bit, the layer-by-layer result of the two stage grids
(lbx_linear_verify with LBX_EXEC_KERNELS), which the linear tests hold to the
float64 oracle."""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _chain(dims, ranks, shared=False, bias=False, seed=0):
    from littlebit_b200 import synthetic

    g = torch.Generator().manual_seed(seed)
    layers = []
    for i in range(len(dims) - 1):
        brs = synthetic.layer(dims[i], dims[i + 1], ranks, g, shared_residual=shared)
        b = (0.1 * torch.randn(dims[i + 1], generator=g)) if bias else None
        layers.append(synthetic.to_packed_linear(dims[i], dims[i + 1], brs, DEV, bias=b))
    return layers, g


def _layerwise(ops, layers, x):
    from littlebit_b200 import _lib as L

    outs = [x]
    for lay in layers:
        y = torch.empty(x.shape[0], lay.out_features, dtype=x.dtype, device=DEV)
        ops.linear_group([lay], outs[-1], [y], exec_mode=L.LBX_EXEC_KERNELS)
        outs.append(y)
    return outs


@pytest.mark.parametrize("k", [1, 2, 4, 5, 8])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_fused_chain_c2_bitwise(k, dtype):
    """C2 layers (4096 -> 4096, draft rank 208 + independent residual rank 1840);
    5 and 8 tokens run as two concurrent sub-chains."""
    from littlebit_b200 import ops

    layers, g = _chain([4096] * 5, [208, 1840], seed=10 + k)
    fc = ops.FusedChain(layers)
    x = torch.randn(k, 4096, generator=g).to(DEV, dtype)
    ref = _layerwise(ops, layers, x)
    acts = [x] + [torch.full_like(r, float("nan")) for r in ref[1:]]
    fc.run(acts)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    for i in range(1, len(acts)):
        assert torch.isfinite(acts[i].float()).all(), i
        assert torch.equal(acts[i].view(torch.int16 if dtype == torch.bfloat16 else torch.int32),
                           ref[i].view(torch.int16 if dtype == torch.bfloat16 else torch.int32)), (k, i)


@pytest.mark.parametrize("k", [1, 3])
def test_fused_chain_shared_factor_bias_and_widths_bitwise(k):
    """The config-4 shared-factor residual (U_R on the draft's V-stage) with a
    bias, through widths 4096 -> 8192 -> 1024 -> 4096 (a two-pass input, and
    blocks fewer than one pass), and a single-branch layer."""
    from littlebit_b200 import ops

    layers, g = _chain([4096, 8192, 1024, 4096], [208, 208], shared=True, bias=True, seed=40 + k)
    single, _ = _chain([4096, 4096], [392], seed=50 + k)
    layers = layers + single
    fc = ops.FusedChain(layers)
    x = torch.randn(k, 4096, generator=g).to(DEV)
    ref = _layerwise(ops, layers, x)
    acts = [x] + [torch.empty_like(r) for r in ref[1:]]
    fc.run(acts)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    for i in range(1, len(acts)):
        assert torch.equal(acts[i].view(torch.int32), ref[i].view(torch.int32)), (k, i)


def test_fused_chain_split_calls_in_a_graph():
    """A 6-token call (two sub-chains on two streams) captured in a CUDA graph
    and replayed gives the layer-by-layer bits every time."""
    from littlebit_b200 import ops

    layers, g = _chain([4096] * 4, [208, 1840], seed=80)
    fc = ops.FusedChain(layers)
    x = torch.randn(6, 4096, generator=g).to(DEV, torch.bfloat16)
    ref = _layerwise(ops, layers, x)
    acts = [x.clone()] + [torch.empty_like(r) for r in ref[1:]]
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        fc.run(acts, stream=stream)  # (workspace allocated outside the capture)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        fc.run(acts, stream=stream)
    for _ in range(3):
        for a in acts[1:]:
            a.fill_(float("nan"))
        graph.replay()
        torch.cuda.synchronize()
        assert ops.device_error() == 0
        for i in range(1, len(acts)):
            assert torch.equal(acts[i].view(torch.int16), ref[i].view(torch.int16)), i


def test_fused_chain_repeated_calls_and_single_layer():
    """Back-to-back calls reuse the partial-sum workspace; a one-layer chain is
    the head launch plus one layer launch."""
    from littlebit_b200 import ops

    layers, g = _chain([4096, 4096], [208, 1840], seed=60)
    fc = ops.FusedChain(layers)
    for it in range(3):
        x = torch.randn(2, 4096, generator=g).to(DEV, torch.bfloat16)
        ref = _layerwise(ops, layers, x)
        acts = [x, torch.empty_like(ref[1])]
        fc.run(acts)
        torch.cuda.synchronize()
        assert torch.equal(acts[1].view(torch.int16), ref[1].view(torch.int16)), it


@pytest.mark.parametrize("k", [1, 5])
def test_fused_chain_cached_graph_replays_with_new_contents(k):
    """Outside stream capture, a call with the same layers, buffers and token
    count as an earlier one replays the library's cached graph of that call.
    The graph reads the buffers through their pointers, so new input contents
    in the same buffers must give the layer-by-layer bits on every call, and a
    new output buffer (a new graph) must too."""
    from littlebit_b200 import ops

    layers, g = _chain([4096, 4096, 4096], [208, 1840], seed=90 + k)
    fc = ops.FusedChain(layers)
    x = torch.empty(k, 4096, dtype=torch.bfloat16, device=DEV)
    acts = [x, torch.empty_like(x), torch.empty_like(x)]
    for it in range(4):
        if it == 3:
            acts[2] = torch.empty_like(x)  # another output buffer: another graph
        x.copy_(torch.randn(k, 4096, generator=g).to(DEV, torch.bfloat16))
        fc.run(acts)
        torch.cuda.synchronize()
        ref = _layerwise(ops, layers, x)
        assert ops.device_error() == 0
        for i in (1, 2):
            assert torch.equal(acts[i].view(torch.int16), ref[i].view(torch.int16)), (it, i)


def test_fused_chain_rejects_unsupported():
    from littlebit_b200 import ops

    layers, _ = _chain([4096, 4096], [208], seed=70)
    fc = ops.FusedChain(layers)
    x = torch.zeros(9, 4096, device=DEV)
    with pytest.raises(RuntimeError, match="tokens"):
        fc.run([x, torch.empty_like(x)])
    odd, _ = _chain([4096, 4112], [208], seed=71)   # out_features not a multiple of 256
    wide, _ = _chain([11008, 4096], [280], seed=72)  # in_features above 8192
    for bad in (odd, wide):
        with pytest.raises(RuntimeError, match="fused chain"):
            ops.FusedChain(bad)
