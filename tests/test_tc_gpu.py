"""The tensor-core executor (LBX_EXEC_TC: tcgen05.mma kind::i8 with TMEM
accumulators, up to 64 tokens per launch).

Every output must equal, bit for bit, the two stage grids (LBX_EXEC_NO_TC,
warp-level mma.sync over batches of at most 16 tokens), which the linear tests
hold to the float64 oracle: the executor changes how the exact integer sums are
formed, never a rounding.  Cases cover every prologue and epilogue, the
shared-factor residual, bias, bf16 and fp32 activations, ranks that are not
multiples of 32 or 128, an input width that ends in half a 256-column block,
and token counts that pad each tensor-core batch (8, 16, 32, 64) or span
several of them."""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _proj(K, N, ranks, g, shared=False, bias=False):
    from littlebit_b200 import synthetic

    brs = synthetic.layer(K, N, ranks, g, shared_residual=shared)
    b = (0.1 * torch.randn(N, generator=g)) if bias else None
    return synthetic.to_packed_linear(K, N, brs, DEV, bias=b)


def _run(projs, x, exec_mode, ydt=torch.float32, init=None, **kw):
    from littlebit_b200 import ops

    k = x.shape[0]
    if init is None:
        outs = [torch.full((k, p.out_features), float("nan"), dtype=ydt, device=DEV) for p in projs]
    else:
        outs = [t.clone() for t in init]
    ws = torch.zeros(ops.linear_workspace_bytes(projs, max(k, 32)), dtype=torch.uint8, device=DEV)
    ops.linear_group(projs, x, outs, ws=ws, exec_mode=exec_mode, **kw)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    return outs


def _same(a, b):
    ia = a.view(torch.int16) if a.dtype == torch.bfloat16 else a.view(torch.int32)
    ib = b.view(torch.int16) if b.dtype == torch.bfloat16 else b.view(torch.int32)
    return torch.equal(ia, ib)


def _check(projs, x, **kw):
    from littlebit_b200 import _lib as L

    ref = _run(projs, x, L.LBX_EXEC_NO_TC, **kw)
    got = _run(projs, x, L.LBX_EXEC_TC, **kw)
    for i, (r, o) in enumerate(zip(ref, got)):
        assert torch.isfinite(r.float()).all(), i
        assert _same(o, r), (i, (o.float() - r.float()).abs().max().item())
    return ref


@pytest.mark.parametrize("k", [1, 5, 16, 33, 64, 100])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_tc_c2_bitwise(k, dtype):
    """C2 layer (4096 -> 4096, ranks 208 + 1840 independent residual)."""
    g = torch.Generator().manual_seed(100 + k)
    p = _proj(4096, 4096, [208, 1840], g)
    x = torch.randn(k, 4096, generator=g).to(DEV, dtype)
    _check([p], x, ydt=dtype)


@pytest.mark.parametrize("k", [24, 64])
def test_tc_gate_up_rmsnorm_silu_bitwise(k):
    """A 70B-width gate/up group: 8192 -> 2 x 14336, ranks 616 + 5736, RMSNorm
    prologue, SiLU on projection 0 (two projections sharing one x staging)."""
    g = torch.Generator().manual_seed(200 + k)
    gate = _proj(8192, 14336, [616, 5736], g)
    up = _proj(8192, 14336, [616, 5736], g)
    x = torch.randn(k, 8192, generator=g).to(DEV)
    w = (1.0 + 0.1 * torch.randn(8192, generator=g)).to(DEV)
    from littlebit_b200 import _lib as L

    _check([gate, up], x, prologue=L.LBX_PRO_RMSNORM, norm_w=w, epilogue=L.LBX_EPI_SILU0)


@pytest.mark.parametrize("pro", ["silu_mul", "mul"])
def test_tc_down_prologues_bitwise(pro):
    """The down projection's input prologues (11008 columns, 43 blocks: the
    last 16-block slots hold two passes, the rest three)."""
    from littlebit_b200 import _lib as L

    g = torch.Generator().manual_seed(300)
    p = _proj(11008, 4096, [280, 96], g)
    x = torch.randn(48, 11008, generator=g).to(DEV, torch.bfloat16)
    x2 = torch.randn(48, 11008, generator=g).to(DEV, torch.bfloat16)
    _check([p], x, ydt=torch.bfloat16, x2=x2,
           prologue=L.LBX_PRO_SILU_MUL if pro == "silu_mul" else L.LBX_PRO_MUL)


def test_tc_shared_residual_bias_qkv_bitwise():
    """Three projections sharing x (q/k/v-like widths), the shared-factor
    residual (one V feeds U and U_R), bias, RMSNorm, bf16 output."""
    from littlebit_b200 import _lib as L

    g = torch.Generator().manual_seed(400)
    q = _proj(4096, 4096, [208, 208], g, shared=True, bias=True)
    kp = _proj(4096, 1024, [120, 40], g, bias=True)
    v = _proj(4096, 1024, [64], g)
    x = torch.randn(40, 4096, generator=g).to(DEV, torch.bfloat16)
    w = (1.0 + 0.1 * torch.randn(4096, generator=g)).to(DEV)
    _check([q, kp, v], x, ydt=torch.bfloat16, prologue=L.LBX_PRO_RMSNORM, norm_w=w)


def test_tc_half_block_width_and_add_epilogue():
    """in_features 4224 (the last 256-column block is half empty), odd ranks,
    out_features not a multiple of 128, the fp32 residual-add epilogue."""
    from littlebit_b200 import _lib as L

    g = torch.Generator().manual_seed(500)
    p = _proj(4224, 1040, [200, 56], g)
    x = torch.randn(20, 4224, generator=g).to(DEV)
    y0 = [torch.randn(20, 1040, generator=g).to(DEV)]
    _check([p], x, init=y0, epilogue=L.LBX_EPI_ADD)


def test_tc_auto_selects_and_matches():
    """AUTO at 64 tokens (the tensor-core executor when the workspace holds a
    batch) gives the stage grids' bits; so does AUTO with a workspace sized
    for 16 tokens (the stage grids)."""
    from littlebit_b200 import _lib as L
    from littlebit_b200 import ops

    g = torch.Generator().manual_seed(600)
    p = _proj(4096, 4096, [208, 1840], g)
    x = torch.randn(64, 4096, generator=g).to(DEV, torch.bfloat16)
    ref = _run([p], x, L.LBX_EXEC_NO_TC, ydt=torch.bfloat16)[0]
    y = torch.empty_like(ref)
    ops.linear_group([p], x, [y], exec_mode=L.LBX_EXEC_AUTO)
    small = torch.zeros(ops.linear_workspace_bytes([p], 16), dtype=torch.uint8, device=DEV)
    y2 = torch.empty_like(ref)
    ops.linear_group([p], x, [y2], ws=small, exec_mode=L.LBX_EXEC_AUTO)
    torch.cuda.synchronize()
    assert _same(y, ref) and _same(y2, ref)


def test_tc_rejects_small_workspace():
    from littlebit_b200 import _lib as L
    from littlebit_b200 import ops

    g = torch.Generator().manual_seed(700)
    p = _proj(4096, 4096, [208], g)
    x = torch.randn(8, 4096, generator=g).to(DEV)
    y = torch.empty(8, 4096, device=DEV)
    small = torch.zeros(256, dtype=torch.uint8, device=DEV)
    with pytest.raises(RuntimeError, match="tensor-core"):
        ops.linear_group([p], x, [y], ws=small, exec_mode=L.LBX_EXEC_TC)
