"""The allocation-free linear entry point (lbx_linear_noalloc).

It exists for callers that cannot give the library device memory (a host
application whose own allocator owns every device allocation, or a service
that sets up all device memory at start-up and may not allocate later).  It keeps its scratch in a
fixed 1 MiB device array instead of a caller workspace.  Its results must
match the allocating entry point (lbx_linear_verify with a caller workspace)
bit for bit -- both run the same kernels, so any difference would be stale
or corrupted scratch -- on consecutive calls that reuse the shared array, and
oversized calls must be refused before any GPU work.

Collected last (file name) so a failure here does not hide the other tests.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _args(L, x, y):
    a = L.LinearArgs()
    a.n_proj = 1
    a.n_tokens = x.shape[0]
    a.x_dtype = L.LBX_BF16
    a.y_dtype = L.LBX_F32
    a.prologue = L.LBX_PRO_NONE
    a.epilogue = L.LBX_EPI_STORE
    a.eps = 1e-6
    a.use_pdl = 0
    a.x = x.data_ptr()
    a.y[0] = y.data_ptr()
    a.y_ld[0] = y.stride(0)
    return a


def test_noalloc_matches_allocating_entry_point():
    from littlebit_b200 import _lib as L
    from littlebit_b200 import ops, synthetic as syn

    lib = L.load()
    g = torch.Generator().manual_seed(91)
    lay = syn.to_packed_linear(4096, 4096, syn.layer(4096, 4096, [208, 1840], g), "cuda")
    arr = ops.projs_array([lay])
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for k in (5, 1):  # two calls in a row on the shared array, different batch sizes
        x = torch.randn(k, 4096, generator=g).bfloat16().cuda()
        y_ref = torch.empty(k, 4096, device="cuda")
        ws = torch.zeros(ops.linear_workspace_bytes([lay], k), dtype=torch.uint8, device="cuda")
        L.check(lib.lbx_linear_verify(arr, ctypes.byref(_args(L, x, y_ref)), ws.data_ptr(),
                                      ws.numel(), stream), "lbx_linear_verify")
        y = torch.full_like(y_ref, float("nan"))
        L.check(lib.lbx_linear_noalloc(arr, ctypes.byref(_args(L, x, y)), stream),
                "lbx_linear_noalloc")
        torch.cuda.synchronize()
        assert torch.equal(y.view(torch.int32), y_ref.view(torch.int32)), k


def test_noalloc_rejects_oversized_calls_without_gpu_work():
    from littlebit_b200 import _lib as L

    lib = L.load()
    cap = lib.lbx_linear_noalloc_max_bytes()
    assert cap == 1 << 20
    # 16 tokens x 3 projections x rank 8192 needs ~1.5 MiB of scratch: refused on the
    # host before anything is launched (the dummy pointers are never dereferenced)
    arr = (L.Proj * 3)()
    for pr in arr:
        pr.in_features, pr.out_features, pr.n_branches = 4096, 4096, 1
        b = pr.br[0]
        b.v_sign = b.v2 = b.mid = b.u_sign = b.u1 = 256
        b.rank = 8192
    a = L.LinearArgs()
    a.n_proj, a.n_tokens = 3, 16
    rc = lib.lbx_linear_noalloc(arr, ctypes.byref(a), None)
    assert rc == L.LBX_EUNSUPPORTED
    assert "fixed buffer holds" in L.last_error()
