"""Decode / verify attention (lbx_attn_decode) on a grouped-query shape against
an fp64 restatement: 16 query heads over 2 kv heads (8 rows of one kv head per
token), head_dim 128, RoPE from the (cos, sin) table, a bf16 cache with a long
prefix (24 key chunks: the merge stages its chunk weights in shared memory,
and the query rows of a kv head are split over several CTAs).  A token scored
inside a causal verify batch gives the same bits as the same token decoded
alone after the batch has written the cache."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

H, KVH, D, THETA = 16, 2, 128, 10000.0


def _rot(x, cs):
    """rotate_half RoPE of x [..., D] with the kernel's float (cos, sin) pairs cs [D/2, 2]."""
    h = D // 2
    c, s = cs[:, 0], cs[:, 1]
    x1, x2 = x[..., :h], x[..., h:]
    return np.concatenate([x1 * c - x2 * s, x2 * c + x1 * s], axis=-1)


def _bf16(a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).bfloat16().double().numpy()


@pytest.mark.parametrize("prefix,n", [(1500, 1), (1500, 5), (100, 5)])
def test_gqa_attention_long_prefix_matches_fp64(prefix, n):
    from littlebit_b200 import ops

    g = torch.Generator().manual_seed(prefix + n)
    S = 2048
    kc = torch.randn(KVH, S, D, generator=g).bfloat16()
    vc = torch.randn(KVH, S, D, generator=g).bfloat16()
    q = torch.randn(n, H * D, generator=g)
    kn, vn = torch.randn(n, KVH * D, generator=g), torch.randn(n, KVH * D, generator=g)
    dev = torch.device("cuda")
    kd, vd = kc.to(dev), vc.to(dev)
    pos = torch.arange(prefix, prefix + n, dtype=torch.int32, device=dev)
    cs = ops.rope_table(pos, D, THETA)
    out = ops.attention(q.to(dev), kn.to(dev), vn.to(dev), pos, kd, vd, prefix, H, KVH, D, D ** -0.5, THETA,
                        rope_cs=cs).cpu().numpy().reshape(n, H, D)
    csn = cs.cpu().double().numpy().reshape(n, D // 2, 2)
    K = kc.double().numpy().copy()
    V = vc.double().numpy().copy()
    # the kernel wrote the new tokens' rotated keys and values, rounded to bf16
    # (the rotation is fp32 in the kernel: within one bf16 step of the fp64 one)
    kw = kd[:, prefix:prefix + n].cpu().double().numpy()
    vw = vd[:, prefix:prefix + n].cpu().double().numpy()
    for i in range(n):
        kr = _rot(kn[i].double().numpy().reshape(KVH, D), csn[i])
        np.testing.assert_allclose(kw[:, i], kr, rtol=2 ** -7, atol=1e-6)
        np.testing.assert_array_equal(vw[:, i], _bf16(vn[i].double().numpy().reshape(KVH, D)))
    K[:, prefix:prefix + n] = kw
    V[:, prefix:prefix + n] = vw
    ref = np.zeros((n, H, D))
    for i in range(n):
        qq = _rot(q[i].double().numpy().reshape(H, D), csn[i])
        for hq in range(H):
            kh = hq // (H // KVH)
            s = K[kh, :prefix + i + 1] @ qq[hq] * D ** -0.5
            p = np.exp(s - s.max())
            ref[i, hq] = (p / p.sum()) @ V[kh, :prefix + i + 1]
    np.testing.assert_allclose(out, ref, rtol=0, atol=1e-4 * np.abs(ref).max())
    # each verify row equals a decode of that token alone over the cache the batch wrote
    for i in range(n):
        one = ops.attention(q[i:i + 1].to(dev), kn[i:i + 1].to(dev), vn[i:i + 1].to(dev), pos[i:i + 1], kd, vd,
                            prefix + i, H, KVH, D, D ** -0.5, THETA, rope_cs=cs[i:i + 1])
        assert torch.equal(one.cpu().view(torch.int32), torch.from_numpy(out[i].reshape(1, -1).astype(np.float32)).view(torch.int32)), i
