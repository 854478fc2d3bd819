"""torch.ops.littlebit_cuda_ops on the GPU against the oracle, with the
reference CPU runtime's semantics: single-branch projections, no rotary
embedding (theta = 0), flat 37-tensors-per-layer argument lists
(cpu_draft_model.py:229-264) and a separate k, v cache per layer."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from test_decoder_gpu import TINY, TINY_RANKS  # noqa: E402


def _flat(st, shape, dev):
    from littlebit_b200.model import PROJ_NAMES, proj_prefix

    tens, dims = [], []
    for i in range(shape.num_hidden_layers):
        tens += [st[f"model.layers.{i}.input_layernorm.weight"].to(dev),
                 st[f"model.layers.{i}.post_attention_layernorm.weight"].to(dev)]
        for nm in PROJ_NAMES:
            p = proj_prefix(i, nm)
            r, in_f = (int(v) for v in st[f"{p}.v_sign_rt_shape"])
            out_f = int(st[f"{p}.u_sign_rt_shape"][0])
            tens += [st[f"{p}.v2"].reshape(-1).to(dev), st[f"{p}.v_sign_rt"].to(dev),
                     st[f"{p}.mid"].reshape(-1).to(dev), st[f"{p}.u_sign_rt"].to(dev),
                     st[f"{p}.u1"].reshape(-1).to(dev)]
            dims += [in_f, r, r, out_f]
    return tens, dims


def test_full_forward_family_matches_oracle():
    import littlebit_b200.torch_ops  # noqa: F401  (registers the namespace)
    from littlebit_b200.model import DecoderShape, synthetic_runtime_state
    from oracle import decoder as od

    shape = DecoderShape(**TINY)
    st = synthetic_runtime_state(shape, {k: v[:1] for k, v in TINY_RANKS.items()}, seed=21, unit_gain=True)
    dev = torch.device("cuda")
    tens, dims = _flat(st, shape, dev)
    kvh, d, S = shape.num_key_value_heads, shape.head_dim, 64
    kv = [torch.zeros(kvh, S, d, dtype=torch.bfloat16, device=dev) for _ in range(2 * shape.num_hidden_layers)]
    emb = st["model.embed_tokens.weight"].float().to(dev)  # fp32 like the reference (bf16-valued)
    fn = st["model.norm.weight"].to(dev)
    head = st["lm_head.weight"].to(dev)
    o = od.from_runtime_state(st, shape.num_hidden_layers, shape.hidden_size, shape.intermediate_size,
                              shape.num_attention_heads, kvh, shape.vocab_size, shape.rms_norm_eps,
                              rope_theta=0.0, max_seq=S)
    scale = 1.0 / d ** 0.5
    common = dict(num_layers=shape.num_hidden_layers, hidden_size=shape.hidden_size, num_kv_heads=kvh,
                  kv_repeat=shape.num_attention_heads // kvh, head_dim=d, max_seq_len=S, attn_scale=scale,
                  rms_eps=shape.rms_norm_eps)
    ops_ = torch.ops.littlebit_cuda_ops
    ids = torch.randint(0, shape.vocab_size, (14,), generator=torch.Generator().manual_seed(4))
    h = ops_.full_forward_batch(ids[:10].to(dev), emb, fn, tens, kv, dims, start_position=0, **common)
    ref = o.final_hidden(o.forward(ids[:10].tolist(), 0))
    np.testing.assert_allclose(h.cpu().numpy(), ref, rtol=0, atol=5e-3 * np.abs(ref).max())
    for t in range(10, 13):
        h1 = ops_.full_forward(int(ids[t]), emb, fn, tens, kv, dims, position=t, **common)
        ref = o.final_hidden(o.forward([int(ids[t])], t))
        np.testing.assert_allclose(h1.cpu().numpy(), ref, rtol=0, atol=5e-3 * np.abs(ref).max())
    tok = ops_.generate_token(int(ids[13]), emb, fn, tens, kv, dims, head, shape.vocab_size, position=13, **common)
    lg = o.logits(o.forward([int(ids[13])], 13))[0]
    top2 = np.sort(lg)[-2:]
    if top2[1] - top2[0] > 1e-2 * np.abs(lg).max():
        assert tok == int(lg.argmax())


def test_fused_attention_matches_oracle_without_rope():
    import littlebit_b200.torch_ops  # noqa: F401

    g = torch.Generator().manual_seed(5)
    kvh, rep, d, S, pos = 2, 4, 64, 32, 9
    dev = torch.device("cuda")
    kc = torch.randn(kvh, S, d, generator=g).bfloat16()
    vc = torch.randn(kvh, S, d, generator=g).bfloat16()
    q = torch.randn(1, kvh * rep * d, generator=g)
    kn, vn = torch.randn(1, kvh * d, generator=g), torch.randn(1, kvh * d, generator=g)
    kd, vd = kc.to(dev), vc.to(dev)
    out = torch.ops.littlebit_cuda_ops.fused_attention(q.to(dev), kd, vd, kn.to(dev), vn.to(dev), pos, kvh,
                                                       rep, d, 0.125)
    K = kc.double().numpy().copy()
    V = vc.double().numpy().copy()
    K[:, pos] = kn.bfloat16().double().numpy().reshape(kvh, d)
    V[:, pos] = vn.bfloat16().double().numpy().reshape(kvh, d)
    qq = q.double().numpy().reshape(kvh * rep, d)
    ref = np.zeros((kvh * rep, d))
    for h in range(kvh * rep):
        s = K[h // rep, :pos + 1] @ qq[h] * 0.125
        p = np.exp(s - s.max())
        ref[h] = (p / p.sum()) @ V[h // rep, :pos + 1]
    np.testing.assert_allclose(out.cpu().numpy().reshape(kvh * rep, d), ref, rtol=0, atol=2e-5 * np.abs(ref).max() + 1e-6)
    assert torch.equal(kd[:, pos].cpu(), kn.bfloat16().reshape(kvh, d))
