"""The native decoder step (lbx_forward) vs the CPU oracle decoder.

Same seeded runtime-layout weights on both sides; the oracle keeps keys and
values rounded to bf16 like the B200 cache.  Bars: logits within 1e-2 of the
largest |logit| (basis in ``_close``); greedy tokens equal wherever the
oracle's top-2 margin exceeds that tolerance; a token's logits bit-identical
whether prefilled alone or in a batch (the property that makes greedy
speculative decoding token-identical).
"""
import numpy as np
import pytest
import torch

from oracle import decoder as od

pytestmark = pytest.mark.gpu

TINY = dict(num_hidden_layers=2, hidden_size=256, intermediate_size=512, num_attention_heads=4,
            num_key_value_heads=2, vocab_size=512)
TINY_RANKS = {"q_proj": [64, 32], "k_proj": [32, 16], "v_proj": [32, 16], "o_proj": [64, 32],
              "gate_proj": [96, 40], "up_proj": [96, 40], "down_proj": [96, 40]}


def oracle_from_state(shape, st, max_seq, include_residual=True):
    return od.from_runtime_state(st, shape.num_hidden_layers, shape.hidden_size, shape.intermediate_size,
                                 shape.num_attention_heads, shape.num_key_value_heads, shape.vocab_size,
                                 shape.rms_norm_eps, shape.rope_theta, max_seq, include_residual)


@pytest.fixture(scope="module")
def tiny():
    from littlebit_b200.model import DecoderShape, LittleBitDecoder, synthetic_runtime_state

    shape = DecoderShape(**TINY)
    # near-unit-gain projections: activations stay in the range of trained
    # checkpoints, so a bf16 ulp of a cached key cannot flip a one-hot softmax
    st = synthetic_runtime_state(shape, TINY_RANKS, seed=5, unit_gain=True)
    return shape, st


def _close(lg, ref):
    """End-to-end logits against the float64 oracle.  Each LittleBit projection is
    held to rtol 1e-3 by the linear tests (it measures 3e-5..7e-5 of its output
    maximum).  Through two layers, attention and the 256-wide lm_head, per-element
    noise of 4e-5 of each projection's maximum moves these logits by up to
    3.7e-3 of the largest logit (oracle-only simulation, three seeds), so the
    bound is 1e-2 of the largest logit, plus argmax agreement wherever the
    oracle's top-2 gap is wider than twice that."""
    lg = np.asarray(lg, np.float64)
    tol = 1e-2 * np.abs(ref).max()
    np.testing.assert_allclose(lg, ref, rtol=0, atol=tol)
    top2 = np.sort(ref, axis=-1)[:, -2:]
    sure = (top2[:, 1] - top2[:, 0]) > 2 * tol
    assert (lg.argmax(-1)[sure] == ref.argmax(-1)[sure]).all()


@pytest.mark.parametrize("shared", [False, True])
def test_decoder_matches_oracle(tiny, shared):
    from littlebit_b200.model import DecoderShape, LittleBitDecoder, synthetic_runtime_state

    shape, st = tiny
    if shared:
        st = synthetic_runtime_state(shape, {k: [v[0], v[0]] for k, v in TINY_RANKS.items()}, seed=6,
                                     shared_residual=True, unit_gain=True)
    m = LittleBitDecoder(shape, st, max_seq=256)
    o = oracle_from_state(shape, st, 256)
    ids = torch.randint(0, shape.vocab_size, (21,), generator=torch.Generator().manual_seed(1))
    # prompt of 13 in two chunks, then 8 single-token steps
    chunks = [(0, 9), (9, 13)] + [(t, t + 1) for t in range(13, 21)]
    for a, b in chunks:
        out = m.forward_tokens(ids[a:b], a)
        ref = o.logits(o.forward(ids[a:b].tolist(), a))
        _close(out["logits"].cpu().numpy(), ref)
        assert torch.equal(out["argmax"].cpu(), out["logits"].argmax(-1).cpu())


def test_batch_invariance_bitwise(tiny):
    from littlebit_b200.model import LittleBitDecoder

    shape, st = tiny
    m = LittleBitDecoder(shape, st, max_seq=256)
    ids = torch.randint(0, shape.vocab_size, (40,), generator=torch.Generator().manual_seed(2))
    m.forward_tokens(ids[:30], 0)
    full = m.forward_tokens(ids[30:40], 30)["logits"]
    # same cache prefix, the ten tokens one at a time
    m2 = LittleBitDecoder(shape, st, max_seq=256)
    m2.forward_tokens(ids[:30], 0)
    for i in range(10):
        one = m2.forward_tokens(ids[30 + i:31 + i], 30 + i)["logits"]
        assert torch.equal(one[0], full[i]), i


@pytest.mark.parametrize("tree", ["small", "binary_d4"])
def test_tree_mask_matches_path_decode(tiny, tree):
    """A tree node's logits are bit-identical to decoding its root-to-node path
    as a plain causal sequence: the property that keeps tree speculation
    token-identical to target-only greedy decoding."""
    from littlebit_b200.model import LittleBitDecoder
    from littlebit_b200.tree_utils import binary_tree_choices, generate_tree_buffers

    shape, st = tiny
    m = LittleBitDecoder(shape, st, max_seq=256)
    ids = torch.randint(0, shape.vocab_size, (64,), generator=torch.Generator().manual_seed(3))
    choices = [[0], [1], [0, 0], [0, 1], [1, 0], [0, 0, 0]] if tree == "small" else binary_tree_choices(4, 2)
    tb = generate_tree_buffers(choices, device="cpu")
    T = tb["tree_len"]
    mask = tb["tree_attn_mask"][0, 0]
    P = 19 if tree == "small" else 50  # the big tree straddles the 64-key chunk boundary
    nodes = ids[:T]
    tmask = [int(sum(1 << j for j in range(T) if mask[i, j])) for i in range(T)]
    tmask = [v - (1 << 64) if v >= (1 << 63) else v for v in tmask]
    pos = P + tb["tree_position_ids"]
    prompt = torch.randint(0, shape.vocab_size, (P,), generator=torch.Generator().manual_seed(7))
    m.forward_tokens(prompt, 0)
    lt = m.forward_tokens(nodes, P, pos=pos, tree_mask=tmask)["logits"].cpu()
    for i in range(T):
        path = [j for j in range(T) if mask[i, j]]
        m2 = LittleBitDecoder(shape, st, max_seq=256)
        m2.forward_tokens(prompt, 0)
        ref = m2.forward_tokens(nodes[path], P)["logits"][-1].cpu()
        assert torch.equal(lt[i], ref), (i, float((lt[i] - ref).abs().max()))


@pytest.mark.parametrize("shared", [False, True])
def test_program_matches_kernel_path_bitwise(tiny, shared):
    """The persistent program (one cooperative launch per step) computes the same
    bits as one grid per op: prefill chunks, single-token steps, a tree step."""
    from littlebit_b200 import _lib as L
    from littlebit_b200.model import LittleBitDecoder, synthetic_runtime_state
    from littlebit_b200.tree_utils import generate_tree_buffers

    shape, st = tiny
    if shared:
        st = synthetic_runtime_state(shape, {k: [v[0], v[0]] for k, v in TINY_RANKS.items()}, seed=6,
                                     shared_residual=True, unit_gain=True)
    mk = LittleBitDecoder(shape, st, max_seq=256, exec_mode=L.LBX_EXEC_KERNELS)
    mp = LittleBitDecoder(shape, st, max_seq=256, exec_mode=L.LBX_EXEC_PROGRAM)
    ids = torch.randint(0, shape.vocab_size, (80,), generator=torch.Generator().manual_seed(8))
    for a, b in [(0, 16), (16, 25), (25, 26), (26, 27), (27, 35), (35, 36)] + [(t, t + 1) for t in range(60, 66)]:
        if a == 60:  # jump over slots 36..59 (a prefix past one 64-key chunk)
            for m in (mk, mp):
                m.forward_tokens(ids[36:60], 36, want_logits=False, want_argmax=False, want_hidden=True)
        ok = mk.forward_tokens(ids[a:b], a, want_hidden=True)
        op = mp.forward_tokens(ids[a:b], a, want_hidden=True)
        assert torch.equal(ok["logits"], op["logits"]), (a, b)
        assert torch.equal(ok["argmax"], op["argmax"]), (a, b)
        assert torch.equal(ok["hidden"], op["hidden"]), (a, b)
    for lk, lp in zip(mk.k_cache + mk.v_cache, mp.k_cache + mp.v_cache):
        assert torch.equal(lk[:, :66], lp[:, :66])
    tb = generate_tree_buffers([[0], [1], [0, 0], [0, 1], [1, 0], [0, 0, 0]], device="cpu")
    T = tb["tree_len"]
    mask = tb["tree_attn_mask"][0, 0]
    tmask = [int(sum(1 << j for j in range(T) if mask[i, j])) for i in range(T)]
    pos = 66 + tb["tree_position_ids"]
    outs = [m.forward_tokens(ids[:T], 66, pos=pos, tree_mask=tmask) for m in (mk, mp)]
    assert torch.equal(outs[0]["logits"], outs[1]["logits"])

