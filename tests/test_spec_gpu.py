"""Speculative decoding on the CUDA models.

Bar (from the task): greedy speculative output is token-identical to greedy
target-only decoding with the same target weights — for the chain loop and the
tree loop, for the per-layer-residual target sharing the draft's packed
factors and for the two-model hidden-sum target.  The residual branch is
scaled down so the draft agrees with the target often enough to exercise
accepted runs, bonus tokens and KV rollback/compaction.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from test_decoder_gpu import TINY, TINY_RANKS, oracle_from_state  # noqa: E402


def _state(seed=7, res_scale=0.08, shared=False, unit_gain=False):
    from littlebit_b200.model import DecoderShape, synthetic_runtime_state

    shape = DecoderShape(**TINY)
    ranks = {k: [v[0], v[0]] for k, v in TINY_RANKS.items()} if shared else TINY_RANKS
    st = synthetic_runtime_state(shape, ranks, seed=seed, shared_residual=shared, unit_gain=unit_gain)
    for k in list(st):
        if k.endswith(".u1_r"):
            st[k] = st[k] * res_scale
    return shape, st


def _models_combined(shared=False, graphs=True, unit_gain=False):
    from littlebit_b200.cuda_models import CudaDraftModel, CudaTargetModel
    from littlebit_b200.model import LittleBitDecoder

    shape, st = _state(shared=shared, unit_gain=unit_gain)
    dec = LittleBitDecoder(shape, st, max_seq=512)
    tgt = CudaTargetModel.from_decoder(dec, use_graphs=graphs)
    drf = CudaDraftModel.from_target(tgt, use_graphs=graphs)
    return shape, st, drf, tgt


def _prompt(shape, n=20, seed=0):
    return torch.randint(0, shape.vocab_size, (1, n), generator=torch.Generator().manual_seed(seed)).cuda()


@pytest.mark.parametrize("shared", [False, True])
def test_chain_token_identity_combined(shared):
    from littlebit_b200.speculative_decoding import autoregressive_generate, speculative_decode

    shape, st, drf, tgt = _models_combined(shared=shared)
    ids = _prompt(shape)
    ar, _ = autoregressive_generate(tgt, ids, None, max_new_tokens=48, eos_token_id=-1)
    sp, stats = speculative_decode(drf, tgt, ids, None, max_new_tokens=48, draft_length=4, eos_token_id=-1)
    assert sp.tolist() == ar.tolist()
    assert stats["total_tokens_generated"] == 48
    assert stats["total_accepted_tokens"] > 0  # accepted runs were exercised


def test_chain_generic_loop_matches_fast_path():
    from littlebit_b200.cuda_models import CudaDraftModel, CudaTargetModel
    from littlebit_b200.speculative_decoding import speculative_decode

    shape, st, drf, tgt = _models_combined()
    ids = _prompt(shape, seed=1)
    fast, _ = speculative_decode(drf, tgt, ids, None, max_new_tokens=24, draft_length=3, eos_token_id=-1)

    class Duck:  # hide the CUDA types: the reference control flow runs
        def __init__(self, m):
            self.m = m

        def __getattr__(self, k):
            return getattr(self.m, k)

    drf.reset(), tgt.reset_cache()
    slow, _ = speculative_decode(Duck(drf), Duck(tgt), ids, None, max_new_tokens=24, draft_length=3,
                                 eos_token_id=-1)
    assert slow.tolist() == fast.tolist()


def test_chain_token_identity_hidden_sum():
    from littlebit_b200.cuda_models import CudaDraftModel, CudaTargetModel
    from littlebit_b200.model import LittleBitDecoder
    from littlebit_b200.speculative_decoding import autoregressive_generate, speculative_decode

    shape, st = _state(seed=9)
    resid_keys = (".v_sign_r_rt", ".v_sign_r_rt_shape", ".u_sign_r_rt", ".u_sign_r_rt_shape", ".v2_r",
                  ".mid_r", ".u1_r")
    draft_st = {k: v for k, v in st.items() if not k.endswith(resid_keys)}
    resid_st = dict(draft_st)
    _, st2 = _state(seed=10)
    for k in list(resid_st):
        if k.endswith((".u_sign_rt", ".v_sign_rt", ".u1", ".v2", ".mid")):
            resid_st[k] = st2[k] * (0.05 if k.endswith(".u1") else 1)
    d_unit = LittleBitDecoder(shape, draft_st, max_seq=512)
    r_unit = LittleBitDecoder(shape, resid_st, max_seq=512, embed=d_unit.embed, lm_head=d_unit.lm_head)
    tgt = CudaTargetModel.from_decoders(d_unit, r_unit)
    drf = CudaDraftModel.from_decoder(LittleBitDecoder(shape, draft_st, max_seq=512))
    ids = _prompt(shape, seed=2)
    ar, _ = autoregressive_generate(tgt, ids, None, max_new_tokens=32, eos_token_id=-1)
    sp, st_ = speculative_decode(drf, tgt, ids, None, max_new_tokens=32, draft_length=4, eos_token_id=-1)
    assert sp.tolist() == ar.tolist()
    # CudaTargetModel.forward (drop-in API) agrees with the fast path's argmax
    lg = tgt.forward(ar[:, :-1])
    assert lg[0, -1].argmax().item() == ar[0, -1].item()


def test_eos_stops_like_reference():
    from littlebit_b200.speculative_decoding import autoregressive_generate, speculative_decode

    shape, st, drf, tgt = _models_combined()
    ids = _prompt(shape, seed=3)
    ar, _ = autoregressive_generate(tgt, ids, None, max_new_tokens=40, eos_token_id=-1)
    eos = int(ar[0, ids.shape[1] + 11])  # a token the target emits: use it as EOS
    ar2, _ = autoregressive_generate(tgt, ids, None, max_new_tokens=40, eos_token_id=eos)
    sp2, _ = speculative_decode(drf, tgt, ids, None, max_new_tokens=40, draft_length=4, eos_token_id=eos)
    first = ar[0, ids.shape[1]:].tolist().index(eos)
    assert ar2.shape[1] == ids.shape[1] + first + 1
    assert sp2[0, :ar2.shape[1]].tolist() == ar2[0].tolist()


def test_tree_token_identity():
    from littlebit_b200.speculative_decoding import autoregressive_generate, speculative_decode_tree
    from littlebit_b200.tree_utils import binary_tree_choices, generate_tree_buffers

    shape, st, drf, tgt = _models_combined()
    ids = _prompt(shape, seed=4)
    tb = generate_tree_buffers(binary_tree_choices(3, 2), device="cuda")
    sp, st_ = speculative_decode_tree(drf, tgt, ids, None, max_new_tokens=40, tree_buffers=tb, top_k=2,
                                      eos_token_id=-1)
    # like speculative_decoding.py:560-566, the last accepted path is not cut at
    # max_new_tokens: up to tree-depth extra tokens, all of them target tokens
    n_new = sp.shape[1] - ids.shape[1]
    assert 40 <= n_new <= 40 + 3
    ar, _ = autoregressive_generate(tgt, ids, None, max_new_tokens=n_new, eos_token_id=-1)
    assert sp.tolist() == ar.tolist()
    assert st_["total_accepted_tokens"] > 0 and st_["decode_mode"] == "tree"


def test_target_logits_match_oracle():
    shape, st, drf, tgt = _models_combined(unit_gain=True)
    o = oracle_from_state(shape, st, 512)
    ids = _prompt(shape, n=12, seed=5)
    lg = tgt.forward(ids)[0].cpu().numpy()
    ref = o.logits(o.forward(ids[0].tolist(), 0))
    np.testing.assert_allclose(lg, ref, rtol=0, atol=1e-2 * np.abs(ref).max())  # basis: test_decoder_gpu._close


def test_littlebit_module_reference_state_dict(golden):
    """LittleBitLinear loads the reference's packed state_dict (littlebit.py:322-345
    keys) without unpacking and matches the reference forward within rtol 1e-3."""
    from helpers import assert_linear_close
    from littlebit_b200.littlebit import LittleBitLinear

    g = golden("linear")
    for name in ("main", "resid", "bias", "tall"):
        in_f, out_f, r, res, bias = (int(v) for v in g[f"{name}_meta"])
        sd = {k[len(f"{name}_sd_"):]: torch.from_numpy(g[k]) for k in g.files if k.startswith(f"{name}_sd_")}
        lin = torch.nn.Linear(in_f, out_f, bias=bool(bias))
        lin.__class__ = LittleBitLinear
        eff = {"main": 1.0, "resid": 2.0, "bias": 1.0, "tall": 0.5}[name]
        lin.__quant_convert__(do_train=False, quant_func=None, split_dim=1024, eff_bit=eff, residual=bool(res))
        lin.load_state_dict(sd, strict=False)
        y = lin(torch.from_numpy(g[f"{name}_x"]).cuda())
        assert_linear_close(y.cpu().numpy(), g[f"{name}_y64"])
        # its own state_dict round-trips the packed words bit-exactly
        sd2 = lin.state_dict()
        assert torch.equal(sd2["U_packed"].cpu(), sd["U_packed"]) and torch.equal(sd2["V_packed"].cpu(), sd["V_packed"])


def test_sampling_mode_device_loop_limits():
    """Sampling-mode chain speculation on the device (drafting, verification
    and the acceptance test of speculative_decoding.py:331-363 on the GPU).
    Two limits pin it: at a vanishing temperature every distribution is one-hot
    and the output is target-only greedy; with the draft equal to the target
    every draft passes the ratio test."""
    from littlebit_b200.cuda_models import CudaDraftModel, CudaTargetModel
    from littlebit_b200.speculative_decoding import autoregressive_generate, speculative_decode

    shape, st, drf, tgt = _models_combined(unit_gain=True)
    ids = _prompt(shape, n=12, seed=3)
    ar, _ = autoregressive_generate(tgt, ids, None, max_new_tokens=32, eos_token_id=-1)
    g = torch.Generator(device="cuda").manual_seed(0)
    from littlebit_b200 import speculative_decoding as sd

    sp, stats = sd._speculative_decode_cuda_sampling(drf, tgt, ids, 32, 4, 1e-6, -1, False, generator=g)
    assert sp.tolist() == ar.tolist()
    assert stats["decode_mode"] == "sampling"
    # the draft is a second copy of the target model: every ratio p/q is 1
    from littlebit_b200.model import LittleBitDecoder

    same = CudaDraftModel.from_decoder(LittleBitDecoder(shape, st, max_seq=512), use_graphs=False)
    sp2, st2 = speculative_decode(same, tgt, ids, None, max_new_tokens=32, draft_length=4, temperature=1.0,
                                  greedy=False, eos_token_id=-1)
    assert st2["acceptance_rate"] == 1.0 and st2["total_tokens_generated"] == 32
    assert sp2.shape[1] == ids.shape[1] + 32
