"""Multi-sequence decoding (lbx_forward_multi, attention with a sequence
dimension, littlebit_b200.batch_decode).

Every sequence of a batched step must get the bits of decoding it alone
(lbx_forward on a single-sequence cache): the linears are batch-invariant and
attention keeps one cache per sequence.  From that, batched greedy decoding
gives each sequence its own target-only greedy tokens, and batched chain
speculation gives them again with per-sequence acceptance.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"

TINY = dict(num_hidden_layers=2, hidden_size=256, intermediate_size=512, num_attention_heads=4,
            num_key_value_heads=2, vocab_size=512)
RANKS = {"q_proj": [64, 32], "k_proj": [32, 16], "v_proj": [32, 16], "o_proj": [64, 32],
         "gate_proj": [96, 40], "up_proj": [96, 40], "down_proj": [96, 40]}


@pytest.fixture(scope="module")
def model():
    from littlebit_b200.model import DecoderShape, LittleBitDecoder, synthetic_runtime_state

    shape = DecoderShape(**TINY)
    st = synthetic_runtime_state(shape, RANKS, seed=21, unit_gain=True)
    for k in list(st):
        if k.endswith(".u1_r"):
            st[k] = st[k] * 0.05  # target close to the draft: speculation accepts often
    return shape, LittleBitDecoder(shape, st, device=DEV, max_seq=96)


def _alone(dec, toks, start_rows=None):
    """Logits of one sequence decoded alone from an empty cache, in the given steps."""
    for c in dec.k_cache + dec.v_cache:
        c.zero_()
    outs, pos = [], 0
    for chunk in toks:
        o = dec.forward_tokens(chunk, pos)
        outs.append(o["logits"])
        pos += len(chunk)
    return torch.cat(outs)


def test_multi_step_bitwise_per_sequence(model):
    from littlebit_b200.batch_decode import BatchDecoder

    shape, dec = model
    S, P = 3, 6
    g = torch.Generator().manual_seed(5)
    prompts = torch.randint(0, shape.vocab_size, (S, P + 3), generator=g)
    bd = BatchDecoder(dec, S, max_seq=96)
    V = shape.vocab_size
    # prefill P tokens of every sequence in one step, then three single-token steps
    lg = torch.empty(S * P, V, device=DEV)
    bd.step(prompts[:, :P].reshape(-1).to(DEV), torch.zeros(S, dtype=torch.int32, device=DEV), 0, P, logits=lg)
    rows = [lg.view(S, P, V)]
    for i in range(3):
        l1 = torch.empty(S, V, device=DEV)
        st = torch.full((S,), P + i, dtype=torch.int32, device=DEV)
        bd.step(prompts[:, P + i].contiguous().to(DEV), st, P + i, 1, logits=l1)
        rows.append(l1.view(S, 1, V))
    got = torch.cat(rows, dim=1)
    torch.cuda.synchronize()
    for s in range(S):
        ref = _alone(dec, [prompts[s, :P].tolist()] + [[int(prompts[s, P + i])] for i in range(3)])
        assert torch.equal(got[s], ref), s


def test_multi_step_ragged_positions(model):
    """Sequences at different cache lengths in one step (the state after
    speculation): each row still equals its own single-sequence step."""
    from littlebit_b200.batch_decode import BatchDecoder

    shape, dec = model
    S = 3
    g = torch.Generator().manual_seed(6)
    lens = [4, 9, 6]
    seqs = [torch.randint(0, shape.vocab_size, (L + 2,), generator=g) for L in lens]
    bd = BatchDecoder(dec, S, max_seq=96)
    # fill each sequence's cache alone-style: step every sequence by its own
    # prefix one token at a time in lockstep batches of 1 (shorter ones pad by
    # re-writing their last slot with the same token, which writes the same bits)
    for t in range(max(lens)):
        tok = torch.tensor([int(seqs[s][min(t, lens[s] - 1)]) for s in range(S)], device=DEV)
        st = torch.tensor([min(t, lens[s] - 1) for s in range(S)], dtype=torch.int32, device=DEV)
        bd.step(tok, st, t, 1)
    # two new tokens per sequence at ragged slots, causal
    tok = torch.stack([seqs[s][lens[s]:lens[s] + 2] for s in range(S)]).reshape(-1).to(DEV)
    st = torch.tensor(lens, dtype=torch.int32, device=DEV)
    lg = torch.empty(S * 2, shape.vocab_size, device=DEV)
    bd.step(tok, st, max(lens), 2, logits=lg)
    torch.cuda.synchronize()
    for s in range(S):
        ref = _alone(dec, [seqs[s][:lens[s]].tolist(), seqs[s][lens[s]:lens[s] + 2].tolist()])
        assert torch.equal(lg.view(S, 2, -1)[s], ref[lens[s]:]), s


def test_batched_greedy_and_speculation_token_identity(model):
    from littlebit_b200.batch_decode import BatchDecoder, greedy_generate, speculative_generate
    from littlebit_b200.cuda_models import CudaTargetModel, _branch0_view
    from littlebit_b200.speculative_decoding import autoregressive_generate

    shape, dec = model
    S, P, G = 4, 8, 20
    g = torch.Generator().manual_seed(7)
    prompts = torch.randint(0, shape.vocab_size, (S, P), generator=g)
    tgt = BatchDecoder(dec, S, max_seq=96)
    drf = BatchDecoder(_branch0_view(dec, 96), S, max_seq=96)
    for bd in (tgt, drf):  # prompt prefill: P-1 tokens; the last one is the first input
        bd.step(prompts[:, :P - 1].reshape(-1).to(DEV), torch.zeros(S, dtype=torch.int32, device=DEV), 0, P - 1)
    last = prompts[:, P - 1].to(DEV)
    greedy = greedy_generate(tgt, last, P - 1, G)
    # (speculation re-writes every slot from P-1 on before any query reads it)
    spec, stats = speculative_generate(drf, tgt, prompts[:, P - 2].to(DEV), last, P - 1, G, gamma=4)
    torch.cuda.synchronize()
    assert torch.equal(spec, greedy)
    assert stats["num_steps"] >= 1 and stats["total_accepted_tokens"] > 0
    # and each sequence's greedy tokens are its own single-sequence greedy run
    single = CudaTargetModel.from_decoder(dec, use_graphs=False)
    for s in range(S):
        single.reset_cache()
        for c in dec.k_cache + dec.v_cache:
            c.zero_()
        out, _ = autoregressive_generate(single, prompts[s:s + 1].to(DEV), None, max_new_tokens=G,
                                         eos_token_id=-1)
        assert out[0, P:].tolist() == greedy[s].tolist(), s
