"""Host-side logic of the B200 package against the reference's own outputs
(tests/golden/*.npz).  No GPU: these modules are plain Python/torch control
flow, key mapping and tree bookkeeping."""
import json

import numpy as np
import pytest
import torch

from littlebit_b200 import runtime as rt
from littlebit_b200 import speculative_decoding as sd
from littlebit_b200 import tree_utils as tu
from littlebit_b200.littlebit import LittleBitLinear


def test_spec_loop_matches_reference(golden):
    from mock_models import MockDraft, MockTarget, mock_tables

    g = golden("spec")
    tabs = mock_tables(vocab=50, seed=5)
    for j in range(4):
        k, n_new, eos = (int(v) for v in g[f"case{j}_params"])
        ids = torch.tensor([[3, 17, 29, 4, 11]])
        out, st = sd.speculative_decode(MockDraft(tabs, torch), MockTarget(tabs, torch), ids, None,
                                        max_new_tokens=n_new, draft_length=k, greedy=True,
                                        eos_token_id=eos)
        assert out[0].tolist() == g[f"case{j}_spec"][0].tolist()
        assert [st["total_tokens_generated"], st["total_draft_tokens"], st["total_accepted_tokens"],
                st["num_steps"]] == g[f"case{j}_stats"].tolist()
        ar, _ = sd.autoregressive_generate(MockTarget(tabs, torch), ids, None, max_new_tokens=n_new,
                                           greedy=True, eos_token_id=eos)
        assert ar[0].tolist() == g[f"case{j}_ar"][0].tolist()


def test_spec_stats_keys():
    from mock_models import MockDraft, MockTarget, mock_tables

    tabs = mock_tables(vocab=50, seed=5)
    _, st = sd.speculative_decode(MockDraft(tabs, torch), MockTarget(tabs, torch),
                                  torch.tensor([[1, 2, 3]]), None, max_new_tokens=5, draft_length=2)
    assert set(st) == {"total_tokens_generated", "total_draft_tokens", "total_accepted_tokens",
                       "num_steps", "mean_acceptance_length", "acceptance_rate",
                       "tokens_per_second", "elapsed_seconds", "draft_length_k"}


def test_tree_buffers_match_reference(golden):
    g = golden("tree")
    names = sorted({k.rsplit("_", 1)[0] for k in g.files if k.endswith("_choices")})
    for n in names:
        ch = json.loads(str(g[f"{n}_choices"]))
        tb = tu.generate_tree_buffers(ch, device="cpu")
        np.testing.assert_array_equal(tb["tree_attn_mask"].numpy(), g[f"{n}_mask"])
        np.testing.assert_array_equal(tb["tree_position_ids"].numpy(), g[f"{n}_pos"])
        np.testing.assert_array_equal(tb["retrieve_indices"].numpy(), g[f"{n}_retrieve"])
        assert tb["depth_counts"] == g[f"{n}_depth_counts"].tolist()
        m = tu.build_tree_attention_mask(7, tb["tree_attn_mask"], "cpu", torch.float32)
        np.testing.assert_array_equal((m[0, 0] == 0).numpy(), g[f"{n}_full_mask_p7"])
    assert tu.binary_tree_choices(4, 2) == json.loads(str(g["binary_d4_choices"]))
    for name, ch in tu.TREE_PRESETS.items():
        assert ch == json.loads(str(g[f"{name}_choices"]))


def test_tree_bitmasks():
    tb = tu.generate_tree_buffers(tu.binary_tree_choices(4, 2), device="cpu")
    bits = tu.tree_bitmasks(tb["tree_attn_mask"])
    m = tb["tree_attn_mask"][0, 0]
    for i in range(tb["tree_len"]):
        for j in range(tb["tree_len"]):
            assert bool((int(bits[i]) >> j) & 1) == bool(m[i, j])


def test_posterior_greedy_matches_reference(golden):
    g = golden("tree")
    for i in range(6):
        b, a, nl = tu.evaluate_posterior_greedy(torch.from_numpy(g[f"post{i}_logits"]),
                                                torch.from_numpy(g[f"post{i}_cand"]))
        assert [int(b), a] == g[f"post{i}_res"].tolist()
        np.testing.assert_array_equal(nl.numpy(), g[f"post{i}_next"])


def test_convert_state_dict_matches_reference(golden):
    g = golden("convert")
    hf = {k[3:]: torch.from_numpy(g[k]) for k in g.files if k.startswith("hf/")}
    out = rt.convert_state_dict(hf)
    assert sorted(out) == sorted(g["rt_keys"].tolist())
    for k, v in out.items():
        np.testing.assert_array_equal(v.numpy(), g["rt/" + k], err_msg=k)
    can = rt.convert_state_dict_canonical(hf)
    assert any(k.endswith(".u_sign_packed") for k in can)
    assert any(k.endswith(".u_sign_r_packed") for k in can)


def test_rank_sizing_matches_reference(golden):
    for a, b, eb, res, s, eff in golden("linear")["ranks"]:
        f = LittleBitLinear._estimate_split_dim(int(a), int(b), eb, bool(res))
        assert LittleBitLinear._finalize_split_dim(f, 1024, 8) == int(s)
        assert LittleBitLinear._compute_eff_bits(int(a), int(b), int(s), bool(res)) == pytest.approx(eff, rel=1e-12)


def test_runtime_directory_roundtrip(tmp_path):
    from littlebit_b200.model import DecoderShape, load_runtime, save_runtime, synthetic_runtime_state

    shape = DecoderShape(1, 256, 512, 4, 2, 300)
    ranks = {k: [16, 8] for k in ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")}
    st = synthetic_runtime_state(shape, ranks, seed=1)
    save_runtime(tmp_path / "ck", st, shape, eff_bit=0.1, residual=True)
    st2, shape2, cfg = load_runtime(tmp_path / "ck")
    assert shape2.hidden_size == 256 and shape2.num_key_value_heads == 2
    assert cfg["format_version"] == 1 and cfg["sign_storage"] == "row_i1"
    assert sorted(st) == sorted(st2)
    for k in st:
        assert torch.equal(st[k], st2[k]), k


def test_littlebit_module_conversion_api():
    lin = torch.nn.Linear(4096, 4096, bias=False)
    lin.__class__ = LittleBitLinear
    lin.__quant_convert__(do_train=False, quant_func=None, split_dim=1024, eff_bit=0.1, residual=False)
    assert int(lin._split_dim_final) == 184
    assert lin.U.shape == (4096, 184) and lin.V.shape == (184, 4096)
    assert lin.eff_bit_target == pytest.approx(0.1)
    with pytest.raises(NotImplementedError):
        lin2 = torch.nn.Linear(128, 128)
        lin2.__class__ = LittleBitLinear
        lin2.__quant_convert__(do_train=True, quant_func=None, eff_bit=1.0)
