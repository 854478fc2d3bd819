"""Runtime checkpoint directories written by the reference's own converter.

tests/golden/runtime_tiny/ holds two tiny HF LittleBit checkpoints ({draft,
residual}_hf: model.safetensors, config.json, littlebit_config.json) and the
directories the reference's convert_hf_to_runtime (convert_hf_to_runtime.py:
238-290) wrote from them; runtime.npz holds the HF model's logits of the
draft and of the hidden-sum target (cpu_target_model.py:516-527).  These
tests pin the config builders, the directory-level converter and the loader
to those files, and the oracle (through the loader) to the HF logits.
"""
import json

import numpy as np
import pytest
import torch

from conftest import GOLDEN

RT = GOLDEN / "runtime_tiny"
TAGS = ("draft", "residual")


@pytest.mark.parametrize("tag", TAGS)
def test_config_builders_match_reference_files(tag):
    from littlebit_b200.runtime import build_dummy_config, build_runtime_config

    hf = RT / f"{tag}_hf"
    args = (str(hf / "config.json"), str(hf / "littlebit_config.json"))
    assert build_dummy_config(*args) == json.loads((RT / tag / "dummy_llama3_config.json").read_text())
    assert build_runtime_config(*args) == json.loads((RT / tag / "littlebit_runtime_config.json").read_text())


@pytest.mark.parametrize("tag", TAGS)
def test_directory_conversion_matches_reference(tag, tmp_path):
    from safetensors.torch import load_file

    from littlebit_b200.runtime import convert_hf_to_runtime

    out = tmp_path / tag
    convert_hf_to_runtime(RT / f"{tag}_hf", out)
    ref = RT / tag
    for f in ("dummy_llama3_config.json", "littlebit_runtime_config.json"):
        assert json.loads((out / f).read_text()) == json.loads((ref / f).read_text()), f
    a = load_file(str(out / "littlebit_runtime.safetensors"))
    b = load_file(str(ref / "littlebit_runtime.safetensors"))
    assert sorted(a) == sorted(b)
    for k in b:
        assert a[k].dtype == b[k].dtype and torch.equal(a[k], b[k]), k


def test_loader_reads_reference_directories():
    from littlebit_b200.model import load_runtime
    from littlebit_b200.runtime import load_runtime_checkpoint

    for tag in TAGS:
        state, shape, rt = load_runtime(RT / tag)
        hf = json.loads((RT / f"{tag}_hf" / "config.json").read_text())
        assert (shape.num_hidden_layers, shape.hidden_size, shape.intermediate_size,
                shape.num_attention_heads, shape.num_key_value_heads, shape.vocab_size) == (
            hf["num_hidden_layers"], hf["hidden_size"], hf["intermediate_size"],
            hf["num_attention_heads"], hf["num_key_value_heads"], hf["vocab_size"])
        assert rt["format_version"] == 1 and rt["sign_storage"] == "row_i1"
        st2, rt2 = load_runtime_checkpoint(RT / tag)
        assert rt2 == rt and sorted(st2) == sorted(state)


def _oracle(tag, kv_bf16=False):
    from littlebit_b200.model import load_runtime
    from oracle.decoder import from_runtime_state

    state, s, _ = load_runtime(RT / tag)
    return from_runtime_state(state, s.num_hidden_layers, s.hidden_size, s.intermediate_size,
                              s.num_attention_heads, s.num_key_value_heads, s.vocab_size,
                              rms_eps=s.rms_norm_eps, rope_theta=s.rope_theta, max_seq=64,
                              kv_bf16=kv_bf16)


def test_oracle_through_reference_directories_matches_hf(golden):
    g = golden("runtime")
    ids = g["ids"].tolist()
    d = _oracle("draft")
    ref = g["draft_logits"]
    np.testing.assert_allclose(d.logits(d.forward(ids, 0)), ref, rtol=1e-4, atol=1e-4 * np.abs(ref).max())
    d.reset()
    r = _oracle("residual")
    h = d.final_hidden(d.forward(ids, 0)) + r.final_hidden(r.forward(ids, 0))
    ref = g["target_logits"]
    np.testing.assert_allclose(h @ d.lm_head.T, ref, rtol=1e-4, atol=1e-4 * np.abs(ref).max())
