"""Generate the golden vectors that pin the oracle to the reference.

Runs ONLY where the reference checkout is available (read-only, imported from
LITTLESPEC_REF, default REF below); the resulting .npz files are
committed and the tests never import the reference.

    python tests/golden/make_golden.py

Records, from the reference's own Python code:
  packing.npz   binary_packer words + unpack round trips (binary_packer.py:4-97)
  linear.npz    LittleBitLinear.forward outputs, main/residual/bias
                (littlebit.py:95-121), rank sizing (littlebit.py:50-93)
  convert.npz   convert_state_dict key map on a real LittleBitLinear state_dict
                (convert_hf_to_runtime.py:29-97, littlebit.py:307-345)
  tree.npz      generate_tree_buffers for every preset and the depth-4/binary
                tree, evaluate_posterior_greedy, build_tree_attention_mask
  spec.npz      speculative_decode / autoregressive_generate greedy outputs
                with deterministic table-driven models (speculative_decoding.py)
  hf_llama.npz  HF LlamaForCausalLM + apply_littlebit_patch logits of a tiny
                model (the reference's GPU/HF model path)
  runtime_tiny/ + runtime.npz  runtime checkpoint directories written by the
                reference's convert_hf_to_runtime from two tiny HF LittleBit
                checkpoints (inputs kept beside them), with the HF logits of
                the draft and of the hidden-sum target
  ref_schemas.json  the reference's littlebit_cpu_ops op schemas (cpp:2321-2377)
"""
from __future__ import annotations

import argparse
import json
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REF = Path(os.environ.get("LITTLESPEC_REF", "/root/reference"))
sys.path.insert(0, str(REF))
sys.path.insert(0, str(HERE.parent))  # tests/ for mock_models

import quantization.utils  # noqa: E402,F401  (must precede quantization.modules: circular import)
from quantization.utils.binary_packer import binary_packer, binary_unpacker  # noqa: E402
from quantization.modules.littlebit import LittleBitLinear  # noqa: E402
from quantization.functions import STEBinary  # noqa: E402
import tree_utils  # noqa: E402
import speculative_decoding  # noqa: E402
import convert_hf_to_runtime  # noqa: E402

from mock_models import MockDraft, MockTarget, mock_tables  # noqa: E402


def gen_packing():
    g = torch.Generator().manual_seed(11)
    out = {}
    kat = torch.ones(2, 40, dtype=torch.int8)
    kat[0, 0] = kat[0, 31] = -1
    kat[1, 32] = kat[1, 39] = -1
    cases = {"kat": kat}
    for (r, c) in [(5, 33), (7, 64), (13, 208), (3, 1), (4, 96), (16, 1840), (1, 31)]:
        cases[f"r{r}c{c}"] = (torch.randint(0, 2, (r, c), generator=g, dtype=torch.int8) * 2 - 1)
    for name, t in cases.items():
        p = binary_packer(t)
        u = binary_unpacker(p, tuple(t.shape))
        assert torch.equal(u, t)
        out[f"{name}_signs"] = t.numpy()
        out[f"{name}_packed"] = p.numpy()
    np.savez_compressed(HERE / "packing.npz", **out)


def _mk_linear(in_f, out_f, eff_bit, residual, bias, g):
    lin = torch.nn.Linear(in_f, out_f, bias=bias)
    lin.__class__ = LittleBitLinear
    lin.__quant_convert__(do_train=False, quant_func=STEBinary, split_dim=1024, eff_bit=eff_bit,
                          residual=residual, min_split_dim=8)
    r = int(lin._split_dim_final)
    def pm(*s):
        return torch.nn.Parameter(torch.randn(*s, generator=g, dtype=torch.float32))
    def sc(*s):
        return torch.nn.Parameter((1 + 0.1 * torch.randn(*s, generator=g)).abs())
    lin.U, lin.V = pm(out_f, r), pm(r, in_f)
    lin.u1, lin.u2, lin.v1, lin.v2 = sc(1, out_f), sc(1, r), sc(1, r), sc(1, in_f)
    if residual:
        lin.U_R, lin.V_R = pm(out_f, r), pm(r, in_f)
        lin.u1_R, lin.u2_R, lin.v1_R, lin.v2_R = sc(1, out_f), sc(1, r), sc(1, r), sc(1, in_f)
    if bias:
        lin.bias = torch.nn.Parameter(torch.randn(out_f, generator=g))
    return lin, r


def gen_linear():
    g = torch.Generator().manual_seed(22)
    out = {}
    cases = [("main", 256, 128, 1.0, False, False), ("resid", 256, 384, 2.0, True, False),
             ("bias", 384, 128, 1.0, False, True), ("tall", 128, 512, 0.5, False, False)]
    for name, in_f, out_f, eb, res, bias in cases:
        lin, r = _mk_linear(in_f, out_f, eb, res, bias, g)
        x = torch.randn(5, in_f, generator=g)
        with torch.no_grad():
            y32 = lin(x)                   # latent weights quantised by STEBinary
            sd = lin.state_dict()          # packed keys (littlebit.py:322-345)
            lin64 = lin.double()
            y64 = lin64(x.double())
        out[f"{name}_x"] = x.numpy()
        out[f"{name}_y32"] = y32.numpy()
        out[f"{name}_y64"] = y64.numpy()
        out[f"{name}_meta"] = np.array([in_f, out_f, r, int(res), int(bias)])
        for k, v in sd.items():
            if k.startswith("_") or k in ("weight",):
                continue
            out[f"{name}_sd_{k}"] = v.detach().float().numpy() if v.is_floating_point() else v.numpy()
    # rank sizing table (littlebit.py:50-93)
    rows = []
    for a, b in [(4096, 4096), (4096, 11008), (11008, 4096), (8192, 8192), (8192, 1024),
                 (8192, 28672), (28672, 8192), (4096, 1024), (256, 256)]:
        for eb in (0.1, 0.55, 0.9, 1.0):
            for res in (False, True):
                f = LittleBitLinear._estimate_split_dim(a, b, eb, res)
                s = LittleBitLinear._finalize_split_dim(f, 1024, 8)
                rows.append([a, b, eb, int(res), s, LittleBitLinear._compute_eff_bits(a, b, s, res)])
    out["ranks"] = np.array(rows, dtype=np.float64)
    np.savez_compressed(HERE / "linear.npz", **out)


def gen_convert():
    g = torch.Generator().manual_seed(33)
    hf = {}
    for i, (res, in_f, out_f) in enumerate([(False, 256, 128), (True, 128, 256)]):
        lin, r = _mk_linear(in_f, out_f, 1.0, res, False, g)
        for k, v in lin.state_dict().items():
            hf[f"model.layers.{i}.mlp.proj.{k}"] = v
    hf["model.embed_tokens.weight"] = torch.randn(10, 8, generator=g)
    rt = convert_hf_to_runtime.convert_state_dict(hf)
    out = {"hf_keys": np.array(sorted(hf)), "rt_keys": np.array(sorted(rt))}
    for k, v in hf.items():
        out["hf/" + k] = v.numpy()
    for k, v in rt.items():
        out["rt/" + k] = v.numpy()
    np.savez_compressed(HERE / "convert.npz", **out)


def gen_tree():
    out = {}
    presets = dict(tree_utils.TREE_PRESETS)
    presets["binary_d4"] = [list(p) for d in range(1, 5) for p in np.ndindex(*([2] * d))]
    for name, choices in presets.items():
        tb = tree_utils.generate_tree_buffers(choices, device="cpu")
        out[f"{name}_choices"] = np.array(json.dumps([list(map(int, c)) for c in choices]))
        out[f"{name}_mask"] = tb["tree_attn_mask"].numpy()
        out[f"{name}_pos"] = tb["tree_position_ids"].numpy()
        out[f"{name}_retrieve"] = tb["retrieve_indices"].numpy()
        out[f"{name}_depth_counts"] = np.array(tb["depth_counts"])
        m = tree_utils.build_tree_attention_mask(7, tb["tree_attn_mask"], "cpu", torch.float32)
        out[f"{name}_full_mask_p7"] = (m[0, 0] == 0).numpy()
    g = torch.Generator().manual_seed(44)
    for i in range(6):
        L, D = 6, 4
        logits = torch.randn(L, D + 1, 9, generator=g)
        cand = torch.randint(0, 9, (L, D + 1), generator=g)
        # plant matches so accept lengths vary
        am = logits.argmax(-1)
        for l in range(L):
            m = int(torch.randint(0, D + 1, (1,), generator=g))
            cand[l, 1:m + 1] = am[l, :m]
        b, a, nl = tree_utils.evaluate_posterior_greedy(logits, cand)
        out[f"post{i}_logits"], out[f"post{i}_cand"] = logits.numpy(), cand.numpy()
        out[f"post{i}_res"] = np.array([int(b), int(a)])
        out[f"post{i}_next"] = nl.numpy()
    np.savez_compressed(HERE / "tree.npz", **out)


def gen_spec():
    out = {}
    tabs = mock_tables(vocab=50, seed=5)
    for j, (k, n_new, eos) in enumerate([(4, 40, -1), (5, 37, -1), (3, 30, 7), (1, 12, -1)]):
        d = MockDraft(tabs, torch)
        t = MockTarget(tabs, torch)
        ids = torch.tensor([[3, 17, 29, 4, 11]])
        o, st = speculative_decoding.speculative_decode(d, t, ids, None, max_new_tokens=n_new,
                                                        draft_length=k, greedy=True,
                                                        eos_token_id=eos)
        ar, _ = speculative_decoding.autoregressive_generate(t, ids, None, max_new_tokens=n_new,
                                                             greedy=True, eos_token_id=eos)
        out[f"case{j}_params"] = np.array([k, n_new, eos])
        out[f"case{j}_spec"] = o.numpy()
        out[f"case{j}_ar"] = ar.numpy()
        out[f"case{j}_stats"] = np.array([st["total_tokens_generated"], st["total_draft_tokens"],
                                          st["total_accepted_tokens"], st["num_steps"]])
    np.savez_compressed(HERE / "spec.npz", **out)


def gen_hf_llama():
    from transformers import LlamaConfig, LlamaForCausalLM
    from quantization.utils.quant_util import apply_littlebit_patch
    import argparse as ap
    torch.manual_seed(0)
    cfg = LlamaConfig(hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, vocab_size=384,
                      max_position_embeddings=256, rms_norm_eps=1e-6, rope_theta=10000.0,
                      tie_word_embeddings=False, attn_implementation="eager")
    model = LlamaForCausalLM(cfg)
    args = ap.Namespace(quant_func="STEBinary", quant_mod="LittleBitLinear", eff_bit=1.0,
                        split_dim=1024, residual=True, kv_factor=1.0, min_split_dim=8, model_id="tiny")
    apply_littlebit_patch(model, args, do_train=False)
    g = torch.Generator().manual_seed(55)
    out = {}
    for name, mod in model.named_modules():
        if isinstance(mod, LittleBitLinear):
            r = mod.split_dim
            for suf in ("", "_R"):
                U = (torch.randint(0, 2, (mod.out_features, r), generator=g) * 2 - 1).float()
                V = (torch.randint(0, 2, (r, mod.in_features), generator=g) * 2 - 1).float()
                s = lambda *sh: (1 + 0.1 * torch.randn(*sh, generator=g)).abs()
                setattr(mod, "U" + suf, torch.nn.Parameter(U, requires_grad=False))
                setattr(mod, "V" + suf, torch.nn.Parameter(V, requires_grad=False))
                for nm, sh in (("u1", (1, mod.out_features)), ("u2", (1, r)), ("v1", (1, r)),
                               ("v2", (1, mod.in_features))):
                    setattr(mod, nm + suf, torch.nn.Parameter(s(*sh), requires_grad=False))
            mod._binarized = True
    with torch.no_grad():
        emb = (0.02 * torch.randn(cfg.vocab_size, cfg.hidden_size, generator=g)).bfloat16().float()
        head = (0.02 * torch.randn(cfg.vocab_size, cfg.hidden_size, generator=g)).bfloat16().float()
        model.model.embed_tokens.weight.copy_(emb)
        model.lm_head.weight.copy_(head)
        for ly in model.model.layers:
            ly.input_layernorm.weight.copy_((1 + 0.1 * torch.randn(cfg.hidden_size, generator=g)).abs())
            ly.post_attention_layernorm.weight.copy_((1 + 0.1 * torch.randn(cfg.hidden_size, generator=g)).abs())
        model.model.norm.weight.copy_((1 + 0.1 * torch.randn(cfg.hidden_size, generator=g)).abs())
        model = model.float().eval()
        ids = torch.randint(0, cfg.vocab_size, (1, 12), generator=g)
        logits = model(input_ids=ids).logits[0]
        sd = model.state_dict()  # packed LittleBit keys (littlebit.py:322-345)
    out["ids"] = ids.numpy()[0]
    out["logits"] = logits.numpy()
    out["config"] = np.array(json.dumps(cfg.to_dict(), default=str))
    for k, v in sd.items():
        if k.endswith(("_eff_bit_target", "_split_dim_final", "_eff_bit_actual")):
            continue
        out["sd/" + k] = v.numpy() if not v.is_floating_point() else v.float().numpy()
    np.savez_compressed(HERE / "hf_llama.npz", **out)


def _tiny_lb_llama(name, eff_bit, residual, g, embed=None, head=None):
    """A tiny HF LlamaForCausalLM patched with the reference's apply_littlebit_patch,
    seeded +-1 factors and near-unit-gain |N(1,0.1)| scales (v1 / sqrt(in),
    u1 / sqrt(rank): activations stay in the range of a trained checkpoint),
    bf16-representable embedding and lm_head.  Returns (config, model, lb_args)."""
    from transformers import LlamaConfig, LlamaForCausalLM
    from quantization.utils.quant_util import apply_littlebit_patch
    import argparse as ap
    torch.manual_seed(0)
    cfg = LlamaConfig(hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, vocab_size=128,
                      max_position_embeddings=256, rms_norm_eps=1e-6, rope_theta=10000.0,
                      tie_word_embeddings=False, attn_implementation="eager")
    cfg._name_or_path = name
    model = LlamaForCausalLM(cfg)
    args = ap.Namespace(quant_func="STEBinary", quant_mod="LittleBitLinear", eff_bit=eff_bit,
                        split_dim=1024, residual=residual, kv_factor=1.0, min_split_dim=8, model_id=name)
    apply_littlebit_patch(model, args, do_train=False)
    for _, mod in model.named_modules():
        if isinstance(mod, LittleBitLinear):
            r = mod.split_dim
            for suf in ("", "_R") if residual else ("",):
                U = (torch.randint(0, 2, (mod.out_features, r), generator=g) * 2 - 1).float()
                V = (torch.randint(0, 2, (r, mod.in_features), generator=g) * 2 - 1).float()
                s = lambda *sh: (1 + 0.1 * torch.randn(*sh, generator=g)).abs()
                setattr(mod, "U" + suf, torch.nn.Parameter(U, requires_grad=False))
                setattr(mod, "V" + suf, torch.nn.Parameter(V, requires_grad=False))
                gain = {"u1": r ** -0.5, "v1": mod.in_features ** -0.5, "u2": 1.0, "v2": 1.0}
                for nm, sh in (("u1", (1, mod.out_features)), ("u2", (1, r)), ("v1", (1, r)),
                               ("v2", (1, mod.in_features))):
                    setattr(mod, nm + suf, torch.nn.Parameter(s(*sh) * gain[nm], requires_grad=False))
            mod._binarized = True
    with torch.no_grad():
        if embed is None:
            embed = (0.02 * torch.randn(cfg.vocab_size, cfg.hidden_size, generator=g)).bfloat16().float()
            head = (0.02 * torch.randn(cfg.vocab_size, cfg.hidden_size, generator=g)).bfloat16().float()
        model.model.embed_tokens.weight.copy_(embed)
        model.lm_head.weight.copy_(head)
        for ly in model.model.layers:
            ly.input_layernorm.weight.copy_((1 + 0.1 * torch.randn(cfg.hidden_size, generator=g)).abs())
            ly.post_attention_layernorm.weight.copy_((1 + 0.1 * torch.randn(cfg.hidden_size, generator=g)).abs())
        model.model.norm.weight.copy_((1 + 0.1 * torch.randn(cfg.hidden_size, generator=g)).abs())
    return cfg, model.float().eval(), args


def gen_runtime():
    """Runtime checkpoint directories written by the reference's own converter.

    Two tiny HF LittleBit Llamas sharing one embedding/lm_head (a 0.5-bit
    "draft" and a 1.0-bit residual-branch "residual" model) are saved as the
    reference's training scripts save a checkpoint (the packed state_dict of
    littlebit.py:322-345 as model.safetensors, config.json, and the
    littlebit_config.json of main.py:282-294).  convert_hf_to_runtime
    (convert_hf_to_runtime.py:238-290) then writes each runtime directory:
    littlebit_runtime.safetensors, littlebit_runtime_config.json and
    dummy_llama3_config.json.  Both the HF inputs and the converter's outputs
    are kept under runtime_tiny/, with the HF logits of the draft and of the
    hidden-sum target lm_head(norm(h_draft) + norm(h_res)) of
    cpu_target_model.py:516-527 in runtime.npz."""
    import shutil
    import tempfile
    from safetensors.torch import save_file

    base = HERE / "runtime_tiny"
    if base.exists():
        shutil.rmtree(base)
    g = torch.Generator().manual_seed(77)
    cd, md, ad = _tiny_lb_llama("tiny-littlebit-draft", 0.5, False, g)
    cr, mr, ar = _tiny_lb_llama("tiny-littlebit-residual", 1.0, True, g,
                                embed=md.model.embed_tokens.weight.detach().clone(),
                                head=md.lm_head.weight.detach().clone())
    out = {}
    ids = torch.randint(0, cd.vocab_size, (1, 12), generator=g)
    with torch.no_grad():
        out["draft_logits"] = md(input_ids=ids).logits[0].numpy()
        hd = md.model(input_ids=ids).last_hidden_state[0]
        hr = mr.model(input_ids=ids).last_hidden_state[0]
        out["target_logits"] = ((hd + hr) @ md.lm_head.weight.T).numpy()
    out["ids"] = ids.numpy()[0]
    for tag, cfg, model, args in (("draft", cd, md, ad), ("residual", cr, mr, ar)):
        hf_dir = base / f"{tag}_hf"
        hf_dir.mkdir(parents=True)
        sd = {}
        for k, v in model.state_dict().items():
            if k in ("model.embed_tokens.weight", "lm_head.weight"):
                v = v.to(torch.bfloat16)  # as saved in torch_dtype bfloat16 (exact: bf16 values)
            sd[k] = v.contiguous()
        save_file(sd, str(hf_dir / "model.safetensors"))
        (hf_dir / "config.json").write_text(json.dumps(cfg.to_dict(), indent=2, default=str))
        lb = {"quant_func": args.quant_func, "eff_bit": args.eff_bit, "split_dim": args.split_dim,
              "residual": args.residual, "kv_factor": args.kv_factor, "min_split_dim": args.min_split_dim,
              "quant_mod": args.quant_mod}
        (hf_dir / "littlebit_config.json").write_text(json.dumps(lb, indent=2))
        with tempfile.TemporaryDirectory() as td:
            convert_hf_to_runtime.convert_hf_to_runtime(str(hf_dir), td)
            rt_dir = base / tag
            rt_dir.mkdir()
            for f in ("littlebit_runtime.safetensors", "littlebit_runtime_config.json",
                      "dummy_llama3_config.json"):
                shutil.copy2(Path(td) / f, rt_dir / f)
    np.savez_compressed(HERE / "runtime.npz", **out)


def gen_schemas():
    """The op schemas of the reference's TORCH_LIBRARY block
    (patches/littlebit_cpu_optimized.cpp:2321-2377), read as text."""
    import re

    src = (REF / "patches" / "littlebit_cpu_optimized.cpp").read_text()
    block = src[src.index("TORCH_LIBRARY(littlebit_cpu_ops"):]
    block = block[:block.index("TORCH_LIBRARY_IMPL")]
    defs = re.findall(r'm\.def\(\s*((?:"[^"]*"\s*)+)\)', block)
    schemas = ["".join(re.findall(r'"([^"]*)"', d)) for d in defs]
    (HERE / "ref_schemas.json").write_text(json.dumps(schemas, indent=1) + "\n")


if __name__ == "__main__":
    ap_ = argparse.ArgumentParser()
    ap_.add_argument("--only", default="")
    a = ap_.parse_args()
    for fn in (gen_packing, gen_linear, gen_convert, gen_tree, gen_spec, gen_hf_llama, gen_runtime,
               gen_schemas):
        if a.only and a.only not in fn.__name__:
            continue
        fn()
        print("wrote", fn.__name__)
