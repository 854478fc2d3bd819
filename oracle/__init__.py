"""CPU oracle for the LittleBit hot path — TEST INFRASTRUCTURE ONLY.

A numpy restatement of the reference algorithms (kimwin2/LittleSpec), each
function citing the reference file:line it follows.  It is the checker the
CUDA path is compared against, never part of the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import it.

Pinning: the restatement is checked against golden vectors produced by the
reference's own Python code (tests/golden/make_golden.py imports the
reference read-only and records binary_packer words, _compute_forward
outputs, convert_state_dict keys, tree buffers, posterior evaluation, the
greedy speculative loop and HF-Llama+LittleBit logits), see tests/test_oracle.py.

Modules:
  packing   — binary_packer / binary_unpacker / sign          (binary_packer.py, binary.py)
  littlebit — rank sizing, _compute_forward, runtime converter (littlebit.py, convert_hf_to_runtime.py)
  decoder   — LittleBit Llama decoder with KV cache, RoPE, tree masks (HF Llama + cpp:1522-2079)
  spec      — greedy speculative loop, tree buffers, posterior  (speculative_decoding.py, tree_utils.py)
"""
