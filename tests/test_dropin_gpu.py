"""The drop-in constructors on directories written by the reference's converter.

CudaDraftModel(runtime_path, base_model_id) and CudaTargetModel(draft_runtime_path,
residual_runtime_path, base_model_id) are what a user of CPUDraftModel /
CPUTargetModel (cpu_draft_model.py:141-268, cpu_target_model.py:371-420) calls.
Here they load tests/golden/runtime_tiny/{draft,residual}, written by the
reference's convert_hf_to_runtime from two tiny HF LittleBit checkpoints, and
their logits are held to the HF model's own logits (runtime.npz) with the
end-to-end decoder tolerance of test_decoder_gpu._close.  Greedy speculative
decoding with the two is token-identical to target-only greedy decoding.
"""
import pytest
import torch

from conftest import GOLDEN
from test_decoder_gpu import _close

pytestmark = pytest.mark.gpu
RT = GOLDEN / "runtime_tiny"


def test_constructors_match_hf_logits(golden):
    from littlebit_b200.cuda_models import CudaDraftModel, CudaTargetModel

    g = golden("runtime")
    ids = torch.tensor(g["ids"], dtype=torch.int64)[None]
    drf = CudaDraftModel(str(RT / "draft"), None, max_seq_len=64)
    _close(drf.forward(ids).logits[0].cpu().numpy(), g["draft_logits"])
    tgt = CudaTargetModel(str(RT / "draft"), str(RT / "residual"), None, max_seq_len=64)
    _close(tgt.forward(ids)[0].cpu().numpy(), g["target_logits"])


def test_constructors_spec_decode_token_identity(golden):
    from littlebit_b200.cuda_models import CudaDraftModel, CudaTargetModel
    from littlebit_b200.speculative_decoding import autoregressive_generate, speculative_decode

    g = golden("runtime")
    ids = torch.tensor(g["ids"], dtype=torch.int64)[None].cuda()
    drf = CudaDraftModel(str(RT / "draft"), None, max_seq_len=64)
    tgt = CudaTargetModel(str(RT / "draft"), str(RT / "residual"), None, max_seq_len=64)
    ar, _ = autoregressive_generate(tgt, ids, None, max_new_tokens=24, eos_token_id=-1)
    tgt.reset_cache()
    sp, st = speculative_decode(drf, tgt, ids, None, max_new_tokens=24, draft_length=4, eos_token_id=-1)
    assert sp.tolist() == ar.tolist()
    assert st["num_steps"] >= 1
