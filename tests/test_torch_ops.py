"""torch.ops.littlebit_cuda_ops registers schemas parallel to the reference's
littlebit_cpu_ops (tests/golden/ref_schemas.json, read from
patches/littlebit_cpu_optimized.cpp:2321-2377).  No GPU needed."""
import json
import re
from pathlib import Path

import torch

import littlebit_b200.torch_ops as tops

GOLD = Path(__file__).resolve().parent / "golden" / "ref_schemas.json"
# formats the B200 path does not use: int8 activation quantisation (W1A8, lossy),
# the i2 sign repack (drops signs when cols % 128 != 0) and Q4_0 lm_head blocks
NOT_PROVIDED = {"quantize_per_row_int8", "gemv_int8xsign", "repack_signs_to_i2", "littlebit_linear_i2",
                "quantize_lm_head_q4"}


def _args(schema: str):
    """[(type, name)] of a schema string, alias annotations removed."""
    inner = schema[schema.index("(") + 1: schema.rindex(")", 0, schema.index("->"))]
    out = []
    for a in inner.split(","):
        typ, name = a.strip().rsplit(" ", 1)
        out.append((re.sub(r"\([a-z]!?\)", "", typ), name))
    return out


def test_schemas_parallel_the_reference():
    ref = {s[:s.index("(")]: s for s in json.loads(GOLD.read_text())}
    assert set(ref) == set(tops.SCHEMAS) | NOT_PROVIDED
    for name, schema in tops.SCHEMAS.items():
        assert _args(schema) == _args(ref[name]), name
        assert schema.split("->")[1].strip() == ref[name].split("->")[1].strip(), name
        op = getattr(torch.ops.littlebit_cuda_ops, name)
        assert str(op.default._schema).startswith(f"littlebit_cuda_ops::{name}(")


def test_cpu_tensors_have_no_kernel():
    x = torch.zeros(1, 4)
    try:
        torch.ops.littlebit_cuda_ops.silu_mul(x, x)
    except (NotImplementedError, RuntimeError) as e:
        assert "CPU" in str(e) or "kernel" in str(e).lower()
    else:
        raise AssertionError("a CPU tensor must not be served")
