"""The C-ABI library loads on a CPU-only host, exports every symbol
include/lbx.h declares, and the ctypes mirrors match the C struct layouts."""
import ctypes
import re
import shutil
import subprocess
from pathlib import Path

import pytest

from littlebit_b200 import _lib as L

ROOT = Path(__file__).resolve().parent.parent
HDR = ROOT / "include" / "lbx.h"


def declared_functions():
    txt = re.sub(r"/\*.*?\*/", "", HDR.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(lbx_[a-z0-9_]+)\s*\(", txt)))


def test_library_exports_every_declared_symbol():
    lib = L.load()
    names = declared_functions()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    assert set(names) == set(L.EXPORTED)
    assert lib.lbx_version().decode().startswith("lbx")


def test_last_error_roundtrip_without_gpu():
    # argument validation runs on the host: no GPU needed
    lib = L.load()
    rc = lib.lbx_pack_signs(None, -1, 3, None, None, None)
    assert rc == L.LBX_EINVAL
    assert "negative" in L.last_error()
    with pytest.raises(RuntimeError, match="invalid argument"):
        L.check(rc, "pack")


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc missing")
def test_struct_layouts_match_c(tmp_path):
    structs = {"lbx_branch": L.Branch, "lbx_proj": L.Proj, "lbx_linear_args": L.LinearArgs,
               "lbx_attn_args": L.AttnArgs, "lbx_layer": L.Layer, "lbx_model": L.Model}
    src = ['#include <stdio.h>', '#include <stddef.h>', f'#include "{HDR}"', "int main(void){"]
    for c in structs:
        src.append(f'printf("{c} %zu\\n", sizeof({c}));')
    for c, py in structs.items():
        for f, _ in py._fields_:
            src.append(f'printf("{c}.{f} %zu\\n", offsetof({c}, {f}));')
    src.append("return 0;}")
    (tmp_path / "s.c").write_text("\n".join(src))
    exe = tmp_path / "s"
    cuda_inc = "/usr/local/cuda/include"
    subprocess.run(["gcc", "-I", cuda_inc, str(tmp_path / "s.c"), "-o", str(exe)], check=True)
    out = dict(l.rsplit(" ", 1) for l in subprocess.run([str(exe)], capture_output=True, text=True,
                                                         check=True).stdout.splitlines())
    for c, py in structs.items():
        assert int(out[c]) == ctypes.sizeof(py), c
        for f, _ in py._fields_:
            assert int(out[f"{c}.{f}"]) == getattr(py, f).offset, f"{c}.{f}"
