"""The C-ABI library: it loads, exports every entry point the header declares,
and the ctypes mirror has the header's exact struct layout (checked against a
C program compiled from include/mace_b200.h).  No GPU calls."""

import ctypes as C
import re
import shutil
import subprocess
from pathlib import Path

import pytest

from mace_mlx_b200 import native as nv

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "mace_b200.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*int\s+(mace_\w+)\s*\(", text, flags=re.M)))


def test_library_exports_every_declared_symbol():
    lib = nv.load_library()
    names = declared_functions()
    assert len(names) >= 10
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(nv.EXPORTED)


def test_last_error_and_bad_args_without_gpu():
    lib = nv.load_library()
    buf = C.create_string_buffer(64)
    assert lib.mace_last_error(buf, 64) == nv.MACE_OK
    assert lib.mace_ctx_create(None, 0, None) == nv.MACE_ERR_BAD_ARG
    assert "null" in nv.last_error(lib)
    assert lib.mace_forward_backward(None, None, None, 0, None) == nv.MACE_ERR_BAD_ARG


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc not available")
def test_struct_layout_matches_header(tmp_path):
    structs = {"Slots": "mace_slots", "ConvSlot": "mace_conv_slot", "LinGroup": "mace_lin_group",
               "ScOut": "mace_sc_out", "LayerDesc": "mace_layer_desc", "ModelDesc": "mace_model_desc",
               "System": "mace_system", "Outputs": "mace_outputs"}
    fields = [("ModelDesc", "mace_model_desc", "layers"), ("ModelDesc", "mace_model_desc", "floats"),
              ("ModelDesc", "mace_model_desc", "n_ints"), ("LayerDesc", "mace_layer_desc", "conv"),
              ("LayerDesc", "mace_layer_desc", "sc"), ("LayerDesc", "mace_layer_desc", "f_ro2"),
              ("LayerDesc", "mace_layer_desc", "mlp_w"), ("ScOut", "mace_sc_out", "f_G"),
              ("LayerDesc", "mace_layer_desc", "density"), ("LayerDesc", "mace_layer_desc", "f_density"),
              ("ModelDesc", "mace_model_desc", "agnesi"), ("ModelDesc", "mace_model_desc", "f_radius_agnesi"),
              ("ModelDesc", "mace_model_desc", "zbl_a_prefactor"), ("ModelDesc", "mace_model_desc", "f_znum"),
              ("System", "mace_system", "rev")]
    src = ["#include <stdio.h>", "#include <stddef.h>", '#include "mace_b200.h"', "int main(void){"]
    for py, c in structs.items():
        src.append(f'printf("{py} %zu\\n", sizeof({c}));')
    for py, c, f in fields:
        src.append(f'printf("{py}.{f} %zu\\n", offsetof({c}, {f}));')
    src.append("return 0;}")
    (tmp_path / "l.c").write_text("\n".join(src))
    subprocess.run(["gcc", f"-I{ROOT / 'include'}", str(tmp_path / "l.c"), "-o", str(tmp_path / "l")], check=True)
    got = dict(line.split() for line in subprocess.run([str(tmp_path / "l")], capture_output=True, text=True,
                                                         check=True).stdout.splitlines())
    for py in structs:
        assert C.sizeof(getattr(nv, py)) == int(got[py]), py
    for py, _, f in fields:
        name = "in_" if f == "in" else f
        assert getattr(getattr(nv, py), name).offset == int(got[f"{py}.{f}"]), f"{py}.{f}"
