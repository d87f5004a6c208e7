"""CPU checks of the C-ABI library: it loads without a GPU, exports exactly the entry points
include/gyro_moe.h declares, and its struct layouts match the C compiler's."""
import re
import subprocess
from pathlib import Path

import pytest

from gyro_moe import abi, build

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "gyro_moe.h"


@pytest.fixture(scope="module")
def lib():
    build.build()
    return abi.load()


def declared():
    return sorted(set(re.findall(r"GX_API\s+gx_result\s+(gx_\w+)\s*\(", HEADER.read_text())))


def test_header_declares_the_binding(lib):
    assert declared() == sorted(abi.SIGNATURES)


def test_library_exports_every_declared_symbol(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", str(abi.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    exported = sorted(set(re.findall(r"\sT\s(gx_\w+)$", out, flags=re.M)))
    assert exported == declared()
    for name in declared():
        assert getattr(lib, name) is not None


def test_struct_layouts_match_c(tmp_path):
    src = tmp_path / "sz.c"
    src.write_text('#include "gyro_moe.h"\n#include <stdio.h>\n#include <stddef.h>\n'
                   'int main(void){printf("%zu %zu %zu %zu %zu %zu %zu %zu\\n", sizeof(gx_options), sizeof(gx_caps),'
                   ' sizeof(gx_layer_desc), sizeof(gx_timings), offsetof(gx_options, nccl_id),'
                   ' offsetof(gx_layer_desc, router), sizeof(gx_shared_desc), offsetof(gx_shared_desc, gate_inp));'
                   'printf("%zu %zu %zu\\n", sizeof(gx_gguf_layer_info), sizeof(gx_hc_desc),'
                   ' offsetof(gx_hc_desc, down_bytes));return 0;}\n')
    exe = tmp_path / "sz"
    subprocess.run(["gcc", "-I", str(ROOT / "include"), str(src), "-o", str(exe)], check=True)
    sizes = [int(v) for v in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    import ctypes
    assert sizes == [ctypes.sizeof(abi.Options), ctypes.sizeof(abi.Caps), ctypes.sizeof(abi.LayerDesc),
                     ctypes.sizeof(abi.Timings), abi.Options.nccl_id.offset, abi.LayerDesc.router.offset,
                     ctypes.sizeof(abi.SharedDesc), abi.SharedDesc.gate_inp.offset, ctypes.sizeof(abi.GgufLayerInfo),
                     ctypes.sizeof(abi.HcDesc), abi.HcDesc.down_bytes.offset]


def test_create_rejects_bad_options_without_touching_a_device(lib):
    import ctypes
    opts = abi.Options(0, 0, 1, 16, 1, 0, None, 8192)  # no codebook
    h = ctypes.c_void_p()
    assert lib.gx_create(ctypes.byref(opts), ctypes.byref(h)) == -1
    table = ctypes.create_string_buffer(8192)
    opts = abi.Options(0, 0, 1, 16, 1, 0, ctypes.cast(table, ctypes.c_void_p), 4096)  # wrong codebook size
    assert lib.gx_create(ctypes.byref(opts), ctypes.byref(h)) == -1
    opts = abi.Options(0, 2, 2, 16, 1, 0, ctypes.cast(table, ctypes.c_void_p), 8192)  # rank >= world
    assert lib.gx_create(ctypes.byref(opts), ctypes.byref(h)) == -1
    assert lib.gx_destroy(None, 0) == -1
    assert lib.gx_wait(None, 1, 0) == -1
