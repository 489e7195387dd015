"""CPU checks of the C ABI library: it loads and exports what the header
declares.  No compute call is made here (there is no GPU)."""
import os
import re
import subprocess

import pytest
import torch

from qmoe_b200 import capi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    src = open(capi.HEADER_PATH).read()
    return sorted(set(re.findall(r"QMOE_API\s+[\w\s\*]*?\b(qmoe_\w+)\s*\(", src)))


def test_header_declares_entry_points():
    names = header_functions()
    assert "qmoe_layer_forward" in names and "qmoe_packed_forward" in names
    assert len(names) >= 17


def test_library_exports_every_header_symbol():
    lib = capi.lib()
    for name in header_functions():
        assert hasattr(lib, name), name


def test_binding_covers_header_exactly():
    assert sorted(capi.SIGNATURES) == header_functions()


def test_exported_symbols_are_only_the_abi():
    out = subprocess.run(["nm", "-D", "--defined-only", capi.LIB_PATH],
                         capture_output=True, text=True, check=True).stdout
    exported = sorted({l.split()[-1] for l in out.splitlines()
                       if l.split()[1:2] == ["T"] and l.split()[-1].startswith("qmoe_")})
    assert exported == header_functions()


def test_library_is_sm100a_only():
    # the fat binary carries sm_100a code only (cuobjdump lists the ELF arch;
    # its listing of architectures is tool output, not disassembly)
    out = subprocess.run(["/usr/local/cuda/bin/cuobjdump", "--list-elf", capi.LIB_PATH],
                         capture_output=True, text=True)
    if out.returncode != 0:
        pytest.skip("cuobjdump unavailable")
    arches = set(re.findall(r"sm_\d+a?", out.stdout))
    assert arches == {"sm_100a"}, arches


def test_abi_version():
    assert capi.lib().qmoe_abi_version() == 1


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU error path")
def test_context_without_gpu_fails_cleanly():
    from qmoe_b200 import Context, QmoeError
    with pytest.raises(QmoeError) as ei:
        Context(0)
    assert ei.value.code == capi.QMOE_ERR_CUDA


def test_package_never_imports_oracle():
    pkg = os.path.join(ROOT, "qmoe-rs_b200")
    for dirpath, _, files in os.walk(pkg):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".h", ".cpp", ".hpp")):
                text = open(os.path.join(dirpath, f)).read()
                assert "import oracle" not in text and "from oracle" not in text, f
                assert "qmoe_oracle" not in text, f
