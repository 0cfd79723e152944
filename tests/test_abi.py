"""CPU tests of the C ABI: the library builds, loads, and exports what the header declares."""
import ctypes as C
import os
import re
import subprocess

import pytest

from common import ROOT

HEADER = os.path.join(ROOT, "include", "si_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"SI_API\s+[\w\s\*]+?\b(\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def libpath():
    import sib200
    if not os.path.exists(sib200.LIB_PATH):
        sib200.build()
    return sib200.LIB_PATH


def test_header_declares_the_reference_entry_points():
    syms = declared_symbols()
    for name in ("quantize_q8", "matvec_q4q8", "si_ref_run_layer", "si_decode_step",
                 "si_prefill", "si_matmul_dev"):
        assert name in syms
    text = open(HEADER).read()
    for inline in ("rmsnorm", "rope", "attention_compute", "run_layer", "load_layer"):
        assert re.search(rf"static inline [\w\s\*]+\b{inline}\s*\(", text), inline


def test_library_exports_every_declared_symbol(libpath):
    out = subprocess.run(["nm", "-D", "--defined-only", libpath], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    missing = [s for s in declared_symbols() if s not in exported]
    assert not missing, f"declared but not exported: {missing}"


def test_library_loads_and_reports_status_strings(libpath):
    import sib200
    L = sib200.lib()
    assert L.si_status_str(0) == b"ok"
    assert L.si_status_str(4) == b"no sm_100 CUDA device"


def test_header_compiles_as_c(tmp_path):
    src = tmp_path / "t.c"
    src.write_text('#include "si_b200.h"\nint main(void){ block_q8_0 b; (void)b;'
                   ' return (int)sizeof(block_q8_0) - 34; }\n')
    exe = tmp_path / "t"
    subprocess.run(["gcc", "-std=c11", "-Wall", "-Werror", f"-I{ROOT}/include", str(src), "-o",
                    str(exe)], check=True)
    assert subprocess.run([str(exe)]).returncode == 0


def test_no_device_is_a_clean_error(libpath):
    """Without a visible sm_100 device, context creation fails with a status, no fallback."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is visible")
    import sib200
    L = sib200.lib()
    h = C.c_void_p()
    st = L.si_ctx_create(0, 128, 1e6, 128, C.byref(h))
    assert st == 4 and not h.value
