"""CPU-side checks of the C-ABI library: it loads, exports every symbol the
public header declares, and reports a missing GPU as an error (no compute
call is made without a GPU)."""
import ctypes
import os
import subprocess

import numpy as np

from aljabr_b200 import native


def test_library_exports_every_header_symbol():
    declared = native.header_symbols()
    assert len(declared) >= 20
    out = subprocess.run(["nm", "-D", "--defined-only", native.LIB_PATH], capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    missing = [s for s in declared if s not in exported]
    assert not missing, missing
    assert sorted(native.SIGNATURES) == declared


def test_library_loads_and_binds():
    L = native.lib()
    for name in native.header_symbols():
        assert getattr(L, name) is not None


def test_without_gpu_calls_fail_loudly():
    import torch
    if torch.cuda.is_available():
        return
    L = native.lib()
    assert L.aljabr_blackwell_device_count() == 0
    assert L.aljabr_blackwell_init(0) == native.ALJ_ERR_NOT_INITIALIZED
    assert "no CUDA device" in native.last_error()
    y = np.zeros(4, np.float32)
    x = np.zeros(256, np.float32)
    w = np.zeros(4 * 8 * 18, np.uint8)
    rc = L.aljabr_blackwell_matvec_tb_q4_0(y.ctypes.data, x.ctypes.data, w.ctypes.data, 256, 4)
    assert rc == native.ALJ_ERR_NOT_INITIALIZED


def test_header_compiles_as_c():
    src = '#include "aljabr_blackwell.h"\nint main(void){return ALJ_TYPE_Q4_0 == 2 ? 0 : 1;}\n'
    inc = os.path.dirname(native.HEADER_PATH)
    r = subprocess.run(["gcc", "-x", "c", "-std=c99", "-Wall", "-Werror", "-I", inc, "-fsyntax-only", "-"],
                       input=src, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
