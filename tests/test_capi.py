"""The C-ABI library loads here (no GPU) and exports every entry point that
include/*.h declares; host-side argument checks run before any device work.
No compute call is made without a GPU."""
import ctypes as C
import glob
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"\b(minq_\w+)\s*\(", text):
            names.add(m.group(1))
    names.discard("minq_token_cb")
    return names


def test_library_exports_every_declared_symbol(mq):
    from minq_b200 import _lib
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = {l.split()[-1] for l in out.splitlines() if " T " in l and "minq_" in l}
    declared = declared_functions()
    assert declared, "no declarations found"
    missing = declared - exported
    assert not missing, f"declared but not exported: {sorted(missing)}"
    # and the Python binding knows every one of them
    assert declared <= set(_lib.SIGNATURES), sorted(declared - set(_lib.SIGNATURES))


def test_abi_version_and_error_text(mq):
    from minq_b200 import _lib
    L = _lib.lib()
    assert L.minq_abi_version() == 1
    assert isinstance(L.minq_last_error(), bytes)


def test_host_side_shape_checks_run_before_the_device(mq):
    from minq_b200 import _lib
    L = _lib.lib()
    # quantize.rs:67-75: n % 32 != 0 is a Shape error, reported without a GPU
    assert L.minq_quantize(_lib.Q8_0, None, 17, None, None) == _lib.ERR_SHAPE
    assert b"multiple of 32" in L.minq_last_error()
    # quantize.rs:216-222: input length must equal cols
    assert L.minq_qmatvec(_lib.Q4_0, None, 4, 64, None, 63, None, None) == _lib.ERR_SHAPE
    assert b"64 cols vs input len 63" in L.minq_last_error()
    assert L.minq_quantize(7, None, 32, None, None) == _lib.ERR_FORMAT


def test_no_cpu_fallback_without_gpu(mq):
    """Without a CUDA device the model API refuses instead of computing on the CPU."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from minq_b200 import _lib
    cfg = _lib.Config()
    h = C.c_void_p()
    st = _lib.lib().minq_model_new(C.byref(cfg), C.byref(h))
    assert st == _lib.ERR_CUDA
    assert b"no CUDA device" in _lib.lib().minq_last_error()


def test_prefill_attention_argument_checks(mq):
    """minq_attend_prefill rejects unsupported shapes before touching a device."""
    from minq_b200 import _lib
    L = _lib.lib()
    d = C.c_void_p(256)  # never dereferenced: every check below comes first
    assert L.minq_attend_prefill(None, d, d, 128, 0, 4, 8, 2, 128, d, None, 0, None) == _lib.ERR_ARG
    assert L.minq_attend_prefill(d, d, d, 128, 0, 4, 7, 2, 128, d, None, 0, None) == _lib.ERR_MODEL
    assert L.minq_attend_prefill(d, d, d, 96, 0, 4, 8, 2, 96, d, None, 0, None) == _lib.ERR_SHAPE
    assert b"head_dim 96" in L.minq_last_error()
    assert L.minq_attend_prefill(d, d, d, 128, 0, 0, 8, 2, 128, d, None, 0, None) == _lib.ERR_SHAPE
    assert L.minq_attn_prefill_workspace_bytes(0, 8, 2, 128) == 0
