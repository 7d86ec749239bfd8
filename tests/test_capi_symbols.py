"""The C-ABI library loads on a CPU-only box and exports every entry point
that ``include/hcp_ring.h`` declares (no compute calls without a GPU)."""

import os
import re

from hcp_vllm_plugin_b200 import _capi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    names = set()
    for fn in os.listdir(os.path.join(ROOT, "include")):
        if fn.endswith(".h"):
            src = open(os.path.join(ROOT, "include", fn)).read()
            src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
            names |= set(re.findall(r"^\s*(?:int64_t|int|const char\*|void)\s+(hcp_\w+)\s*\(", src, flags=re.M))
    return names


def test_library_exports_every_declared_symbol():
    lib = _capi.load()
    declared = _declared()
    assert declared, "no declarations parsed"
    for name in declared:
        assert hasattr(lib, name), f"{name} declared but not exported"
    assert declared == set(_capi.SIGNATURES), "ctypes signatures out of sync with the header"
    assert b"sm_100a" in lib.hcp_version()


def test_struct_layout_matches_header():
    # hcp_attn_work is 12 int32; hcp_fwd_args layout is fixed by the header
    import ctypes
    assert ctypes.sizeof(_capi.HcpAttnWork) == 48
    assert _capi.HcpFwdArgs.q.offset == 24
    assert _capi.HcpFwdArgs.work.offset % 8 == 0
