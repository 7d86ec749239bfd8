"""The C-ABI library loads on a CPU-only box and exports every entry point
that ``include/hcp_ring.h`` declares (no compute calls without a GPU)."""

import ctypes
import os
import re

import pytest

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


def test_struct_layouts_match_the_header(tmp_path):
    """The ctypes structures have the C header's sizes and field offsets
    (compiled with the host C compiler, no GPU)."""
    import shutil
    import subprocess

    from hcp_vllm_plugin_b200 import _capi
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    checks = {
        "hcp_kv_source": (_capi.HcpKvSource, ["k", "v", "rows", "row_stride"]),
        "hcp_attn_work": (_capi.HcpAttnWork, ["q_start", "q_len", "paged_req", "lse_col", "seg"]),
        "hcp_fwd_args": (_capi.HcpFwdArgs, [n for n, _ in _capi.HcpFwdArgs._fields_]),
        "hcp_decode_seq": (_capi.HcpDecodeSeq, [n for n, _ in _capi.HcpDecodeSeq._fields_]),
        "hcp_decode_args": (_capi.HcpDecodeArgs, [n for n, _ in _capi.HcpDecodeArgs._fields_]),
    }
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "hcp_ring.h"', "int main(void) {"]
    for st, (_, fields) in checks.items():
        lines.append(f'printf("{st} %zu\\n", sizeof({st}));')
        for f in fields:
            lines.append(f'printf("{st}.{f} %zu\\n", offsetof({st}, {f}));')
    lines.append("return 0; }")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run([cc, "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    got = dict(line.split() for line in subprocess.run([str(exe)], capture_output=True, text=True,
                                                       check=True).stdout.splitlines())
    for st, (cls, fields) in checks.items():
        assert int(got[st]) == ctypes.sizeof(cls), st
        for f in fields:
            assert int(got[f"{st}.{f}"]) == getattr(cls, f).offset, f"{st}.{f}"
