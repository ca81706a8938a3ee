"""The C ABI library: it loads without a GPU, exports every symbol that
include/cc1d.h declares, and the ctypes mirror of each params struct has the
exact layout the C compiler gives the header.  No compute calls.  CPU only."""

from __future__ import annotations

import re
import shutil
import subprocess
from pathlib import Path

import pytest

from causal_conv1d_b200 import _lib

REPO = Path(__file__).resolve().parent.parent
HEADER = REPO / "include" / "cc1d.h"


def declared_symbols() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"CC1D_API\s+[\w\s\*]+?\b(cc1d_\w+)\s*\(", text)))


def test_header_declares_expected_entry_points():
    syms = declared_symbols()
    assert syms == sorted(_lib.SIGNATURES), syms


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared_symbols():
        assert hasattr(lib, name), f"{name} not exported by {_lib.LIB_PATH.name}"


def test_library_exports_nothing_else():
    nm = shutil.which("nm")
    if nm is None:
        pytest.skip("nm not available")
    res = subprocess.run([nm, "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True, check=True)
    exported = {ln.split()[-1] for ln in res.stdout.splitlines() if " T " in ln}
    ours = {s for s in exported if s.startswith("cc1d_")}
    assert ours == set(declared_symbols())
    # C++ internals stay hidden (-fvisibility=hidden).
    assert not any(s.startswith("_ZN4cc1d") for s in exported)


def test_version_and_abi():
    lib = _lib.load()
    assert lib.cc1d_version().decode() == "1.6.1"
    assert lib.cc1d_abi_version() == 2
    assert lib.cc1d_last_error() is not None


def test_null_params_rejected_without_gpu():
    lib = _lib.load()
    assert lib.cc1d_fwd(None, None) == _lib.CC1D_ERR_INVALID_ARGUMENT
    assert b"NULL" in lib.cc1d_last_error()
    assert lib.cc1d_update(None, None) == _lib.CC1D_ERR_INVALID_ARGUMENT


def test_width_rejected_without_gpu():
    import ctypes

    lib = _lib.load()
    p = _lib.FwdParams()
    p.dtype = 2
    p.width = 6  # fp32 supports 2..5
    assert lib.cc1d_fwd(ctypes.byref(p), None) == _lib.CC1D_ERR_UNSUPPORTED
    assert b"width must be in 2..5" in lib.cc1d_last_error()
    u = _lib.UpdateParams()
    u.dtype = 1
    u.width = 4
    u.state_len = 2
    u.batch, u.dim, u.seqlen = 1, 1, 1
    assert lib.cc1d_update(ctypes.byref(u), None) == _lib.CC1D_ERR_INVALID_ARGUMENT
    assert b"must be >=" in lib.cc1d_last_error()


def test_zero_size_calls_launch_nothing():
    import ctypes

    lib = _lib.load()
    p = _lib.FwdParams()
    p.dtype, p.width = 1, 4
    p.batch, p.dim, p.seqlen = 0, 64, 128
    assert lib.cc1d_fwd(ctypes.byref(p), None) == _lib.CC1D_OK


STRUCTS = {
    "cc1d_fwd_params": _lib.FwdParams,
    "cc1d_bwd_params": _lib.BwdParams,
    "cc1d_update_params": _lib.UpdateParams,
    "cc1d_varlen_states_params": _lib.VarlenParams,
    "cc1d_peer_reduce": _lib.PeerReduceParams,
    "cc1d_inproj_conv_params": _lib.InprojConvParams,
}


def test_ctypes_struct_layout_matches_header(tmp_path):
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    lines = ["#include <stdio.h>", "#include <stddef.h>", '#include "cc1d.h"', "int main(void) {"]
    for cname, cls in STRUCTS.items():
        lines.append(f'  printf("{cname} sizeof %zu\\n", sizeof({cname}));')
        for fname, _ in cls._fields_:
            lines.append(f'  printf("{cname} {fname} %zu\\n", offsetof({cname}, {fname}));')
    lines += ["  return 0;", "}"]
    src = tmp_path / "probe.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "probe"
    subprocess.run([cc, f"-I{REPO / 'include'}", str(src), "-o", str(exe)], check=True)
    got = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split("\n")
    c_layout = {}
    for ln in got:
        if ln.strip():
            s, f, v = ln.split()
            c_layout[(s, f)] = int(v)
    for cname, cls in STRUCTS.items():
        assert c_layout[(cname, "sizeof")] == __import__("ctypes").sizeof(cls), cname
        for fname, _ in cls._fields_:
            assert c_layout[(cname, fname)] == getattr(cls, fname).offset, f"{cname}.{fname}"
