"""The C ABI: the shared library loads without a GPU, exports every entry point include/isaac_net_b200.h declares,
and the ctypes mirror of every structure has the C layout (sizes and field offsets compiled from the header)."""
import ctypes
import importlib
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "isaac_net_b200.h")
nat = importlib.import_module("isaac-net_b200._native")


def _declared():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*int\s+(inb_\w+)\s*\(", src, re.M)))


def test_header_declares_the_exports():
    assert _declared() == sorted(nat.EXPORTS)


def test_library_loads_and_exports_every_symbol():
    L = nat.lib()
    for name in _declared():
        assert hasattr(L, name), name
    assert L.inb_abi_version() == nat.ABI_VERSION


STRUCTS = {"InbState": nat.InbState, "InbOutputs": nat.InbOutputs, "InbArrivals": nat.InbArrivals,
           "InbTables": nat.InbTables, "InbParams": nat.InbParams, "InbStepArgs": nat.InbStepArgs,
           "InbResetArgs": nat.InbResetArgs, "InbTrafficSource": nat.InbTrafficSource,
           "InbTrafficArgs": nat.InbTrafficArgs, "InbRadio": nat.InbRadio, "InbObsArgs": nat.InbObsArgs}


def _c_layout(tmp_path):
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "isaac_net_b200.h"', "int main(void) {"]
    for cname, cls in STRUCTS.items():
        lines.append(f'  printf("{cname} size %zu\\n", sizeof({cname}));')
        for f, _ in cls._fields_:
            lines.append(f'  printf("{cname}.{f} %zu\\n", offsetof({cname}, {f}));')
    lines += ["  return 0;", "}"]
    c = tmp_path / "layout.c"
    c.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", os.path.dirname(HEADER), str(c), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout
    return dict(l.rsplit(" ", 1) for l in out.strip().splitlines())


def test_struct_layouts_match_the_header(tmp_path):
    got = _c_layout(tmp_path)
    for cname, cls in STRUCTS.items():
        assert int(got[f"{cname} size"]) == ctypes.sizeof(cls), cname
        for f, _ in cls._fields_:
            assert int(got[f"{cname}.{f}"]) == getattr(cls, f).offset, f"{cname}.{f}"
