"""The ctypes mirrors of the C ABI structs (hearth_b200/_lib.py) have the layout the header declares:
a small C program compiled against include/hearth_b200.h prints every size and field offset, and
they must equal the ctypes ones (CPU only; gcc)."""
import ctypes
import os
import shutil
import subprocess

import pytest

from hearth_b200._lib import ContainerInfo, MoeConfig, MoeStats

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
STRUCTS = {"hxb_moe_config": MoeConfig, "hxb_moe_stats": MoeStats, "hxb_container_info": ContainerInfo}


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc not available")
def test_ctypes_structs_match_the_header(tmp_path):
    lines = ["#include <stdio.h>", "#include <stddef.h>", '#include "hearth_b200.h"', "int main(void) {"]
    for cname, py in STRUCTS.items():
        lines.append(f'    printf("{cname} size %zu\\n", sizeof({cname}));')
        for field, _ in py._fields_:
            lines.append(f'    printf("{cname} {field} %zu\\n", offsetof({cname}, {field}));')
    lines += ["    return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c11", "-I", os.path.join(REPO, "include"), str(src), "-o", str(exe)], check=True)
    got = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split("\n")
    c_layout = {tuple(l.split()[:2]): int(l.split()[2]) for l in got if l}
    for cname, py in STRUCTS.items():
        assert c_layout[(cname, "size")] == ctypes.sizeof(py), cname
        for field, _ in py._fields_:
            assert c_layout[(cname, field)] == getattr(py, field).offset, f"{cname}.{field}"

