"""Native (C++) tools driving this framework's engine: `capture` (hidden-state dumps) and `meter`
(bounded decode with per-call accounting). `build()` compiles them into `native_tools/bin/`."""

from __future__ import annotations

import os
import subprocess
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
BIN = os.path.join(HERE, "bin")
TOOLS = ("capture", "meter")


def build(verbose: bool = False) -> list:
    """g++ -O2 each tool against this interpreter's libpython; returns the binary paths."""
    inc = sysconfig.get_config_var("INCLUDEPY")
    libdir = sysconfig.get_config_var("LIBDIR")
    ver = sysconfig.get_config_var("LDVERSION") or sysconfig.get_python_version()
    os.makedirs(BIN, exist_ok=True)
    out = []
    for t in TOOLS:
        dst = os.path.join(BIN, t)
        cmd = ["g++", "-O2", "-std=c++17", "-Wall", f"-I{inc}", os.path.join(HERE, f"{t}.cpp"), "-o", dst,
               f"-L{libdir}", f"-Wl,-rpath,{libdir}", f"-lpython{ver}", "-ldl", "-lm"]
        if verbose:
            print(" ".join(cmd))
        subprocess.check_call(cmd)
        out.append(dst)
    return out


def tool_path(name: str) -> str:
    return os.path.join(BIN, name)
