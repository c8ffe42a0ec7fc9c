"""Build the C++ control plane in-tree with g++:

* shift_b200/ft/libshift_ft.so   lighthouse + replica manager server (C API)
* shift_b200/ft/shift_lighthouse standalone lighthouse daemon

Run: ``python shift_b200/ft/native_build.py`` (also done by __graft_entry__.build).
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(os.path.dirname(HERE), "csrc", "ft")


def build(verbose: bool = False) -> None:
    lib = os.path.join(HERE, "libshift_ft.so")
    exe = os.path.join(HERE, "shift_lighthouse")
    flags = ["-O2", "-std=c++17", "-pthread", "-Wall", "-Wno-unused-result"]
    srcs = [os.path.join(SRC, "lighthouse.cpp")]
    newest = max(os.path.getmtime(p) for p in srcs + [os.path.join(SRC, "net.hpp"),
                                                      os.path.join(SRC, "lighthouse_main.cpp")])
    if not (os.path.exists(lib) and os.path.getmtime(lib) >= newest):
        subprocess.run(["g++", *flags, "-shared", "-fPIC", *srcs, "-o", lib], check=True)
    if not (os.path.exists(exe) and os.path.getmtime(exe) >= newest):
        subprocess.run(["g++", *flags, *srcs, os.path.join(SRC, "lighthouse_main.cpp"), "-o", exe], check=True)
    if verbose:
        print(lib, exe)


if __name__ == "__main__":
    build(verbose=True)
    sys.exit(0)
