"""include/qg_compat.hpp, the reference's C++ class API (include/qg.hpp) over
libflashgann.so, without a GPU: a program of our own compiles against it and
links the library, and the constructor's failures take the reference's form
(std::runtime_error, "Cannot open codebook file: <path>" for a missing file)
before any device is touched.  The reference's own main.cu is built against
the header and run on a GPU in tests/test_gpu_cli.py."""

from __future__ import annotations

import os
import shutil
import subprocess

import pytest

from tests.common import ROOT

PROGRAM = r'''
#include <cstdio>
#include <stdexcept>
#include "qg_compat.hpp"

int main(int argc, char** argv) {
    for (int i = 1; i < argc; ++i) {
        try {
            QuantizationGraph qg(1000, 128, 32, argv[i]);
            printf("constructed\n");
        } catch (const std::runtime_error& e) {
            printf("runtime_error: %s\n", e.what());
        }
    }
    static_assert(sizeof(vidType) == 4, "vidType");
    static_assert(METRIC_L2 == 0 && METRIC_IP == 1, "MetricType");
    return 0;
}
'''


def test_class_header_compiles_links_and_throws_like_the_reference(tmp_path):
    lib = os.path.join(ROOT, "flashgann_b200", "libflashgann.so")
    if not os.path.exists(lib):
        pytest.fail("libflashgann.so is not built (make lib)")
    cxx = shutil.which("g++") or shutil.which("c++")
    src = tmp_path / "prog.cpp"
    src.write_text(PROGRAM)
    exe = tmp_path / "prog"
    subprocess.run([cxx, "-std=c++17", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe),
                    "-L", os.path.dirname(lib), "-lflashgann", f"-Wl,-rpath,{os.path.dirname(lib)}"], check=True)
    short = tmp_path / "short.index"
    short.write_bytes(b"\0" * 64)
    missing = tmp_path / "missing.index"
    r = subprocess.run([str(exe), str(missing), str(short)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stderr
    lines = r.stdout.splitlines()
    assert lines[0] == f"runtime_error: Cannot open codebook file: {missing}"
    assert lines[1].startswith("runtime_error: fg_index_load: ") and "needs" in lines[1]
