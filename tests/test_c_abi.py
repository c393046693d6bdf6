"""The C ABI from plain C (no GPU): both public headers compile as pedantic C11 and as C++17,
and a C program linked against libmsgl.so drives the host-side entry points (prefix cache,
checkpoint index, last-error string) -- what a cgo / JNI / ctypes binding of the reference's
host code would see."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INC = os.path.join(ROOT, "include")
LIBDIR = os.path.join(ROOT, "mini-sglang-cpp_b200")

PROGRAM = r"""
#include <stdio.h>
#include <string.h>
#include "msgl_kernels.h"
#include "msgl_engine.h"
int main(void) {
    msgl_radix* r = 0;
    if (msgl_radix_create(2, &r) != MSGL_OK) return 1;
    int32_t tok[6] = {1, 1, 2, 2, 3, 3}, pages[3] = {7, 8, 9}, out[3] = {0, 0, 0};
    int present = -1, nd = -1, m = -1;
    int64_t node = -1;
    if (msgl_radix_insert(r, tok, 6, pages, &present, 0, &nd, &node) != MSGL_OK) return 2;
    if (msgl_radix_match(r, tok, 5, out, 3, &m, &node) != MSGL_OK) return 3;  /* 2 whole pages */
    if (present != 0 || nd != 0 || m != 4 || out[0] != 7 || out[1] != 8) return 4;
    if (msgl_radix_lock(r, node, -1) != MSGL_ERR_INVALID_ARG) return 5;  /* never locked */
    msgl_radix_destroy(r);
    int64_t n = 0, b = 0;
    if (msgl_safetensors_index("/nonexistent-dir", &n, &b) != MSGL_ERR_INVALID_ARG) return 6;
    if (!strstr(msgl_last_error(), "cannot open model directory")) return 7;
    printf("ok\n");
    return 0;
}
"""


def _need(tool):
    if not shutil.which(tool):
        pytest.skip(f"{tool} not available")


def test_headers_compile_as_c_and_cxx(tmp_path):
    _need("gcc")
    _need("g++")
    src = tmp_path / "h.c"
    src.write_text('#include "msgl_kernels.h"\n#include "msgl_engine.h"\nint main(void){return 0;}\n')
    for cmd in (["gcc", "-std=c11", "-Wall", "-Wextra", "-pedantic", "-Werror"],
                ["g++", "-std=c++17", "-Wall", "-Wextra", "-Werror", "-x", "c++"]):
        r = subprocess.run(cmd + ["-I" + INC, "-c", str(src), "-o", str(tmp_path / "h.o")],
                           capture_output=True, text=True)
        assert r.returncode == 0, r.stderr


def test_c_program_uses_the_host_entry_points(tmp_path):
    _need("gcc")
    import msgl
    msgl.lib()  # builds / locates libmsgl.so
    src, exe = tmp_path / "t.c", tmp_path / "t"
    src.write_text(PROGRAM)
    r = subprocess.run(["gcc", "-std=c11", "-I" + INC, str(src), "-o", str(exe), "-L" + LIBDIR,
                        "-lmsgl", "-Wl,-rpath," + LIBDIR], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0 and r.stdout.strip() == "ok", (r.returncode, r.stdout, r.stderr)
