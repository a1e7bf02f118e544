"""The C ABI from plain C: include/h3q.h compiles as C99 and C11 (gcc, -pedantic, warnings as errors), and a C11
program (tests/c/gemm_s8_capi.c) links against libh3q.so and the CUDA runtime only.  On a GPU the program runs
h3q_gemm_s8 and checks its outputs bit for bit against the C oracle (the GPU test)."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")
LIB = os.path.join(ROOT, "h3-rs_b200", "lib")
ORACLE = os.path.join(ROOT, "oracle")

pytestmark = pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc not available")


def _build(tmp_path):
    exe = tmp_path / "gemm_s8_capi"
    cmd = ["gcc", "-std=c11", "-Wall", "-Wextra", "-Werror", "-O2", "-I", os.path.join(ROOT, "include"),
           "-I", os.path.join(CUDA, "include"), os.path.join(ROOT, "tests", "c", "gemm_s8_capi.c"), "-o", str(exe),
           "-L", LIB, "-lh3q", "-L", ORACLE, "-loracle", "-L", os.path.join(CUDA, "lib64"), "-lcudart",
           f"-Wl,-rpath,{LIB}:{ORACLE}:{os.path.join(CUDA, 'lib64')}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


@pytest.mark.parametrize("std", ["c99", "c11"])
def test_header_is_plain_c(tmp_path, std):
    src = tmp_path / "h.c"
    src.write_text('#include "h3q.h"\nint main(void) { return (int)h3q_gemm_s8_workspace_size(1, 64) == 0; }\n')
    r = subprocess.run(["gcc", f"-std={std}", "-pedantic", "-Wall", "-Wextra", "-Werror", "-fsyntax-only",
                        "-I", os.path.join(ROOT, "include"), str(src)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def test_c_program_links(tmp_path):
    if not os.path.exists(os.path.join(LIB, "libh3q.so")) or not os.path.exists(os.path.join(ORACLE, "liboracle.so")):
        pytest.skip("native libraries not built")
    assert _build(tmp_path).exists()


@pytest.mark.gpu
@pytest.mark.parametrize("M,K,N", [(256, 1024, 512), (300, 5120, 768)])
def test_c_program_gemm_s8_bit_exact(tmp_path, cuda, M, K, N):
    exe = _build(tmp_path)
    r = subprocess.run([str(exe), str(M), str(K), str(N)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.startswith("ok")
