"""The C ABI as a C caller sees it: every header in include/ compiles as C11 with warnings
on, the program links against libb200attn.so, and the library's host-side entry points
return the reference's known answers (tests/c_abi/c_abi_check.c; no GPU needed)."""
import os
import shutil
import subprocess

import pytest

import b200attn

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_headers_compile_as_c_and_host_entry_points_answer(tmp_path):
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    b200attn.lib()  # builds nothing; raises if the library is missing
    libdir = os.path.dirname(b200attn.LIB_PATH)
    exe = tmp_path / "c_abi_check"
    build = subprocess.run(
        [cc, "-std=c11", "-Wall", "-Wextra", "-Werror", "-I", os.path.join(ROOT, "include"),
         os.path.join(ROOT, "tests", "c_abi", "c_abi_check.c"), "-L", libdir, "-lb200attn",
         f"-Wl,-rpath,{libdir}", "-lm", "-o", str(exe)],
        capture_output=True, text=True)
    assert build.returncode == 0, build.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert run.returncode == 0, run.stderr
    assert "c abi ok" in run.stdout


@pytest.mark.gpu
def test_attention_from_c_matches_the_c_oracle(cuda, tmp_path):
    """b200_attn_fwd called from a C program (CUDA runtime buffers, the library's host
    mirrors for layout and RoPE, the default stream) against the C oracle compiled into
    the same program: ragged prefixes, B = 2 (tests/c_abi/c_abi_gpu.c)."""
    cc = shutil.which("gcc") or shutil.which("cc")
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    if cc is None or not os.path.exists(os.path.join(cuda_home, "include", "cuda_runtime.h")):
        pytest.skip("no C compiler or CUDA runtime headers")
    b200attn.lib()
    libdir = os.path.dirname(b200attn.LIB_PATH)
    cudalib = os.path.join(cuda_home, "lib64")
    exe = tmp_path / "c_abi_gpu"
    build = subprocess.run(
        [cc, "-std=c11", "-O2", "-Wall", "-Wextra", "-Werror", "-fopenmp",
         "-I", os.path.join(ROOT, "include"), "-I", os.path.join(cuda_home, "include"),
         os.path.join(ROOT, "tests", "c_abi", "c_abi_gpu.c"),
         os.path.join(ROOT, "oracle", "cpu_attention.c"),
         "-L", libdir, "-lb200attn", "-L", cudalib, "-lcudart",
         f"-Wl,-rpath,{libdir}", f"-Wl,-rpath,{cudalib}", "-lm", "-o", str(exe)],
        capture_output=True, text=True)
    assert build.returncode == 0, build.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert run.returncode == 0, run.stdout + run.stderr
    assert "c abi gpu ok" in run.stdout
