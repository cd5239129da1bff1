"""The C ABI from plain C (tests/c_abi_check.c): the header compiles as C99 and the program
links against libdory_decode.so with a C linker (CPU); on a GPU it runs its known-answer
decode and error checks through the header alone (no Python binding in the way)."""

from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
PKG = ROOT / "dory-vllm-experiments_b200"
CUDA = Path("/usr/local/cuda")


def build(tmp_path: Path) -> Path:
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("no C compiler")
    if not (PKG / "libdory_decode.so").exists():
        pytest.skip("libdory_decode.so is not built")
    exe = tmp_path / "c_abi_check"
    cmd = [gcc, "-std=c99", "-O2", "-Wall", "-Werror", str(ROOT / "tests" / "c_abi_check.c"),
           "-I", str(ROOT / "include"), "-I", str(CUDA / "include"), "-L", str(PKG),
           "-ldory_decode", "-L", str(CUDA / "lib64"), "-lcudart", "-lm",
           f"-Wl,-rpath,{PKG}", f"-Wl,-rpath,{CUDA / 'lib64'}", "-o", str(exe)]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return exe


def test_header_compiles_and_links_as_c(tmp_path):
    assert build(tmp_path).exists()


@pytest.mark.gpu
def test_c_program_known_answer(tmp_path):
    exe = build(tmp_path)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "c abi ok" in r.stdout
