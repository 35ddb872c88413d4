"""The C++ host mirror (emel.rs_b200/cpp/emel_kernels_cuda.hpp): it compiles
and links against the device library on any machine; on a GPU its tests --
restated from the reference's unit tests -- pass."""

import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
BIN = ROOT / "tests" / "cpp" / "test_kernel_events"


def build_binary(emel):
    emel.lib()  # the shared library exists
    cmd = ["g++", "-std=c++17", "-O1", "-Wall", "-I", str(ROOT / "include"), "-I", str(ROOT / "emel.rs_b200" / "cpp"),
           str(ROOT / "tests" / "cpp" / "test_kernel_events.cpp"), "-o", str(BIN), "-L", str(ROOT / "emel.rs_b200"),
           "-lemel_cuda", f"-Wl,-rpath,{ROOT / 'emel.rs_b200'}"]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return BIN


def test_cpp_mirror_compiles_and_links(emel):
    assert build_binary(emel).exists()


@pytest.mark.gpu
def test_cpp_mirror_reference_known_answers_on_device(emel):
    b = build_binary(emel)
    out = subprocess.run([str(b)], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stdout + out.stderr
    assert "ok: 0 failure(s)" in out.stdout
