"""The device exponential cores (fastmath.cuh) compiled for the host.

The binary64 core (standalone tanh, attention, RoPE, silu_back): its exp /
expm1 / tanh equal binary64 libm rounded once to binary32 (the
correctly-rounded-libm oracle's definition) on a strided sweep of all
binary32 bit patterns (saturating arguments, infinities and NaNs included),
allowing at most a handful of 1-ulp ties.

The binary32 core (activations, soft_max, GLU gates): exp and expm1 within
1 ulp and tanh within 2 ulp of binary64 libm rounded once, on the same kind
of sweep (a full sweep of all 2^32 inputs gives the same maxima), and the
reference's GELU built on it within one binary16 step of the same formula
on glibc's tanhf for every binary16 input."""

import subprocess
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def test_fast_exponential_core_matches_binary64_libm(tmp_path):
    exe = tmp_path / "fastmath_check"
    subprocess.run(["g++", "-O2", "-std=c++17", "-ffp-contract=off", "-I", str(ROOT / "emel.rs_b200" / "csrc"),
                    str(ROOT / "tests" / "cpp" / "fastmath_check.cpp"), "-o", str(exe), "-lm"], check=True)
    out = subprocess.run([str(exe), "1009"], capture_output=True, text=True, check=True).stdout.split()
    # plus every binary32 in the windows around the saturation thresholds
    edge = subprocess.run([str(exe), "edges"], capture_output=True, text=True, check=True).stdout.split()
    n_e, e_exp, e_expm1, e_tanh, worst_e = map(int, edge)
    assert n_e > 1_000_000
    assert e_exp <= 2 and e_expm1 <= 2 and e_tanh <= 2 and worst_e <= 1, edge
    n, d_exp, d_expm1, d_tanh, worst = map(int, out)
    assert n > 1_000_000
    assert d_exp <= 2 and d_expm1 <= 2 and d_tanh <= 2, out
    assert worst <= 1, out


def build_checker(tmp_path):
    exe = tmp_path / "fastmath_check"
    subprocess.run(["g++", "-O2", "-std=c++17", "-ffp-contract=off", "-I", str(ROOT / "emel.rs_b200" / "csrc"),
                    str(ROOT / "tests" / "cpp" / "fastmath_check.cpp"), "-o", str(exe), "-lm"], check=True)
    return exe


def test_binary32_exponential_core_error_bounds(tmp_path):
    exe = build_checker(tmp_path)
    out = subprocess.run([str(exe), "b32", "131"], capture_output=True, text=True, check=True).stdout.split()
    n, u_exp, u_expm1, u_tanh, nan_bad = map(int, out)
    assert n > 30_000_000
    assert u_exp <= 1 and u_expm1 <= 1 and u_tanh <= 2 and nan_bad == 0, out


def test_gelu_on_the_binary32_tanh_within_one_binary16_step(tmp_path):
    exe = build_checker(tmp_path)
    inputs, worst = map(int, subprocess.run([str(exe), "gelu"], capture_output=True, text=True, check=True).stdout.split())
    assert inputs == 65536 - 2046 and worst <= 1, (inputs, worst)


def test_gate_exponential_keeps_sigmoid_and_silu_within_two_ulp(tmp_path):
    """sigmoid and silu on the gate exponential (exp32, and the correctly
    rounded binary64 exp where 1 + exp(-x) rounds) against the same formulas
    on binary64 exp rounded once: a strided sweep of all binary32 inputs plus
    every input of the band x in [-104, -15]."""
    exe = build_checker(tmp_path)
    n, u_sig, u_silu = map(int, subprocess.run([str(exe), "gate", "131"], capture_output=True, text=True,
                                               check=True).stdout.split())
    assert n > 40_000_000
    assert u_sig <= 2 and u_silu <= 2, (u_sig, u_silu)
