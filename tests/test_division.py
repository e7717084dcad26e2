"""The codec's division shortcuts are exact (CPU): compiles tests/div_check.c with gcc and runs it.

The 512-value encode divides by float32(sqrt(512)) with a Brisebarre-Muller
constant multiplication and by the group scale (and the absmax by 7) with
Markstein's correction step; the generic encode uses Markstein for every
divisor.  Each must reproduce the IEEE quotient the reference computes
(quantization/kv.py:32 and kv.py:104-110) on the ranges the kernels use them.
"""
from __future__ import annotations

import math
import shutil
import subprocess
from pathlib import Path

import pytest

SRC = Path(__file__).with_name("div_check.c")


@pytest.fixture(scope="module")
def checker(tmp_path_factory):
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    exe = tmp_path_factory.mktemp("divcheck") / "div_check"
    subprocess.run([cc, "-O2", "-o", str(exe), str(SRC), "-lm"], check=True)
    return exe


def run(exe, *args) -> list[int]:
    out = subprocess.run([str(exe), *map(str, args)], check=True, capture_output=True, text=True).stdout
    return [int(v) for v in out.split()]


@pytest.mark.parametrize("n", [128, 512])
def test_markstein_and_constant_multiplication_by_sqrt_n(checker, n):
    c = repr(float(math.sqrt(n)))
    assert run(checker, "sig", c) == [0, 0]


def test_markstein_division_by_seven(checker):
    assert run(checker, "sig", 7)[0] == 0


def test_markstein_division_by_random_scales(checker):
    assert run(checker, "random", 2_000_000, 1) == [0]
