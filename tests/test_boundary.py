"""The C ABI pinned to the reference's own headers at compile time.

Compiles tests/boundary/pin.cpp with g++ -std=c++23 against the reference
checkout: every field of fz_step's head sits at the offset and has the size of
kernels::Step's (src/core/kernels/interface.h:163-185), and fz_record is
sampler::SampledRecord (src/core/sampler/sampler.h:187-193).  Then compiles
the CudaProgram adapter that INTEGRATION.md shows a Frizzle maintainer would
add, against include/frizzle_b200.h and the reference's interface.h (with a
stand-in for program.h, whose WebGPU include is not present here).

The reference checkout comes from FRIZZLE_REFERENCE or the path BASELINE.json
records; without it (as on a GPU box) these tests skip."""
import os
import re
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HERE = os.path.join(ROOT, "tests", "boundary")


def _reference():
    import sys
    sys.path.insert(0, ROOT)
    import __graft_entry__
    ref = __graft_entry__.reference_checkout()
    if not ref or not os.path.exists(os.path.join(ref, "src", "core", "kernels", "interface.h")):
        pytest.skip("the reference checkout is not present")
    if not shutil.which("g++"):
        pytest.skip("g++ is not present")
    return ref


def _compile(src, ref, tmp_path, extra_includes=()):
    out = str(tmp_path / (os.path.basename(src) + ".o"))
    cmd = ["g++", "-std=c++23", "-fsyntax-only" if src.endswith(".h") else "-c", "-Wall", "-Werror",
           *[f"-I{d}" for d in extra_includes], f"-I{os.path.join(ROOT, 'include')}",
           f"-I{os.path.join(ref, 'src')}", f"-I{ref}", src, "-o", out]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-4000:]


def test_step_and_record_match_the_reference_headers(tmp_path):
    ref = _reference()
    _compile(os.path.join(HERE, "pin.cpp"), ref, tmp_path)


def test_integration_adapter_compiles(tmp_path):
    ref = _reference()
    text = open(os.path.join(ROOT, "INTEGRATION.md")).read()
    blocks = re.findall(r"```cpp\n(.*?)```", text, flags=re.S)
    adapter = next(b for b in blocks if "class CudaProgram" in b)
    src = tmp_path / "cuda_program.cpp"
    src.write_text("#include <memory>\n#include <string>\n" + adapter)
    _compile(str(src), ref, tmp_path, extra_includes=[os.path.join(HERE, "stub")])
