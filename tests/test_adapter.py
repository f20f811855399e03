"""CPU: the reference-side adapter (matcoredsl_b200/integration/
closed_cuda_candidate_mcb.cpp) compiled against the reference's own headers
and linked against the real libmcb.so, with the library's CUDA runtime calls
replaced by fakes (mcb_test_set_runtime_hooks_v1).

Modelled on the reference's fake-driver adapter test
(compiler/tests/generated_gpu/cuda_adapter_test.cpp): the binary is run once
per injected failure, for every call the successful run makes, and checks
that the adapter returns a failure Code, leaves E untouched, keeps the
caller's errno and FP environment, runs no library call on the caller's
thread, and after a candidate failure (uncertain completion, including an
expired device-side wait) is poisoned and makes no further library call;
after any other failure the same call succeeds. The reference's headers are
read from MCB_REFERENCE_DIR or a `reference` directory beside this
repository; without them the test is skipped.
"""
import os
import re
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.environ.get("MCB_REFERENCE_DIR", os.path.join(os.path.dirname(ROOT), "reference"))
RUNTIME_H = os.path.join(REF, "compiler", "lib", "runtime", "closed_cuda_candidate_v1.h")


@pytest.fixture(scope="module")
def adapter_binary(tmp_path_factory, mcb):
    if not os.path.exists(RUNTIME_H):
        pytest.skip("MatcoreDSL headers not present (set MCB_REFERENCE_DIR)")
    cxx = shutil.which("g++")
    if not cxx:
        pytest.skip("no C++ compiler")
    from matcoredsl_b200 import _abi
    libdir = os.path.dirname(_abi.LIB_PATH)
    out = str(tmp_path_factory.mktemp("adapter") / "adapter_fault_test")
    cmd = [cxx, "-std=c++20", "-O1", "-ffp-contract=off", "-pthread", "-Wall",
           "-I", os.path.join(REF, "compiler", "include"),
           "-I", os.path.join(REF, "compiler", "lib", "runtime"),
           "-I", os.path.join(ROOT, "include"),
           os.path.join(ROOT, "matcoredsl_b200", "integration", "closed_cuda_candidate_mcb.cpp"),
           os.path.join(ROOT, "tests", "adapter", "adapter_fault_test.cpp"),
           "-L", libdir, "-lmcb", f"-Wl,-rpath,{libdir}", "-o", out]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return out


def _run(binary, mode):
    r = subprocess.run([binary, mode], capture_output=True, text=True, timeout=60)
    return r.returncode, r.stdout + r.stderr


def test_adapter_success_and_call_count(adapter_binary):
    rc, out = _run(adapter_binary, "count")
    assert rc == 0 and "PASS" in out, out
    assert int(re.search(r"calls=(\d+)", out).group(1)) >= 10


def test_adapter_every_injected_failure(adapter_binary):
    _, out = _run(adapter_binary, "count")
    n = int(re.search(r"calls=(\d+)", out).group(1))
    codes = set()
    for k in range(1, n + 1):
        rc, out = _run(adapter_binary, str(k))
        assert rc == 0 and "PASS" in out, (k, rc, out)
        codes.add(int(re.search(r"code=(\d+)", out).group(1)))
    # Code::allocation_failure (8), candidate_failure (9), candidate_unavailable (14)
    assert {8, 9, 14} <= codes, codes


@pytest.mark.parametrize("mode", ["timeout", "gemm", "zero-N", "real"])
def test_adapter_modes(adapter_binary, mode):
    rc, out = _run(adapter_binary, mode)
    assert rc == 0 and "PASS" in out, (mode, rc, out)
