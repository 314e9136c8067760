"""The reference's own sampler tests run against this library.

oracle/Makefile (target reftests) compiles the reference's
tests/test_sampling.c and tests/test_bugfixes.c unmodified, linking
libpz_sampling.so where the reference links its src/sampling objects: the
drop-in of INTEGRATION.md, checked by the reference's callers themselves.
Every sample_* / apply_temperature / rng_* call in them runs through the
library's legacy entry points and its sm_100a kernels."""
import os
import re
import subprocess

import pytest

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_BIN = os.path.join(REPO, "oracle", "_ref")
LIB = os.path.realpath(os.path.join(REPO, "project-zero_b200", "libpz_sampling.so"))


@pytest.mark.parametrize("name", ["test_sampling", "test_bugfixes"])
def test_reference_suite_runs_on_this_library(cuda, name, tmp_path):
    exe = os.path.join(REF_BIN, name)
    if not os.path.exists(exe):
        pytest.skip("built by oracle/Makefile reftests where the reference tree is present")
    ldd = subprocess.run(["ldd", exe], capture_output=True, text=True, check=True).stdout
    m = re.search(r"libpz_sampling\.so => (\S+)", ldd)
    assert m and os.path.realpath(m.group(1)) == LIB, ldd
    r = subprocess.run([exe], capture_output=True, text=True, timeout=900, cwd=tmp_path)
    out = r.stdout + r.stderr
    s = re.search(r"=== (\d+)/(\d+) tests passed(, (\d+) FAILED)? ===", out)
    assert s, out[-2000:]
    passed, run = int(s.group(1)), int(s.group(2))
    print(f"{name}: {passed}/{run} assertions passed on libpz_sampling.so")
    assert r.returncode == 0 and passed == run and run > 0, out[-2000:]
