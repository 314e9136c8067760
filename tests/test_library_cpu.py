"""CPU-side checks of the product library: it loads, exports every symbol the
C header declares, and its host-only pieces (RNG word arithmetic, row
sharding, status strings) behave.  No kernel is launched here."""
import ctypes
import os
import re

import numpy as np

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(REPO, "project-zero_b200", "libpz_sampling.so")


def _declared_functions():
    names = set()
    for fn in os.listdir(os.path.join(REPO, "include")):
        if not fn.endswith(".h"):
            continue
        text = open(os.path.join(REPO, "include", fn)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        text = re.sub(r"//[^\n]*", "", text)
        for m in re.finditer(r"^\s*(?:const\s+)?(?:unsigned\s+|struct\s+)?[A-Za-z_]\w*[\s\*]+([A-Za-z_]\w*)\s*\(",
                             text, flags=re.M):
            if m.group(1) not in ("if", "while", "for", "return", "sizeof"):
                names.add(m.group(1))
    return sorted(names)


def test_library_exports_every_declared_symbol():
    assert os.path.exists(LIB), "build with make -C project-zero_b200"
    lib = ctypes.CDLL(LIB)
    names = _declared_functions()
    assert "pz_sample_batch" in names and "sample_top_p" in names and len(names) >= 25
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_python_module_imports_and_reports():
    import pz_sampling
    assert "sm_100a" in pz_sampling.version()
    assert pz_sampling.library_path() == LIB


def test_host_rng_matches_reference_known_answers(golden):
    import pz_sampling
    for seed, rec in golden["legacy"]["rng"].items():
        s = pz_sampling.rng_seed(int(seed))
        for bits in rec["float_bits"]:
            v, s = pz_sampling.rng_float(s)
            assert int(np.float32(v).view(np.uint32)) == bits
        assert s == rec["final"]
    v, _ = pz_sampling.rng_float(golden["legacy"]["rng_one_state"])
    assert v == 1.0


def test_row_shard_partitions_rows():
    import pz_sampling
    for B in [0, 1, 7, 1024, 8192, 8193]:
        for world in [1, 2, 3, 4, 8]:
            spans = [pz_sampling.row_shard(B, world, r) for r in range(world)]
            assert spans[0][0] == 0
            for (b0, c0), (b1, _) in zip(spans, spans[1:]):
                assert b0 + c0 == b1
            assert sum(c for _, c in spans) == B
            assert max(c for _, c in spans) - min(c for _, c in spans) <= 1


def test_status_strings():
    lib = ctypes.CDLL(LIB)
    lib.pz_status_str.restype = ctypes.c_char_p
    for s in range(8):
        assert lib.pz_status_str(s)


def test_no_silent_cpu_path_without_gpu():
    """Without a usable GPU the context refuses (no CPU fallback)."""
    import torch
    if torch.cuda.is_available():
        return
    import pz_sampling
    try:
        pz_sampling.Sampler(0, 4, 1000, 8, 0)
    except pz_sampling.PZError as e:
        assert e.status in (2, 7)
    else:
        raise AssertionError("context created without a GPU")
