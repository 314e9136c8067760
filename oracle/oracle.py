"""ctypes bindings of the CPU checker — TEST INFRASTRUCTURE ONLY.

Two libraries, both built by ``oracle/Makefile``:

* ``libpzoracle.so`` — the C restatement of Project Zero's sampler plus the
  pipeline contract (``pz_oracle.c``).
* ``_ref/libpzref.so`` — the reference's OWN sampler sources
  (src/sampling/*.c, src/math/softmax*.c) compiled unmodified with
  ``ref_pipeline.c`` as driver.  Built only where the reference tree exists;
  the built file travels with the repository snapshot.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg may
import this module, and only to check or time the CPU path.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
# The reference checkout: PZ_REFERENCE, else a directory named `reference`
# beside this repository.
REFERENCE_DIR = os.environ.get("PZ_REFERENCE") or os.path.join(
    os.path.dirname(os.path.dirname(HERE)), "reference")
ORACLE_SO = os.path.join(HERE, "libpzoracle.so")
REF_DIR = os.path.join(HERE, "_ref")

_i32p = ctypes.POINTER(ctypes.c_int32)
_u64p = ctypes.POINTER(ctypes.c_uint64)
_f32p = ctypes.POINTER(ctypes.c_float)


class SamplerConfig(ctypes.Structure):
    """Mirror of ``pz_sampler_config`` (include/pz_sampling.h), 32 bytes."""

    _fields_ = [
        ("temperature", ctypes.c_float),
        ("top_k", ctypes.c_int32),
        ("top_p", ctypes.c_float),
        ("repetition_penalty", ctypes.c_float),
        ("frequency_penalty", ctypes.c_float),
        ("presence_penalty", ctypes.c_float),
        ("flags", ctypes.c_uint32),
        ("reserved", ctypes.c_uint32),
    ]


CONFIG_DTYPE = np.dtype(
    [
        ("temperature", "<f4"),
        ("top_k", "<i4"),
        ("top_p", "<f4"),
        ("repetition_penalty", "<f4"),
        ("frequency_penalty", "<f4"),
        ("presence_penalty", "<f4"),
        ("flags", "<u4"),
        ("reserved", "<u4"),
    ]
)
assert CONFIG_DTYPE.itemsize == 32


def make_configs(B, temperature=1.0, top_k=0, top_p=1.0, rep=1.0, freq=0.0,
                 pres=0.0, flags=0):
    """Structured array of B configs; scalars broadcast, arrays per row."""
    c = np.zeros(B, dtype=CONFIG_DTYPE)
    c["temperature"] = temperature
    c["top_k"] = top_k
    c["top_p"] = top_p
    c["repetition_penalty"] = rep
    c["frequency_penalty"] = freq
    c["presence_penalty"] = pres
    c["flags"] = flags
    return c


def build(ref: bool = True) -> None:
    """Builds the restatement (always) and the reference library (when the
    reference tree is present)."""
    targets = ["oracle"]
    if ref and os.path.isdir(REFERENCE_DIR):
        targets.append("ref")
    subprocess.run(["make", "-s", "-C", HERE, f"PZ_REFERENCE={REFERENCE_DIR}"] + targets, check=True)


def _ptr(a, t):
    return a.ctypes.data_as(t) if a is not None else None


def _cpu_has_avx512() -> bool:
    try:
        with open("/proc/cpuinfo") as f:
            flags = f.read()
        return all(x in flags for x in ("avx512f", "avx512bw", "avx512dq",
                                          "avx512vl", "avx512cd"))
    except OSError:
        return False


class _Lib:
    def __init__(self, path, prefix):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} not built (run make -C oracle)")
        self.path = path
        self.lib = ctypes.CDLL(path)
        self.p = prefix
        L, p = self.lib, prefix
        getattr(L, p + "rng_seed").argtypes = [_u64p, ctypes.c_uint64]
        getattr(L, p + "rng_float").argtypes = [_u64p]
        getattr(L, p + "rng_float").restype = ctypes.c_float
        getattr(L, p + "sample_argmax").argtypes = [_f32p, ctypes.c_int]
        getattr(L, p + "sample_argmax").restype = ctypes.c_int
        getattr(L, p + "sample_top_p").argtypes = [_f32p, ctypes.c_int, ctypes.c_float, _u64p]
        getattr(L, p + "sample_top_p").restype = ctypes.c_int
        getattr(L, p + "sample_top_k").argtypes = [_f32p, ctypes.c_int, ctypes.c_int, _u64p]
        getattr(L, p + "sample_top_k").restype = ctypes.c_int
        getattr(L, p + "sample_softmax").argtypes = [_f32p, ctypes.c_int, _u64p]
        getattr(L, p + "sample_softmax").restype = ctypes.c_int

    # --- the six reference calls (numpy in, python out) -------------------
    def rng_seed(self, seed):
        s = ctypes.c_uint64(0)
        getattr(self.lib, self.p + "rng_seed")(ctypes.byref(s), ctypes.c_uint64(seed))
        return s.value

    def rng_float(self, state):
        s = ctypes.c_uint64(state)
        v = getattr(self.lib, self.p + "rng_float")(ctypes.byref(s))
        return float(np.float32(v)), s.value

    def sample_argmax(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32)
        return getattr(self.lib, self.p + "sample_argmax")(_ptr(x, _f32p), x.size)

    def sample_top_p(self, x, p, state):
        x = np.array(x, dtype=np.float32, copy=True)
        s = ctypes.c_uint64(state)
        t = getattr(self.lib, self.p + "sample_top_p")(_ptr(x, _f32p), x.size, ctypes.c_float(p), ctypes.byref(s))
        return t, s.value

    def sample_top_k(self, x, k, state):
        x = np.array(x, dtype=np.float32, copy=True)
        s = ctypes.c_uint64(state)
        t = getattr(self.lib, self.p + "sample_top_k")(_ptr(x, _f32p), x.size, int(k), ctypes.byref(s))
        return t, s.value

    def sample_softmax(self, x, state):
        x = np.array(x, dtype=np.float32, copy=True)
        s = ctypes.c_uint64(state)
        t = getattr(self.lib, self.p + "sample_softmax")(_ptr(x, _f32p), x.size, ctypes.byref(s))
        return t, s.value, x


class Oracle(_Lib):
    """The C restatement (libpzoracle.so)."""

    def __init__(self, path=ORACLE_SO):
        super().__init__(path, "pzo_")
        L = self.lib
        L.pzo_apply_temperature.argtypes = [_f32p, ctypes.c_int, ctypes.c_float, ctypes.c_int]
        L.pzo_apply_penalties.argtypes = [_f32p, ctypes.c_int, _i32p, ctypes.c_int,
                                          ctypes.c_float, ctypes.c_float, ctypes.c_float]
        L.pzo_sample_batch.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                       ctypes.c_int64, ctypes.c_void_p, _i32p, _i32p, _u64p, _i32p,
                                       _i32p, _f32p, _i32p, ctypes.c_int]
        L.pzo_sample_batch.restype = ctypes.c_int
        L.pzo_row_trace.argtypes = [_f32p, ctypes.c_int, ctypes.c_void_p, _i32p, ctypes.c_int, ctypes.c_uint64,
                                    _f32p, _i32p, _f32p, ctypes.POINTER(ctypes.c_int),
                                    ctypes.POINTER(ctypes.c_int32)]
        L.pzo_row_trace.restype = ctypes.c_int

    def apply_temperature(self, x, T, divide=False):
        x = np.array(x, dtype=np.float32, copy=True)
        self.lib.pzo_apply_temperature(_ptr(x, _f32p), x.size, ctypes.c_float(T), int(divide))
        return x

    def apply_penalties(self, x, hist, rep, freq, pres):
        x = np.array(x, dtype=np.float32, copy=True)
        h = np.ascontiguousarray(hist, dtype=np.int32)
        self.lib.pzo_apply_penalties(_ptr(x, _f32p), x.size, _ptr(h, _i32p), h.size,
                                     ctypes.c_float(rep), ctypes.c_float(freq), ctypes.c_float(pres))
        return x

    def row_trace(self, row, cfg_row, rng, hist=None):
        """The draw of one pipeline row, traced (pzo_row_trace): returns
        (token, r, order, cdf, fallback) where order/cdf are the walk's ids
        and running float CDF (empty when the row draws nothing), r the draw
        as compared with the CDF and fallback the id taken past its end.
        row: [V] float32 or uint16 (bf16 bits); rng: the state before."""
        row = np.ascontiguousarray(row)
        if row.dtype == np.uint16:
            row = (row.astype(np.uint32) << np.uint32(16)).view(np.float32)
        row = np.ascontiguousarray(row, dtype=np.float32)
        V = row.size
        cfg = np.ascontiguousarray(np.asarray(cfg_row, dtype=CONFIG_DTYPE).reshape(1))
        h = np.ascontiguousarray(hist, dtype=np.int32) if hist is not None else np.zeros(0, np.int32)
        order = np.zeros(V, dtype=np.int32)
        cdf = np.zeros(V, dtype=np.float32)
        r = ctypes.c_float(0.0)
        n = ctypes.c_int(0)
        fb = ctypes.c_int32(-1)
        tok = self.lib.pzo_row_trace(_ptr(row, _f32p), V, cfg.ctypes.data, _ptr(h, _i32p), h.size,
                                     ctypes.c_uint64(int(rng)), ctypes.byref(r), _ptr(order, _i32p),
                                     _ptr(cdf, _f32p), ctypes.byref(n), ctypes.byref(fb))
        k = n.value
        return int(tok), float(np.float32(r.value)), order[:k].copy(), cdf[:k].copy(), int(fb.value)

    def sample_batch(self, logits, cfg, rng, hist=None, hist_off=None, cand_stride=0):
        """logits: [B, V] float32 or uint16 (bf16 bits).  Returns
        (tokens, new_rng, cand_ids, cand_probs, n_cand)."""
        logits = np.ascontiguousarray(logits)
        B, V = logits.shape
        dtype = 0 if logits.dtype == np.float32 else 1
        if dtype == 1:
            assert logits.dtype == np.uint16
        cfg = np.ascontiguousarray(cfg, dtype=CONFIG_DTYPE)
        rng = np.array(rng, dtype=np.uint64, copy=True)
        out = np.zeros(B, dtype=np.int32)
        h = np.ascontiguousarray(hist, dtype=np.int32) if hist is not None else None
        ho = np.ascontiguousarray(hist_off, dtype=np.int32) if hist_off is not None else None
        ci = cp = nc = None
        if cand_stride:
            ci = np.full((B, cand_stride), -1, dtype=np.int32)
            cp = np.zeros((B, cand_stride), dtype=np.float32)
            nc = np.zeros(B, dtype=np.int32)
        rc = self.lib.pzo_sample_batch(
            logits.ctypes.data, dtype, B, V, V, cfg.ctypes.data,
            _ptr(h, _i32p), _ptr(ho, _i32p), _ptr(rng, _u64p), _ptr(out, _i32p),
            _ptr(ci, _i32p), _ptr(cp, _f32p), _ptr(nc, _i32p), int(cand_stride))
        if rc != 0:
            raise ValueError("pzo_sample_batch rejected its arguments")
        return out, rng, ci, cp, nc


class Reference(_Lib):
    """The reference's own compiled sampler (oracle/_ref/libpzref*.so)."""

    def __init__(self, path=None):
        if path is None:
            name = "libpzref.so" if _cpu_has_avx512() else "libpzref_v3.so"
            path = os.path.join(REF_DIR, name)
        super().__init__(path, "pzr_")
        L = self.lib
        L.pzr_apply_temperature.argtypes = [_f32p, ctypes.c_int, ctypes.c_float]
        L.pzr_build_info.restype = ctypes.c_int
        L.pzr_softmax_kernel.restype = ctypes.c_char_p
        L.pzr_sample_batch.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                       ctypes.c_int64, ctypes.c_void_p, _i32p, _i32p, _u64p, _i32p]
        L.pzr_sample_batch.restype = ctypes.c_int

    @property
    def avx512(self) -> bool:
        """True when apply_temperature multiplies by 1/T (TN_HAS_AVX512)."""
        return bool(self.lib.pzr_build_info() & 1)

    @property
    def softmax_kernel(self) -> str:
        return self.lib.pzr_softmax_kernel().decode()

    def apply_temperature(self, x, T):
        x = np.array(x, dtype=np.float32, copy=True)
        self.lib.pzr_apply_temperature(_ptr(x, _f32p), x.size, ctypes.c_float(T))
        return x

    def sample_batch(self, logits, cfg, rng, hist=None, hist_off=None):
        logits = np.ascontiguousarray(logits)
        B, V = logits.shape
        dtype = 0 if logits.dtype == np.float32 else 1
        cfg = np.ascontiguousarray(cfg, dtype=CONFIG_DTYPE)
        rng = np.array(rng, dtype=np.uint64, copy=True)
        out = np.zeros(B, dtype=np.int32)
        h = np.ascontiguousarray(hist, dtype=np.int32) if hist is not None else None
        ho = np.ascontiguousarray(hist_off, dtype=np.int32) if hist_off is not None else None
        rc = self.lib.pzr_sample_batch(logits.ctypes.data, dtype, B, V, V, cfg.ctypes.data,
                                       _ptr(h, _i32p), _ptr(ho, _i32p), _ptr(rng, _u64p),
                                       _ptr(out, _i32p))
        if rc != 0:
            raise ValueError("pzr_sample_batch rejected its arguments")
        return out, rng


def reference_available() -> bool:
    name = "libpzref.so" if _cpu_has_avx512() else "libpzref_v3.so"
    return os.path.exists(os.path.join(REF_DIR, name))
