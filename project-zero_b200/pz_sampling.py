"""Python host side of the B200 token sampler (ctypes over libpz_sampling.so).

Mirrors the reference's sampler interface (Project Zero include/sampling/
sampling.h and rng.h) with the same names, argument meaning and results:

    sample_argmax(logits)                   -> int     (argmax.c:3-13)
    apply_temperature(logits, T)            -> array   (temperature.c:8-25)
    sample_top_p(logits, p, state)          -> (int, state)   (top_p.c:30-108)
    sample_top_k(logits, k, state)          -> (int, state)   (top_k.c:8-73)
    rng_seed(seed)                          -> state   (rng.c:3-6)
    rng_float(state)                        -> (float, state) (rng.c:8-17)

The C functions update the RNG word and logits in place; Python integers are
immutable, so these wrappers return the new state (and apply_temperature
returns the scaled array, writing it back when given a float32 numpy array).

`Sampler` wraps the batched device API: logits already on the GPU (a torch
tensor or a raw device pointer), per-row configs, penalty histories and RNG
states, sampled on a CUDA stream with no host round trip.

There is no CPU fallback: importing this module without the built library
raises.  torch is only used here to pass device pointers and streams.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
# PZ_SAMPLING_LIB may point at another build of the same library.
LIB_PATH = os.environ.get("PZ_SAMPLING_LIB") or os.path.join(HERE, "libpz_sampling.so")

if not os.path.exists(LIB_PATH):
    raise ImportError(
        f"{LIB_PATH} is not built (run `make -C {HERE}`); the sampler has no CPU fallback")

_lib = ctypes.CDLL(LIB_PATH)

PZ_OK = 0
PZ_ERR_NCCL = 4
PZ_ERR_TIMEOUT = 5
PZ_ERR_UNSUPPORTED = 6
PZ_DTYPE_F32, PZ_DTYPE_BF16 = 0, 1
PZ_CFG_TEMP_DIVIDE = 0x1
PZ_ROW_OK, PZ_ROW_HISTORY_TOO_LONG, PZ_ROW_HINT_VIOLATED = 0, 1, 2
TOP_K_MAX = 1024

_vp = ctypes.c_void_p
_u64p = ctypes.POINTER(ctypes.c_ulonglong)
_f32p = ctypes.POINTER(ctypes.c_float)


class CtxLimits(ctypes.Structure):
    _fields_ = [("max_batch", ctypes.c_int32), ("max_vocab", ctypes.c_int32),
                ("max_top_k", ctypes.c_int32), ("max_history", ctypes.c_int32)]


class BatchHints(ctypes.Structure):
    _fields_ = [("max_top_k", ctypes.c_int32), ("max_history", ctypes.c_int32),
                ("no_full_vocab", ctypes.c_int32), ("reserved", ctypes.c_int32)]


class BatchOutputs(ctypes.Structure):
    _fields_ = [("cand_ids", _vp), ("cand_probs", _vp), ("n_cand", _vp),
                ("row_status", _vp), ("cand_stride", ctypes.c_int32),
                ("reserved", ctypes.c_int32), ("token_logprob", _vp), ("cand_logprobs", _vp)]


class Shard(ctypes.Structure):
    """pz_shard: one device's part of a pz_sample_batch_multi call."""
    _fields_ = [("ctx", ctypes.c_void_p), ("logits", ctypes.c_void_p), ("ld", ctypes.c_int64),
                ("B", ctypes.c_int32), ("V", ctypes.c_int32), ("v_offset", ctypes.c_int64),
                ("cfg", ctypes.c_void_p), ("hist", ctypes.c_void_p), ("hist_off", ctypes.c_void_p),
                ("rng_state", ctypes.c_void_p), ("out_tokens", ctypes.c_void_p),
                ("outputs", ctypes.c_void_p), ("stream", ctypes.c_void_p)]


SHARD_ROWS, SHARD_VOCAB = 0, 1


class SamplerConfigC(ctypes.Structure):
    """pz_sampler_config as a ctypes structure (32 bytes)."""
    _fields_ = [("temperature", ctypes.c_float), ("top_k", ctypes.c_int32), ("top_p", ctypes.c_float),
                ("repetition_penalty", ctypes.c_float), ("frequency_penalty", ctypes.c_float),
                ("presence_penalty", ctypes.c_float), ("flags", ctypes.c_uint32), ("reserved", ctypes.c_uint32)]


class SamplingParams(ctypes.Structure):
    """pz_sampling_params: a request's settings from the command line or a
    chat-completions JSON body."""
    _fields_ = [("cfg", SamplerConfigC), ("seed", ctypes.c_int64), ("logprobs", ctypes.c_int32),
                ("top_logprobs", ctypes.c_int32)]

    def as_config(self, B=1):
        """The config as a CONFIG_DTYPE array of B identical rows."""
        c = self.cfg
        return make_configs(B, c.temperature, c.top_k, c.top_p, c.repetition_penalty,
                            c.frequency_penalty, c.presence_penalty, c.flags)


# pz_sampler_config, 32 bytes
CONFIG_DTYPE = np.dtype([
    ("temperature", "<f4"), ("top_k", "<i4"), ("top_p", "<f4"),
    ("repetition_penalty", "<f4"), ("frequency_penalty", "<f4"),
    ("presence_penalty", "<f4"), ("flags", "<u4"), ("reserved", "<u4")])
assert CONFIG_DTYPE.itemsize == 32


def make_configs(B, temperature=1.0, top_k=0, top_p=1.0, rep=1.0, freq=0.0,
                 pres=0.0, flags=0):
    """Structured array of B pz_sampler_config; scalars broadcast."""
    c = np.zeros(B, dtype=CONFIG_DTYPE)
    c["temperature"] = temperature
    c["top_k"] = top_k
    c["top_p"] = top_p
    c["repetition_penalty"] = rep
    c["frequency_penalty"] = freq
    c["presence_penalty"] = pres
    c["flags"] = flags
    return c


def _sig(name, res, args):
    f = getattr(_lib, name)
    f.restype = res
    f.argtypes = args
    return f


_sig("pz_status_str", ctypes.c_char_p, [ctypes.c_int])
_sig("pz_version", ctypes.c_char_p, [])
_sig("pz_last_error", ctypes.c_int, [])
_sig("pz_last_error_detail", ctypes.c_char_p, [])
_sig("pz_sample_argmax", ctypes.c_int, [_f32p, ctypes.c_int])
_sig("pz_apply_temperature", None, [_f32p, ctypes.c_int, ctypes.c_float])
_sig("pz_sample_top_p", ctypes.c_int, [_f32p, ctypes.c_int, ctypes.c_float, _u64p])
_sig("pz_sample_top_k", ctypes.c_int, [_f32p, ctypes.c_int, ctypes.c_int, _u64p])
_sig("pz_sample_softmax", ctypes.c_int, [_f32p, ctypes.c_int, _u64p])
_sig("pz_rng_seed", None, [_u64p, ctypes.c_ulonglong])
_sig("pz_rng_float", ctypes.c_float, [_u64p])
_sig("pz_ctx_create", ctypes.c_int, [ctypes.POINTER(_vp), ctypes.c_int, ctypes.POINTER(CtxLimits)])
_sig("pz_ctx_destroy", ctypes.c_int, [_vp])
_sig("pz_ctx_scratch_bytes", ctypes.c_size_t, [_vp])
_sig("pz_sample_batch", ctypes.c_int,
     [_vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int64, _vp, _vp, _vp, _vp, _vp,
      ctypes.POINTER(BatchHints), ctypes.POINTER(BatchOutputs), _vp])
_sig("pz_rng_seed_batch", ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_ulonglong, _vp, _vp])
_sig("pz_ctx_profile", ctypes.c_int, [_vp, ctypes.c_int])
_sig("pz_ctx_profile_read", ctypes.c_int,
     [_vp, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_int),
      ctypes.POINTER(ctypes.c_int)])
_sig("pz_ctx_profile_phases", ctypes.c_int,
     [_vp, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int)])
_sig("pz_ctx_init_nccl_timeout", ctypes.c_int,
     [_vp, ctypes.c_int, ctypes.c_int, _vp, ctypes.c_size_t, ctypes.c_int])
_sig("pz_ctx_wait", ctypes.c_int, [_vp, _vp, ctypes.c_int])
_sig("pz_ctx_abort_nccl", ctypes.c_int, [_vp])
_sig("pz_sample_batch_static", ctypes.c_int,
     [_vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int64, _vp, _vp, _vp, _vp, _vp,
      ctypes.POINTER(BatchOutputs), _vp])
_sig("pz_row_shard", None, [ctypes.c_int, ctypes.c_int, ctypes.c_int,
                            ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int)])
_sig("pz_nccl_get_unique_id", ctypes.c_int, [_vp, ctypes.c_size_t])
_sig("pz_ctx_init_nccl", ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, _vp, ctypes.c_size_t])
_sig("pz_sample_batch_vocab_sharded", ctypes.c_int,
     [_vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int64, ctypes.c_int64,
      ctypes.c_int, _vp, _vp, _vp, _vp, _vp, ctypes.POINTER(BatchOutputs), _vp])


_sig("pz_multi_init_nccl", ctypes.c_int, [ctypes.POINTER(_vp), ctypes.c_int, ctypes.c_int])
_sig("pz_sample_batch_multi", ctypes.c_int,
     [ctypes.c_int, ctypes.c_int, ctypes.POINTER(Shard), ctypes.c_int, ctypes.c_int, ctypes.POINTER(BatchHints)])


_sig("pz_params_init_cli", None, [ctypes.POINTER(SamplingParams)])
_sig("pz_params_init_api", None, [ctypes.POINTER(SamplingParams)])
_sig("pz_params_from_args", ctypes.c_int,
     [ctypes.POINTER(SamplingParams), ctypes.c_int, ctypes.POINTER(ctypes.c_char_p)])
_sig("pz_params_from_json", ctypes.c_int, [ctypes.POINTER(SamplingParams), ctypes.c_char_p])


_sig("pz_history_append", ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, _vp, _vp, _vp])
_sig("pz_lm_head_logits", ctypes.c_int,
     [_vp, _vp, ctypes.c_int, ctypes.c_int, _vp, ctypes.c_int, _vp, ctypes.c_int64, _vp])
_sig("pz_sample_from_hidden", ctypes.c_int,
     [_vp, _vp, ctypes.c_int, ctypes.c_int, _vp, ctypes.c_int, _vp, ctypes.c_int64, _vp, _vp, _vp, _vp, _vp,
      ctypes.POINTER(BatchHints), ctypes.POINTER(BatchOutputs), _vp])
_sig("pz_decode_step_create", ctypes.c_int,
     [_vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int64, _vp, _vp, ctypes.c_int, _vp, _vp,
      ctypes.POINTER(BatchHints), ctypes.POINTER(_vp)])
_sig("pz_decode_step_launch", ctypes.c_int, [_vp, _vp])
_sig("pz_decode_step_count", ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_int32)])
_sig("pz_decode_step_destroy", ctypes.c_int, [_vp])


class PZError(RuntimeError):
    def __init__(self, status, what=""):
        self.status = status
        detail = _lib.pz_last_error_detail().decode()
        super().__init__(f"{what}: {_lib.pz_status_str(status).decode()} (status {status})"
                         + (f" [{detail}]" if detail else ""))


def _check(status, what):
    if status != PZ_OK:
        raise PZError(status, what)


def version() -> str:
    return _lib.pz_version().decode()


def library_path() -> str:
    return LIB_PATH


# --------------------------------------------------------------------------
# The reference's six calls (host arrays; the row is staged to the GPU).
# --------------------------------------------------------------------------
def _f32(x):
    return np.ascontiguousarray(x, dtype=np.float32)


def _legacy_check(what):
    s = _lib.pz_last_error()
    if s != PZ_OK:
        raise PZError(s, what)


def sample_argmax(logits) -> int:
    x = _f32(logits)
    t = _lib.pz_sample_argmax(x.ctypes.data_as(_f32p), x.size)
    _legacy_check("sample_argmax")
    return int(t)


def apply_temperature(logits, temperature):
    """Scales in place when given a float32 array; returns the scaled array."""
    inplace = isinstance(logits, np.ndarray) and logits.dtype == np.float32 and logits.flags.c_contiguous
    x = logits if inplace else np.array(logits, dtype=np.float32)
    _lib.pz_apply_temperature(x.ctypes.data_as(_f32p), x.size, ctypes.c_float(temperature))
    _legacy_check("apply_temperature")
    return x


def sample_top_p(logits, top_p, state):
    x = _f32(logits)
    s = ctypes.c_ulonglong(state)
    t = _lib.pz_sample_top_p(x.ctypes.data_as(_f32p), x.size, ctypes.c_float(top_p), ctypes.byref(s))
    _legacy_check("sample_top_p")
    return int(t), s.value


def sample_top_k(logits, k, state):
    x = _f32(logits)
    s = ctypes.c_ulonglong(state)
    t = _lib.pz_sample_top_k(x.ctypes.data_as(_f32p), x.size, int(k), ctypes.byref(s))
    _legacy_check("sample_top_k")
    return int(t), s.value


def sample_softmax(logits, state):
    """Full-softmax draw of the reference's generate loop (generate.c:157-168)."""
    x = _f32(logits)
    s = ctypes.c_ulonglong(state)
    t = _lib.pz_sample_softmax(x.ctypes.data_as(_f32p), x.size, ctypes.byref(s))
    _legacy_check("sample_softmax")
    return int(t), s.value


def rng_seed(seed) -> int:
    s = ctypes.c_ulonglong(0)
    _lib.pz_rng_seed(ctypes.byref(s), ctypes.c_ulonglong(seed))
    return s.value


def rng_float(state):
    s = ctypes.c_ulonglong(state)
    v = _lib.pz_rng_float(ctypes.byref(s))
    return float(np.float32(v)), s.value


def params_from_args(argv):
    """pz_params_from_args over a command line (argv[0] is the program)."""
    p = SamplingParams()
    arr = (ctypes.c_char_p * len(argv))(*[a.encode() for a in argv])
    _check(_lib.pz_params_from_args(ctypes.byref(p), len(argv), arr), "pz_params_from_args")
    return p


def params_from_json(body):
    """pz_params_from_json over a chat-completions request body."""
    p = SamplingParams()
    _check(_lib.pz_params_from_json(ctypes.byref(p), body.encode() if isinstance(body, str) else body),
           "pz_params_from_json")
    return p


def row_shard(B, world, rank):
    """Contiguous row range (begin, count) that `rank` owns."""
    b, c = ctypes.c_int(0), ctypes.c_int(0)
    _lib.pz_row_shard(B, world, rank, ctypes.byref(b), ctypes.byref(c))
    return b.value, c.value


# --------------------------------------------------------------------------
# Batched device API.
# --------------------------------------------------------------------------
def _ptr(t):
    """Device pointer of a torch tensor (or an int pointer, or None)."""
    if t is None:
        return None
    if isinstance(t, int):
        return t
    return t.data_ptr()


def _stream_handle(stream):
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


class Sampler:
    """One device's sampling context (owns the scratch; allocation happens
    here, never inside sample())."""

    def __init__(self, device=0, max_batch=1024, max_vocab=262144, max_top_k=TOP_K_MAX,
                 max_history=2048):
        self.device = device
        self.limits = CtxLimits(max_batch, max_vocab, max_top_k, max_history)
        h = _vp()
        _check(_lib.pz_ctx_create(ctypes.byref(h), device, ctypes.byref(self.limits)), "pz_ctx_create")
        self._h = h
        self.world, self.rank = 1, 0

    @property
    def scratch_bytes(self) -> int:
        return int(_lib.pz_ctx_scratch_bytes(self._h))

    def close(self):
        if getattr(self, "_h", None):
            _lib.pz_ctx_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @staticmethod
    def _dtype_code(logits):
        import torch
        if logits.dtype == torch.float32:
            return PZ_DTYPE_F32
        if logits.dtype == torch.bfloat16:
            return PZ_DTYPE_BF16
        raise TypeError(f"logits dtype {logits.dtype} (want float32 or bfloat16)")

    @staticmethod
    def _outputs(cand_ids=None, cand_probs=None, n_cand=None, row_status=None, token_logprob=None,
                 cand_logprobs=None):
        if all(t is None for t in (cand_ids, cand_probs, n_cand, row_status, token_logprob, cand_logprobs)):
            return None
        stride = 0
        for t in (cand_ids, cand_probs, cand_logprobs):
            if t is not None:
                stride = t.shape[1]
                break
        return BatchOutputs(_ptr(cand_ids), _ptr(cand_probs), _ptr(n_cand), _ptr(row_status), stride, 0,
                            _ptr(token_logprob), _ptr(cand_logprobs))

    def sample(self, logits, cfg, rng_state, out, hist=None, hist_off=None, *,
               max_top_k=0, max_history=0, no_full_vocab=False, cand_ids=None,
               cand_probs=None, n_cand=None, row_status=None, token_logprob=None,
               cand_logprobs=None, stream=None):
        """logits: [B, V] (row stride = logits.stride(0)) float32/bfloat16 CUDA
        tensor; cfg: device tensor holding B pz_sampler_config (32 bytes each);
        rng_state: [B] int64 device tensor (xorshift64* words, advanced in
        place); out: [B] int32 device tensor; hist/hist_off: CSR int32 device
        tensors or None."""
        B, V = logits.shape
        hints = BatchHints(max_top_k, max_history, 1 if no_full_vocab else 0, 0)
        outs = self._outputs(cand_ids, cand_probs, n_cand, row_status, token_logprob, cand_logprobs)
        st = _lib.pz_sample_batch(
            self._h, _ptr(logits), self._dtype_code(logits), B, V, logits.stride(0),
            _ptr(cfg), _ptr(hist), _ptr(hist_off), _ptr(rng_state), _ptr(out),
            ctypes.byref(hints), ctypes.byref(outs) if outs is not None else None,
            _stream_handle(stream))
        _check(st, "pz_sample_batch")
        return out

    def lm_head(self, hidden, w_cls, logits, stream=None):
        """pz_lm_head_logits: logits[B, V] = hidden[B, dim] (fp32) @ w_cls[V, dim]^T
        (bf16), on the device."""
        B, dim = hidden.shape
        V = w_cls.shape[0]
        _check(_lib.pz_lm_head_logits(self._h, _ptr(hidden), B, dim, _ptr(w_cls), V, _ptr(logits),
                                      logits.stride(0), _stream_handle(stream)), "pz_lm_head_logits")
        return logits

    def sample_from_hidden(self, hidden, w_cls, logits, cfg, rng_state, out, hist=None, hist_off=None, *,
                           max_top_k=0, max_history=0, no_full_vocab=False, stream=None):
        """pz_sample_from_hidden: the classifier into `logits`, then the batch
        sampler on it, both on the stream."""
        B, dim = hidden.shape
        V = w_cls.shape[0]
        hints = BatchHints(max_top_k, max_history, 1 if no_full_vocab else 0, 0)
        _check(_lib.pz_sample_from_hidden(self._h, _ptr(hidden), B, dim, _ptr(w_cls), V, _ptr(logits),
                                          logits.stride(0), _ptr(cfg), _ptr(hist), _ptr(hist_off),
                                          _ptr(rng_state), _ptr(out), ctypes.byref(hints), None,
                                          _stream_handle(stream)), "pz_sample_from_hidden")
        return out

    def profile(self, n_calls):
        """Times the kernels of the next n_calls sampling calls with CUDA
        events (0 turns timing off)."""
        _check(_lib.pz_ctx_profile(self._h, int(n_calls)), "pz_ctx_profile")

    def profile_read(self):
        """(slice_kernel ms, rest ms, calls, kernels launched) summed over the
        timed calls since the last read."""
        a, b, n, k = ctypes.c_double(), ctypes.c_double(), ctypes.c_int(), ctypes.c_int()
        _check(_lib.pz_ctx_profile_read(self._h, ctypes.byref(a), ctypes.byref(b), ctypes.byref(n),
                                        ctypes.byref(k)), "pz_ctx_profile_read")
        return a.value, b.value, n.value, k.value

    def profile_phases(self):
        """({'slice', 'full', 'allgather', 'merge'} ms summed over the timed
        calls, calls, kernels launched) since the last read."""
        ph = (ctypes.c_double * 4)()
        n, k = ctypes.c_int(), ctypes.c_int()
        _check(_lib.pz_ctx_profile_phases(self._h, ph, ctypes.byref(n), ctypes.byref(k)),
               "pz_ctx_profile_phases")
        return dict(zip(("slice", "full", "allgather", "merge"), list(ph))), n.value, k.value

    def wait(self, timeout_ms, stream=None):
        """Bounded wait for the stream's work (NCCL errors and the deadline
        abort the communicator and raise)."""
        _check(_lib.pz_ctx_wait(self._h, _stream_handle(stream), int(timeout_ms)), "pz_ctx_wait")

    def abort_nccl(self):
        _check(_lib.pz_ctx_abort_nccl(self._h), "pz_ctx_abort_nccl")

    # ---- vocab sharding --------------------------------------------------
    @staticmethod
    def nccl_unique_id() -> bytes:
        buf = ctypes.create_string_buffer(128)
        _check(_lib.pz_nccl_get_unique_id(buf, 128), "pz_nccl_get_unique_id")
        return buf.raw

    def init_nccl(self, world, rank, unique_id: bytes, timeout_ms=60000):
        buf = ctypes.create_string_buffer(unique_id, 128)
        _check(_lib.pz_ctx_init_nccl_timeout(self._h, world, rank, buf, 128, int(timeout_ms)),
               "pz_ctx_init_nccl")
        self.world, self.rank = world, rank

    def sample_vocab_sharded(self, logits_slice, v_offset, V_global, cfg, rng_state, out,
                             hist=None, hist_off=None, *, cand_ids=None, cand_probs=None,
                             n_cand=None, row_status=None, stream=None):
        B, V_local = logits_slice.shape
        outs = self._outputs(cand_ids, cand_probs, n_cand, row_status)
        st = _lib.pz_sample_batch_vocab_sharded(
            self._h, _ptr(logits_slice), self._dtype_code(logits_slice), B, V_local,
            logits_slice.stride(0), v_offset, V_global, _ptr(cfg), _ptr(hist), _ptr(hist_off),
            _ptr(rng_state), _ptr(out), ctypes.byref(outs) if outs is not None else None,
            _stream_handle(stream))
        _check(st, "pz_sample_batch_vocab_sharded")
        return out


def multi_init_nccl(samplers, timeout_ms=60000):
    """pz_multi_init_nccl: joins the samplers (one per device of this
    process) to one communicator, samplers[i] as rank i."""
    arr = (_vp * len(samplers))(*[s._h for s in samplers])
    _check(_lib.pz_multi_init_nccl(arr, len(samplers), int(timeout_ms)), "pz_multi_init_nccl")
    for i, s in enumerate(samplers):
        s.world, s.rank = len(samplers), i


def sample_multi(mode, parts, V_global, *, max_top_k=0, max_history=0, no_full_vocab=False):
    """pz_sample_batch_multi from one thread.  parts: one dict per device with
    keys sampler, logits, cfg, rng_state, out and optionally hist, hist_off,
    v_offset (vocab mode), stream, and the candidate outputs (cand_ids,
    cand_probs, n_cand, row_status)."""
    n = len(parts)
    arr = (Shard * n)()
    keep = []
    dtype = None
    for i, d in enumerate(parts):
        x = d["logits"]
        dt = Sampler._dtype_code(x)
        if dtype is not None and dt != dtype:
            raise TypeError("every shard needs the same logits dtype")
        dtype = dt
        outs = Sampler._outputs(d.get("cand_ids"), d.get("cand_probs"), d.get("n_cand"), d.get("row_status"))
        if outs is not None:
            keep.append(outs)
        arr[i] = Shard(d["sampler"]._h.value, _ptr(x), x.stride(0), x.shape[0], x.shape[1],
                       int(d.get("v_offset", 0)), _ptr(d["cfg"]), _ptr(d.get("hist")), _ptr(d.get("hist_off")),
                       _ptr(d["rng_state"]), _ptr(d["out"]),
                       ctypes.addressof(outs) if outs is not None else None,
                       _stream_handle(d.get("stream")) if d.get("stream") is not None else _current_stream(x))
    hints = BatchHints(max_top_k, max_history, 1 if no_full_vocab else 0, 0)
    _check(_lib.pz_sample_batch_multi(mode, n, arr, dtype, int(V_global), ctypes.byref(hints)),
           "pz_sample_batch_multi")


def _current_stream(t):
    import torch
    return torch.cuda.current_stream(t.device).cuda_stream


class DecodeStep:
    """One sampling step of the generate loop as a CUDA graph
    (pz_decode_step_*): the fixed logits buffer sampled, the RNG states
    advanced and each sampled id appended to its row's history window, all
    on the device.  The tensors given here stay bound to the step."""

    def __init__(self, sampler, logits, cfg, rng_state, out, hist_ring=None, *, max_top_k=0,
                 max_history=0, no_full_vocab=False):
        B, V = logits.shape
        W = 0 if hist_ring is None else hist_ring.shape[1]
        hints = BatchHints(max_top_k, max_history, 1 if no_full_vocab else 0, 0)
        h = _vp()
        _check(_lib.pz_decode_step_create(sampler._h, _ptr(logits), Sampler._dtype_code(logits), B, V,
                                          logits.stride(0), _ptr(cfg), _ptr(hist_ring), W, _ptr(rng_state),
                                          _ptr(out), ctypes.byref(hints), ctypes.byref(h)),
               "pz_decode_step_create")
        self._h = h
        self._keep = (sampler, logits, cfg, rng_state, out, hist_ring)

    def launch(self, stream=None):
        _check(_lib.pz_decode_step_launch(self._h, _stream_handle(stream)), "pz_decode_step_launch")

    def steps(self):
        n = ctypes.c_int32()
        _check(_lib.pz_decode_step_count(self._h, ctypes.byref(n)), "pz_decode_step_count")
        return n.value

    def close(self):
        if getattr(self, "_h", None):
            _lib.pz_decode_step_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def history_append(hist_ring, tokens, counter, stream=None):
    """pz_history_append: tokens[r] into hist_ring[r, counter % W], counter += 1."""
    B, W = hist_ring.shape
    _check(_lib.pz_history_append(_ptr(hist_ring), B, W, _ptr(tokens), _ptr(counter), _stream_handle(stream)),
           "pz_history_append")


STATIC_MAX_BATCH = 1024
STATIC_MAX_VOCAB = 1048576
STATIC_MAX_TOP_K = 64
STATIC_MAX_HISTORY = 1024


def sample_static(logits, cfg, rng_state, out, hist=None, hist_off=None, *, cand_ids=None,
                  cand_probs=None, n_cand=None, row_status=None, stream=None):
    """pz_sample_batch_static: Sampler.sample without a context, on the
    current CUDA device, with the library's fixed per-device scratch (no
    allocation; B <= 1024, top_k 1..64, history <= 1024 ids per row).  The
    first call on a device does the set-up.  Calls on one device must not
    overlap in time: they share that scratch."""
    B, V = logits.shape
    outs = Sampler._outputs(cand_ids, cand_probs, n_cand, row_status)
    st = _lib.pz_sample_batch_static(
        _ptr(logits), Sampler._dtype_code(logits), B, V, logits.stride(0), _ptr(cfg), _ptr(hist),
        _ptr(hist_off), _ptr(rng_state), _ptr(out),
        ctypes.byref(outs) if outs is not None else None, _stream_handle(stream))
    _check(st, "pz_sample_batch_static")
    return out


def seed_states(rng_state, seed_base=0, seeds=None, stream=None):
    """state[r] = seeds[r] (device tensor) or seed_base + r; 0 becomes 1."""
    _check(_lib.pz_rng_seed_batch(_ptr(rng_state), rng_state.numel(), seed_base, _ptr(seeds),
                                  _stream_handle(stream)), "pz_rng_seed_batch")
    return rng_state


def configs_to_device(cfg_np, device="cuda"):
    """Copies a CONFIG_DTYPE array to a device byte tensor."""
    import torch
    raw = np.ascontiguousarray(cfg_np, dtype=CONFIG_DTYPE).view(np.uint8)
    return torch.from_numpy(raw.copy()).to(device)
