"""ctypes binding of libspk.so (the C ABI declared in include/spk.h).

The library is loaded from this package directory.  There is no fallback: if
it is missing or the device is not sm_100, calls raise ``RuntimeError``.
"""

import ctypes
import os
import re
import threading

import torch

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libspk.so")
HEADER = os.path.join(os.path.dirname(PKG), "include", "spk.h")

F32, F16, BF16, U8, FP8, BIT = 0, 1, 2, 3, 4, 5
DTYPE_CODE = {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16, torch.uint8: U8,
              torch.float8_e4m3fn: FP8}

SURROGATE = {"superspike": 0, "arctan": 1}

_p = ctypes.c_void_p
_i = ctypes.c_int
_i64 = ctypes.c_int64
_f = ctypes.c_float

# argument/return types of every exported entry point
SIGNATURES = {
    "spk_version": ([], _i),
    "spk_status_string": ([_i], ctypes.c_char_p),
    "spk_last_error": ([], ctypes.c_char_p),
    "spk_device_error_check": ([_p], _i),
    "spk_test_bounded_wait": ([_i64, _p], _i),
    "spk_lif_fwd": ([_p, _i, _p, _i, _p, _p, _p, _p, _f, _i64, _i64, _p], _i),
    "spk_lif_bwd_workspace_bytes": ([_i64, _i64], _i64),
    "spk_lif_bwd": ([_p, _p, _p, _i, _p, _i, _p, _p, _p, _f, _i, _f, _p, _p, _p, _i64, _i64, _i64, _p], _i),
    "spk_lif_bwd_noalloc": ([_p, _p, _p, _i, _p, _i, _p, _p, _p, _f, _i, _f, _p, _p, _i64, _i64, _p], _i),
    "spk_linear_ln_lif_fwd": ([_p, _p, _p, _p, _p, _f, _p, _p, _p, _f, _i64, _i64, _i64, _i64, _i, _p, _i, _p,
                               _p, _p], _i),
    "spk_linear_fwd": ([_p, _p, _p, _p, _i64, _i64, _i64, _p], _i),
    "spk_linear_dgrad": ([_p, _p, _p, _i64, _i64, _i64, _p], _i),
    "spk_linear_wgrad_workspace_bytes": ([_i64, _i64, _i64], _i64),
    "spk_linear_wgrad": ([_p, _p, _p, _p, _i64, _i64, _i64, _i64, _p], _i),
    "spk_linear_affine_lif_fwd": ([_p, _p, _p, _p, _p, _p, _p, _p, _f, _i64, _i64, _i64, _i64, _i, _p, _i, _p, _p],
                                  _i),
    "spk_im2col": ([_p, _i, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _p, _p], _i),
    "spk_ln_lif_fwd": ([_p, _i, _p, _p, _p, _f, _p, _p, _p, _f, _i64, _i64, _i64, _i64, _i64, _i64, _p, _i, _p, _p],
                       _i),
    "spk_ln_lif_fwd_residual": ([_p, _i, _p, _p, _p, _f, _p, _p, _p, _f, _i64, _i64, _i64, _i64, _p, _p, _p, _p,
                                 _p], _i),
    "spk_ln_lif_bwd_workspace_bytes": ([_i64, _i64, _i64], _i64),
    "spk_ln_lif_bwd": ([_p, _i, _p, _i, _p, _p, _p, _p, _p, _p, _p, _f, _i, _f, _i64, _i64, _i64, _i64, _i64, _i64,
                        _p, _p, _p, _p, _p, _p, _i64, _p], _i),
    "spk_ssa_fwd": ([_p, _p, _p, _i, _i, _p, _i64, _i64, _i64, _i64, _p, _p, _p, _p, _f, _i64, _i64, _i64, _i64,
                     _i64, _i64, _p, _i, _p, _p], _i),
    "spk_ssa_fwd_heads": ([_p, _p, _p, _p, _i, _p, _p, _p, _p, _f, _i64, _i64, _i64, _i64, _i64, _i64, _p, _i,
                           _p, _p], _i),
    "spk_embed_pe_lif_fwd": ([_p, _p, _f, _p, _p, _p, _p, _f, _i64, _i64, _i64, _i64, _i64, _p, _i, _p, _p], _i),
    "spk_patch_im2col": ([_p, _i64, _i64, _i64, _i64, _i64, _p, _p], _i),
    "spk_synth_text_lines": ([_p, _i64, _i64, _i64, ctypes.c_uint64, _p, _i64, _i64, _p], _i),
    "spk_ce_over_t_workspace_bytes": ([_i64], _i64),
    "spk_ce_over_t": ([_p, _i, _p, _i64, _i64, _i64, _i64, _f, _p, _p, _p, _i64, _p, _p], _i),
    "spk_attn_masked_train_fwd": ([_p, _p, _p, _i, _p, _p, _i64, _i64, _i64, _i64, _i, _p, _i64, _i64, _i64, _i64,
                                   _i64, _i64, _p, _p], _i),
    "spk_attn_masked_train_bwd": ([_p, _p, _p, _i, _p, _p, _i64, _i64, _i64, _i64, _i, _p, _i64, _i64, _i64, _i64,
                                   _i64, _i64, _p, _p, _p, _p, _p, _p], _i),
    "spk_xnor_train_combine": ([_p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _p], _i),
    "spk_xnor_train_prep_chunks": ([_i64], _i64),
    "spk_xnor_train_grad_prep": ([_p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _p], _i),
    "spk_xnor_train_grad_finish": ([_p, _p, _p, _p, _p, _p, _i, _i64, _i64, _i64, _i64, _p], _i),
    "spk_xnor_train_n_major": ([_p, _p, _i64, _i64, _i64, _p], _i),
    "spk_xnor_train_combine_lif": ([_p, _p, _p, _p, _p, _p, _p, _f, _p, _p, _i, _i64, _i64, _i64, _i64, _i64, _p], _i),
    "spk_xnor_train_grad_prep_lif": ([_p, _i, _p, _p, _p, _p, _p, _f, _i, _f, _p, _p, _p, _p, _p, _i64, _i64, _i64,
                                      _i64, _i64, _p], _i),
}

_lib = None
_lock = threading.Lock()


def load():
    """Load libspk.so (once) and declare the signatures."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    "libspk.so not found at %s; build it with `python -m spikingtransformer_b200.build`"
                    % LIB_PATH)
            lib = ctypes.CDLL(LIB_PATH)
            for name, (argtypes, restype) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = argtypes
                fn.restype = restype
            _lib = lib
    return _lib


def header_symbols():
    """Names of the functions declared in include/spk.h."""
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(spk_[a-z0-9_]+)\s*\(", text)))


class LaunchRecorder:
    """Records a CUDA event pair around every entry-point call made while it is
    active (on the stream the kernels are launched on), with the call's tag
    and algorithmic work, for per-kernel timing inside a timed region."""

    def __init__(self):
        self.records = []

    def __enter__(self):
        global _recorder
        self._prev = _recorder
        _recorder = self
        return self

    def __exit__(self, *exc):
        global _recorder
        _recorder = self._prev
        return False

    def summary(self):
        """{tag: dict(launches, ms, flops, bytes)} (synchronises)."""
        torch.cuda.synchronize()
        out = {}
        for tag, e0, e1, work in self.records:
            d = out.setdefault(tag, dict(launches=0, ms=0.0, flops=0.0, bytes=0.0))
            d["launches"] += work.get("launches", 1)
            d["ms"] += e0.elapsed_time(e1)
            d["flops"] += work.get("flops", 0.0)
            d["bytes"] += work.get("bytes", 0.0)
        return out


class LaunchCounter:
    """Counts the kernels this library launches while it is active, by tag,
    without events (usable while a CUDA graph is being captured)."""

    def __init__(self):
        self.counts = {}

    def __enter__(self):
        global _counter
        self._prev = _counter
        _counter = self
        return self

    def __exit__(self, *exc):
        global _counter
        _counter = self._prev
        return False

    def total(self):
        return sum(self.counts.values())


_recorder = None
_counter = None


def call(name, *args, tag=None, work=None):
    """Call an int-returning entry point; raise RuntimeError on failure."""
    lib = load()
    if _counter is not None:
        k = tag or name
        _counter.counts[k] = _counter.counts.get(k, 0) + (work or {}).get("launches", 1)
    rec = _recorder
    if rec is not None:
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
    rc = getattr(lib, name)(*args)
    if rec is not None:
        e1.record()
        rec.records.append((tag or name, e0, e1, work or {}))
    if rc != 0:
        msg = lib.spk_last_error().decode(errors="replace")
        status = lib.spk_status_string(rc).decode()
        raise RuntimeError("%s failed (%s): %s" % (name, status, msg))
    return rc


def stream_ptr(device=None):
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t):
    return None if t is None else t.data_ptr()


def dtype_code(t):
    try:
        return DTYPE_CODE[t.dtype]
    except KeyError:
        raise TypeError("unsupported dtype %s" % t.dtype)
