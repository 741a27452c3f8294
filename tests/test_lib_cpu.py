"""Host-side checks of the C ABI that need no GPU: the library loads, exports
every entry point include/spk.h declares, and rejects bad arguments before
touching the device."""

import ctypes

import pytest

from spikingtransformer_b200 import _lib


def test_exports_every_declared_symbol():
    lib = _lib.load()
    declared = _lib.header_symbols()
    assert len(declared) >= 10
    missing = [s for s in declared if not hasattr(lib, s)]
    assert not missing, missing
    # every declared symbol has a ctypes signature in the binding
    assert set(declared) <= set(_lib.SIGNATURES), set(declared) - set(_lib.SIGNATURES)


def test_binding_argument_counts_match_the_header():
    """Every prototype in include/spk.h takes as many arguments as the ctypes
    binding passes (a drifted binding would push arguments into the wrong
    slots without any error from ctypes)."""
    import re
    text = re.sub(r"/\*.*?\*/", "", open(_lib.HEADER).read(), flags=re.S)
    protos = re.findall(r"\b(spk_[a-z0-9_]+)\s*\(([^;{]*?)\)\s*;", text, flags=re.S)
    assert len(protos) >= 10
    wrong = {}
    for name, args in protos:
        args = args.strip()
        n = 0 if args in ("", "void") else args.count(",") + 1
        if name in _lib.SIGNATURES and len(_lib.SIGNATURES[name][0]) != n:
            wrong[name] = (n, len(_lib.SIGNATURES[name][0]))
    assert not wrong, wrong


def test_version_and_status_strings():
    lib = _lib.load()
    assert lib.spk_version() >= 1
    assert lib.spk_status_string(0) == b"ok"
    assert lib.spk_status_string(5) == b"device wait timed out"


def test_null_arguments_rejected_without_device():
    lib = _lib.load()
    rc = lib.spk_lif_fwd(None, 0, None, 0, None, None, None, None, 1.0, 4, 16, None)
    assert rc == 1
    assert b"null" in lib.spk_last_error()
    rc = lib.spk_ssa_fwd(None, None, None, 1, 0, None, 0, 0, 0, 0, None, None, None, None, 1.0,
                         1, 1, 1, 1, 1, 48, None, 2, None, None)
    assert rc == 1
    rc = lib.spk_ssa_fwd_heads(None, None, None, None, 1, None, None, None, None, 1.0, 1, 1, 1, 1, 1, 48, None, 2,
                               None, None)
    assert rc == 1


def test_shape_limits_rejected_without_device():
    lib = _lib.load()
    buf = ctypes.c_void_p(16)  # never dereferenced: shape checks come first
    rc = lib.spk_lif_fwd(buf, 0, buf, 0, None, buf, buf, buf, 1.0, 65, 16, None)
    assert rc == 2
    rc = lib.spk_ssa_fwd(buf, buf, buf, 1, 0, None, 0, 0, 0, 0, buf, buf, buf, buf, 1.0,
                         1, 1, 1, 8, 8, 100, buf, 2, None, None)
    assert rc == 2
    rc = lib.spk_linear_ln_lif_fwd(buf, buf, None, None, None, 1e-5, buf, buf, buf, 1.0, 4, 8, 12, 64, 0, buf,
                                   2, None, None, None)
    assert rc == 2  # K % 8 != 0
    strides = (ctypes.c_int64 * 9)(*([8] * 9))
    rc = lib.spk_ssa_fwd_heads(buf, buf, buf, strides, 1, buf, buf, buf, buf, 1.0, 1, 1, 1, 300, 8, 48, buf, 2,
                               None, None)
    assert rc == 2  # Nq > 256


def test_workspace_query():
    lib = _lib.load()
    assert lib.spk_lif_bwd_workspace_bytes(4, 1000) >= 4


def test_ops_refuse_cpu_tensors():
    import torch
    from spikingtransformer_b200 import ops
    with pytest.raises(RuntimeError):
        ops.lif_fwd(torch.zeros(2, 4), 0.9, 1.0, 0.0)


def test_stream_forward_checks_host_buffers():
    import torch
    from spikingtransformer_b200.streaming import stream_forward
    x = torch.zeros(2, 3)
    with pytest.raises(ValueError, match="entries"):
        stream_forward(lambda t: t, [(x,), (x,)], [torch.zeros(2, 3)])
    with pytest.raises(ValueError, match="shape or dtype"):
        stream_forward(lambda t: t, [(x,), (torch.zeros(3, 2),)], [x, x])
    with pytest.raises(ValueError, match="tensors"):
        stream_forward(lambda t: t, [(x,), (x, x)], [x, x])
    stream_forward(lambda t: t, [], [])  # nothing to do
