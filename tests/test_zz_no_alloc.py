"""spk_lif_bwd_noalloc: the LIF backward that allocates nothing (its grad_beta
partial sums live in a static device array) must give the same results as
spk_lif_bwd with a caller-provided workspace.  Both are called through the
C ABI with ctypes.  The calls come in a row with different sizes, so a
result that depended on the previous call's leftovers in the shared array
would show.  The file is named to be collected last; it also passes alone
in a fresh process.
"""

import pytest
import torch

from spikingtransformer_b200 import _lib

pytestmark = pytest.mark.gpu


def _inputs(T, N, seed, x_dtype=torch.float32, spike_dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(T, N, generator=g) * 0.8 + 0.6).to(x_dtype)
    v = torch.zeros(N)
    spikes = torch.empty(T, N)
    for t in range(T):  # spikes of the forward pass, beta 0.9, v_th 1, v_reset 0
        v = 0.9 * v + x[t].float()
        spikes[t] = (v >= 1.0).float()
        v = torch.where(spikes[t] > 0, torch.zeros_like(v), v)
    gs = torch.randn(T, N, generator=g)
    gv = torch.randn(N, generator=g)
    dev = torch.device("cuda", 0)
    return x.to(dev), spikes.to(spike_dtype).to(dev), gs.to(dev), gv.to(dev)


def _params(dev):
    return (torch.tensor([0.9], device=dev), torch.tensor([1.0], device=dev), torch.tensor([0.0], device=dev))


def _bwd_workspace(lib, x, spikes, gs, gv, prm, surrogate, k, gain):
    T, N = x.shape[0], x[0].numel()
    gx = torch.empty_like(x)
    gb = torch.empty(1, device=x.device)
    wsb = int(lib.spk_lif_bwd_workspace_bytes(T, N))
    ws = torch.empty(wsb // 4, device=x.device)
    rc = lib.spk_lif_bwd(gs.data_ptr(), gv.data_ptr(), x.data_ptr(), _lib.dtype_code(x), spikes.data_ptr(),
                         _lib.dtype_code(spikes), prm[0].data_ptr(), prm[1].data_ptr(), prm[2].data_ptr(),
                         gain, surrogate, k, gx.data_ptr(), gb.data_ptr(), ws.data_ptr(), wsb, T, N,
                         _lib.stream_ptr(x.device))
    assert rc == 0, lib.spk_last_error().decode()
    return gx, gb


def _bwd_noalloc(lib, x, spikes, gs, gv, prm, surrogate, k, gain, gx, gb):
    T, N = x.shape[0], x[0].numel()
    return lib.spk_lif_bwd_noalloc(gs.data_ptr(), gv.data_ptr(), x.data_ptr(), _lib.dtype_code(x),
                                   spikes.data_ptr(), _lib.dtype_code(spikes), prm[0].data_ptr(),
                                   prm[1].data_ptr(), prm[2].data_ptr(), gain, surrogate, k, gx.data_ptr(),
                                   gb.data_ptr(), T, N, _lib.stream_ptr(x.device))


def test_noalloc_matches_workspace_entry_point_two_calls_in_a_row():
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    prm = _params(dev)
    # large (3072-block grid, vector path), then small and odd (scalar path),
    # then large and odd (scalar path at the 4096-block cap, every partial of
    # the static array in use), then the first one again: bit-exact, the
    # tolerance the LIF tests use
    # the last case has bf16 spikes, which the shared-memory-staged backward
    # (persistent blocks, one partial each) takes
    f32, bf16 = torch.float32, torch.bfloat16
    cases = [(4, 3 << 20, 1, _lib.SURROGATE["superspike"], 4.0, 1.0, f32),
             (3, 1001, 2, _lib.SURROGATE["arctan"], 2.0, 0.5, f32),
             (4, (3 << 20) + 1, 5, _lib.SURROGATE["superspike"], 4.0, 1.0, f32),
             (4, 3 << 20, 3, _lib.SURROGATE["superspike"], 4.0, 1.0, f32),
             (4, 3 << 20, 6, _lib.SURROGATE["arctan"], 2.0, 0.5, bf16)]
    for T, N, seed, surrogate, k, gain, sdt in cases:
        x, spikes, gs, gv = _inputs(T, N, seed, spike_dtype=sdt)
        want_gx, want_gb = _bwd_workspace(lib, x, spikes, gs, gv, prm, surrogate, k, gain)
        gx = torch.full_like(x, float("nan"))
        gb = torch.full((1,), float("nan"), device=dev)
        torch.cuda.synchronize()
        before = torch.cuda.memory_stats(dev).get("allocation.all.allocated", 0)
        free_before = torch.cuda.mem_get_info(dev)[0]
        rc = _bwd_noalloc(lib, x, spikes, gs, gv, prm, surrogate, k, gain, gx, gb)
        after = torch.cuda.memory_stats(dev).get("allocation.all.allocated", 0)
        assert rc == 0, lib.spk_last_error().decode()
        assert after == before  # nothing went through torch's allocator
        torch.cuda.synchronize()
        # nor through the driver: the device's free memory is unchanged
        assert torch.cuda.mem_get_info(dev)[0] == free_before
        assert torch.equal(gx, want_gx), (T, N)
        assert torch.equal(gb, want_gb), (T, N, gb.item(), want_gb.item())
    assert lib.spk_device_error_check(None) == 0


def test_noalloc_rejects_sizes_beyond_the_limits():
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    prm = _params(dev)
    x, spikes, gs, gv = _inputs(65, 8, 4)
    gx = torch.empty_like(x)
    gb = torch.empty(1, device=dev)
    rc = _bwd_noalloc(lib, x, spikes, gs, gv, prm, _lib.SURROGATE["superspike"], 4.0, 1.0, gx, gb)
    assert rc == 2  # SPK_ERR_SHAPE
    assert "T=65" in lib.spk_last_error().decode()
