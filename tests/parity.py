"""Comparison rules shared by the parity tests.

* Spike trains: bit-exact, except for a neuron whose reference membrane came
  within ``SPIKE_TOL`` (1e-4) of the threshold at some step; from that step on
  its train is exempt (a flipped spike changes the reset, so the rest of the
  train legitimately diverges).
* Membrane potentials and LayerNorm outputs: within ``REL_TOL`` (1e-3)
  relative, measured against ``max(|ref|, 1)`` so values near zero are
  compared on an absolute 1e-3 scale.
* Integer spike-count products (SSA): bit-exact.
"""

import torch

SPIKE_TOL = 1e-4
REL_TOL = 1e-3


def membrane_history(x3, beta, v_th, v_reset, in_gain=1.0):
    """Pre-reset membrane per step for ``x3 [T, B, F]`` (fp32, oracle order)."""
    x3 = x3.detach().to(torch.float32).cpu()
    beta = float(beta.detach()) if isinstance(beta, torch.Tensor) else float(beta)
    v = torch.zeros_like(x3[0])
    hist = torch.empty_like(x3)
    for t in range(x3.shape[0]):
        cur = x3[t] if in_gain == 1.0 else x3[t] * in_gain
        v = v * beta + cur
        hist[t] = v
        v = torch.where(v > v_th, torch.full_like(v, float(v_reset)), v)
    return hist


def exempt_mask(v_hist, v_th, tol=SPIKE_TOL):
    """True where a spike comparison is exempt (near-threshold at or before t)."""
    near = (v_hist - float(v_th)).abs() < tol
    return torch.cummax(near.to(torch.int8), dim=0).values.bool()


def assert_spikes_match(ours, ref, v_hist=None, v_th=None, max_exempt_frac=0.01, what="spikes"):
    ours = ours.detach().to(torch.float32).cpu()
    ref = ref.detach().to(torch.float32).cpu()
    assert ours.shape == ref.shape, (what, ours.shape, ref.shape)
    bad = ours != ref
    if v_hist is not None:
        ex = exempt_mask(v_hist, v_th).reshape(bad.shape)
        frac = ex.float().mean().item()
        assert frac <= max_exempt_frac, f"{what}: {frac:.4f} of neurons near threshold"
        bad = bad & ~ex
    n = int(bad.sum())
    assert n == 0, f"{what}: {n} of {bad.numel()} spikes differ outside the near-threshold band"


def assert_close_rel(ours, ref, tol=REL_TOL, what="value"):
    ours = ours.detach().to(torch.float32).cpu()
    ref = ref.detach().to(torch.float32).cpu()
    assert ours.shape == ref.shape, (what, ours.shape, ref.shape)
    err = (ours - ref).abs() / ref.abs().clamp(min=1.0)
    worst = err.max().item() if err.numel() else 0.0
    assert worst <= tol, f"{what}: max relative error {worst:.3e} > {tol:.1e}"


def spike_mismatch_rate(a, b):
    a = a.detach().to(torch.float32).cpu()
    b = b.detach().to(torch.float32).cpu()
    return (a != b).float().mean().item()
