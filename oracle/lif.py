"""LIF temporal scan, forward and backward, restated on the CPU in fp32.

Test infrastructure only (see ``oracle/__init__.py``).

Reference: ``Triton_Layers/Lif.py``
  * forward recurrence  ``Lif.py:149-165``  (v0 = 0; v = v*beta + x[t];
    s = v > v_th; v = s ? v_reset : v; v_final stored after the last step)
  * backward            ``Lif.py:221-276``  (recompute pre-reset membrane,
    reverse sweep with the SuperSpike surrogate ``Lif.py:280-282``)
  * grad_beta reduction ``Lif.py:95`` (sum over all neurons)

Every arithmetic step below is a separate fp32 operation in the order the
reference writes it (``v*beta`` rounded, then ``+ x`` rounded), which is how
the reference kernel evaluates when run by the Triton interpreter; the fixtures
in ``tests/golden`` pin this bit-for-bit.

Extension beyond the reference: ``in_gain`` scales
the input current before integration, ``v = beta*v + in_gain*x``.  With
``in_gain == 1`` the computation is exactly the reference one.  The
``tau``-parameterised neuron ``v <- v + (x - v)/tau`` maps to
``beta = 1 - 1/tau``, ``in_gain = 1/tau``.
"""

import math

import torch


def _scalar(v):
    if isinstance(v, torch.Tensor):
        return v.detach().to(torch.float32).reshape(())
    return torch.tensor(float(v), dtype=torch.float32)


def lif_forward(x, beta, v_th, v_reset, in_gain=1.0):
    """Forward scan.  ``x`` is ``[T, B, F]``; returns fp32 ``(spikes, v_final)``.

    Follows ``Lif.py:149-165``.
    """
    x = x.detach().to(torch.float32)
    beta, v_th, v_reset = _scalar(beta), _scalar(v_th), _scalar(v_reset)
    g = float(in_gain)
    T = x.shape[0]
    v = torch.zeros_like(x[0])
    spikes = torch.empty_like(x)
    for t in range(T):
        cur = x[t] if g == 1.0 else x[t] * g
        v = v * beta + cur
        s = v > v_th
        spikes[t] = s.to(torch.float32)
        v = torch.where(s, v_reset, v)
    return spikes, v


def superspike_grad(v_minus_th, k):
    """SuperSpike surrogate ``1/(1+k|u|)/(1+k|u|)`` (``Lif.py:280-282``)."""
    a = 1.0 + k * v_minus_th.abs()
    return 1.0 / a / a


def arctan_grad(v_minus_th, alpha):
    """Arctan surrogate ``(alpha/2) / (1 + (pi/2 * alpha * u)^2)``.

    This is the derivative of ``atan(pi/2 * alpha * u)/pi + 1/2``; the
    reference has no arctan path, the formula is written from its mathematics.
    """
    z = (math.pi / 2.0 * alpha) * v_minus_th
    return (alpha / 2.0) / (1.0 + z * z)


def lif_backward(grad_spikes, grad_v_final, x, spikes, beta, v_th, v_reset,
                 k=4.0, in_gain=1.0, surrogate="superspike"):
    """Backward through the scan.  Returns ``(grad_x fp32, grad_beta scalar)``.

    Follows ``Lif.py:221-276``: pass 1 recomputes the pre-reset membrane
    ``v_hist[t]`` using the forward spikes for the reset; pass 2 walks t from
    T-1 down to 0 with ``g_v = g_s[t]*sg(v_hist[t]-v_th) + (s[t] ? 0 : g_state)``,
    ``grad_beta += g_v * v_post[t-1]`` (``v_post[-1] = v_init = 0``) and
    ``g_state = g_v * beta``.  ``grad_v_final`` seeds ``g_state``
    (``Lif.py:236``).  With ``in_gain`` the input gradient is ``in_gain*g_v``.
    """
    x = x.detach().to(torch.float32)
    spikes = spikes.detach().to(torch.float32)
    gs = grad_spikes.detach().to(torch.float32)
    beta, v_th, v_reset = _scalar(beta), _scalar(v_th), _scalar(v_reset)
    g = float(in_gain)
    T = x.shape[0]
    v = torch.zeros_like(x[0])
    v_hist = torch.empty_like(x)
    for t in range(T):
        cur = x[t] if g == 1.0 else x[t] * g
        v = v * beta + cur
        v_hist[t] = v
        v = torch.where(spikes[t] > 0.0, v_reset, v)
    if grad_v_final is None:
        g_state = torch.zeros_like(x[0])
    else:
        g_state = grad_v_final.detach().to(torch.float32).clone()
    grad_beta_acc = torch.zeros_like(x[0])
    grad_x = torch.empty_like(x)
    for t in range(T - 1, -1, -1):
        u = v_hist[t] - v_th
        if surrogate == "superspike":
            sg = superspike_grad(u, float(k))
        elif surrogate == "arctan":
            sg = arctan_grad(u, float(k))
        else:
            raise ValueError(surrogate)
        from_state = torch.where(spikes[t] > 0.0, torch.zeros_like(g_state), g_state)
        g_v = gs[t] * sg + from_state
        grad_x[t] = g_v if g == 1.0 else g_v * g
        if t > 0:
            v_prev = torch.where(spikes[t - 1] > 0.0, v_reset, v_hist[t - 1])
        else:
            v_prev = torch.zeros_like(g_v)
        grad_beta_acc = grad_beta_acc + g_v * v_prev
        g_state = g_v * beta
    return grad_x, grad_beta_acc.sum()


class LIFFunction(torch.autograd.Function):
    """Autograd wrapper around the restated scan (mirrors ``Lif.py:8-102``)."""

    @staticmethod
    def forward(ctx, x, beta, v_th, v_reset, k, surrogate="superspike", in_gain=1.0):
        s, vf = lif_forward(x, beta, v_th, v_reset, in_gain)
        ctx.save_for_backward(x, s, beta, v_th, v_reset)
        ctx.k = float(k)
        ctx.surrogate = surrogate
        ctx.in_gain = float(in_gain)
        return s, vf

    @staticmethod
    def backward(ctx, g_s, g_vf):
        x, s, beta, v_th, v_reset = ctx.saved_tensors
        gx, gb = lif_backward(g_s, g_vf, x, s, beta, v_th, v_reset, ctx.k,
                              ctx.in_gain, ctx.surrogate)
        gb = gb.reshape(beta.shape) if isinstance(beta, torch.Tensor) else gb
        return gx.to(x.dtype), gb, None, None, None, None, None
