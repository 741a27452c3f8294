"""Leaky integrate-and-fire neuron: drop-in for ``Triton_Layers/Lif.py``.

``LIFLayer`` (autograd function) and ``LIF`` (module) keep the reference's
call signatures, parameter/buffer names and return conventions
(``Lif.py:8-102``, ``Lif.py:288-441``); the scan runs in the sm_100a kernels
of libspk.so (``spk_lif_fwd`` / ``spk_lif_bwd``).

Additions, all defaulting to the reference behaviour:
  * ``surrogate`` ("superspike" | "arctan"); for arctan ``k_superspike`` is
    used as alpha.
  * ``in_gain``: input current scale, ``v = beta*v + in_gain*x``.  A neuron
    written as ``v <- v + (x - v)/tau`` is ``beta = 1 - 1/tau``,
    ``in_gain = 1/tau``.
  * ``LIF.forward`` does not synchronise with the host (the reference calls
    ``k_superspike.item()`` on every call, ``Lif.py:412``); the value is
    cached on the host and refreshed when the state dict is loaded.
"""

from typing import Tuple

import torch
import torch.nn as nn

from . import ops
from ._fused import mark_spike_counts


class LIFLayer(torch.autograd.Function):
    """``apply(input_current[T,B,F], beta, v_th, v_reset, k_superspike
    [, surrogate, in_gain]) -> (spikes fp32 [T,B,F], v_final fp32 [B,F])``.

    Gradients: ``input_current`` (in its own dtype, as ``Lif.py:54``) and
    ``beta`` (summed over neurons, ``Lif.py:95``); none for v_th / v_reset
    (``Lif.py:99-102``).
    """

    @staticmethod
    def forward(ctx, input_current, beta, v_th, v_reset, k_superspike, surrogate="superspike", in_gain=1.0):
        if input_current.dim() != 3:
            raise RuntimeError("LIFLayer expects [T, B, F], got %s" % (tuple(input_current.shape),))
        x = input_current.contiguous()
        spikes, v_final = ops.lif_fwd(x, beta, v_th, v_reset, in_gain, torch.float32)
        ctx.save_for_backward(x, spikes, beta if isinstance(beta, torch.Tensor) else torch.tensor(float(beta)),
                              v_th if isinstance(v_th, torch.Tensor) else torch.tensor(float(v_th)),
                              v_reset if isinstance(v_reset, torch.Tensor) else torch.tensor(float(v_reset)))
        # a tensor k (the reference's LIF module passes a host float) is read
        # back only if the backward runs, never in the forward
        ctx.k = k_superspike
        ctx.surrogate = surrogate
        ctx.in_gain = float(in_gain)
        ctx.mark_non_differentiable(v_final)
        return spikes, v_final

    @staticmethod
    def backward(ctx, grad_output_spikes, grad_v_mem_final):
        x, spikes, beta, v_th, v_reset = ctx.saved_tensors
        need_beta = ctx.needs_input_grad[1]
        k = float(ctx.k)
        gx, gb = ops.lif_bwd(grad_output_spikes, grad_v_mem_final, x, spikes, beta, v_th, v_reset,
                             ctx.in_gain, ctx.surrogate, k, need_beta_grad=need_beta)
        if gb is not None:
            gb = gb.reshape(beta.shape).to(beta.dtype)
        return gx, gb, None, None, None, None, None


class LIF(nn.Module):
    """LIF layer over the t-major fold ``[T*B, ...]`` (``Lif.py:288-441``).

    Args as the reference: beta (0.9), v_th (1.0), v_reset (0.0),
    k_superspike (4.0), n_steps (4), learn_beta, learn_v_th, learn_v_reset;
    plus ``surrogate`` and ``in_gain`` (see the module docstring).
    ``forward(x[T*B, ...]) -> (spikes fp32 same shape, v_final [B, ...])``.
    """

    def __init__(self, beta: float = 0.9, v_th: float = 1.0, v_reset: float = 0.0, k_superspike: float = 4.0,
                 n_steps: int = 4, learn_beta: bool = False, learn_v_th: bool = False,
                 learn_v_reset: bool = False, surrogate: str = "superspike", in_gain: float = 1.0):
        super().__init__()
        self.n_steps = n_steps
        self.learn_beta = learn_beta
        self.learn_v_th = learn_v_th
        self.learn_v_reset = learn_v_reset
        if surrogate not in ("superspike", "arctan"):
            raise ValueError("surrogate must be 'superspike' or 'arctan'")
        self.surrogate = surrogate
        self.in_gain = float(in_gain)
        if learn_beta:
            self.beta_raw = nn.Parameter(torch.tensor(self._inverse_sigmoid(beta)))
        else:
            self.register_buffer("beta", torch.tensor(beta))
        if learn_v_th:
            self.v_th = nn.Parameter(torch.tensor(v_th))
        else:
            self.register_buffer("v_th", torch.tensor(v_th))
        if learn_v_reset:
            self.v_reset = nn.Parameter(torch.tensor(v_reset))
        else:
            self.register_buffer("v_reset", torch.tensor(v_reset))
        self.register_buffer("k_superspike", torch.tensor(k_superspike))
        self._k_host = float(k_superspike)
        self.register_load_state_dict_post_hook(LIF._refresh_host_cache)

    @staticmethod
    def _refresh_host_cache(module, incompatible_keys):
        module._k_host = float(module.k_superspike.detach().cpu())

    @staticmethod
    def _inverse_sigmoid(x: float) -> float:
        """Logit used to initialise ``beta_raw`` (``Lif.py:353-357``)."""
        x = max(min(x, 0.9999), 0.0001)
        return -torch.log(torch.tensor(1.0 / x - 1.0)).item()

    def set_surrogate(self, kind: str, k: float):
        """Backward surrogate: "superspike" (slope k) or "arctan" (alpha k)."""
        if kind not in ("superspike", "arctan"):
            raise ValueError("surrogate must be 'superspike' or 'arctan'")
        self.surrogate = kind
        with torch.no_grad():
            self.k_superspike.fill_(float(k))
        self._k_host = float(k)

    def get_beta(self) -> float:
        if self.learn_beta:
            return torch.sigmoid(self.beta_raw).item()
        return self.beta.item()

    def effective_beta(self) -> torch.Tensor:
        """beta as a 0-dim tensor (``sigmoid(beta_raw)`` when learnable)."""
        return torch.sigmoid(self.beta_raw) if self.learn_beta else self.beta

    def forward(self, input_current: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        shape = input_current.shape
        try:
            x = input_current.reshape(self.n_steps, shape[0] // self.n_steps, *shape[1:])
            x = x.reshape(self.n_steps, shape[0] // self.n_steps, -1)
        except RuntimeError as e:
            raise RuntimeError(
                f"LIF.forward reshape failed: input shape {tuple(shape)}, n_steps={self.n_steps}; "
                f"dim 0 ({shape[0]}) may not be divisible by {self.n_steps}. torch error: {e}")
        spikes, v_final = LIFLayer.apply(x, self.effective_beta(), self.v_th, self.v_reset, self._k_host,
                                         self.surrogate, self.in_gain)
        spikes = spikes.view(shape)
        v_final = v_final.view(shape[0] // self.n_steps, *shape[1:])
        if not spikes.requires_grad:
            mark_spike_counts(spikes)
        return spikes, v_final

    def extra_repr(self) -> str:
        return (f"beta={self.get_beta():.3f} (learnable={self.learn_beta}), "
                f"v_th={self.v_th.item():.3f} (learnable={self.learn_v_th}), "
                f"v_reset={self.v_reset.item():.3f} (learnable={self.learn_v_reset}), "
                f"k_superspike={self.k_superspike.item():.1f}")
