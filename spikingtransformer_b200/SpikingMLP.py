"""Spiking MLP: drop-in for ``Triton_Layers/SpikingMLP.py``.

``SpikingMLP(d_model, ff_dim, n_steps)``: expand Linear(D, F) -> bn_expand
LayerNorm(F) -> lifexpand LIF (learnable beta) -> compress Linear(F, D) ->
bn_compress LayerNorm(D) -> lifcompress LIF (``SpikingMLP.py:4-37``).  No
residual inside (the residual lives in the encoder / decoder layers).

Inference runs the two fused Linear->LN->LIF kernels; the hidden spikes stay
bf16 and never pass through fp32.
"""

import torch.nn as nn
import torch

from ._fused import fast_path_ok, lin_ln_lif, lin_ln_lif_train, mark_spike_counts
from .Lif import LIF


class SpikingMLP(nn.Module):
    def __init__(self, d_model, ff_dim, n_steps=1):
        super().__init__()
        self.n_steps = n_steps
        self.expand = nn.Linear(d_model, ff_dim)
        self.compress = nn.Linear(ff_dim, d_model)
        self.lifexpand = LIF(n_steps=n_steps, learn_beta=True)
        self.lifcompress = LIF(n_steps=n_steps, learn_beta=True)
        self.bn_expand = nn.LayerNorm(ff_dim)
        self.bn_compress = nn.LayerNorm(d_model)

    def _fast(self, x):
        """``x += MLP(x)`` in place on bf16 spike counts ``[T*B, N, D]``."""
        T = self.lifexpand.n_steps
        D = x.shape[-1]
        h = lin_ln_lif(x, self.expand, self.bn_expand, self.lifexpand, T)[0]
        lin_ln_lif(h, self.compress, self.bn_compress, self.lifcompress, T, residual=x.view(-1, D),
                   want_spikes=False)
        return x

    def forward(self, x):
        if fast_path_ok(x, module=self):
            T = self.lifexpand.n_steps
            h = lin_ln_lif(x, self.expand, self.bn_expand, self.lifexpand, T)[0]
            y = lin_ln_lif(h, self.compress, self.bn_compress, self.lifcompress, T, spike_dtype=torch.float32)[0]
            return mark_spike_counts(y.view(*x.shape[:-1], y.shape[-1]))
        # the hidden spikes feed only the compress GEMM: autocast dtype under autocast
        h = lin_ln_lif_train(x, self.expand, self.bn_expand, self.lifexpand, narrow=True)
        return lin_ln_lif_train(h, self.compress, self.bn_compress, self.lifcompress)

    def add_to(self, x):
        """``x + self(x)``, the residual connection of an encoder / decoder layer
        (``Encoder.py:22``, ``Decoder.py:24``); on the autograd path the add is
        fused into the compress LayerNorm->LIF kernel."""
        if fast_path_ok(x, module=self):
            return x + self(x)
        h = lin_ln_lif_train(x, self.expand, self.bn_expand, self.lifexpand, narrow=True)
        return lin_ln_lif_train(h, self.compress, self.bn_compress, self.lifcompress, residual=x)
