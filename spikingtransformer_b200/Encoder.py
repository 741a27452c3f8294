"""Encoder stack: drop-in for ``Triton_Layers/Encoder.py``.

``EncoderLayer``: ``x = x + SSA(x, x, x, mask)``; ``x = x + MLP(x)``
(``Encoder.py:6-24``).  ``Encoder``: ``num_layers`` of them (``:26-41``).

Inference keeps the residual stream as bf16 spike counts (exact: the stream
is a sum of spikes) and the fused kernels add each block's output spikes into
it in place.  A stream that is not exactly representable in bf16 takes the
per-module path with an fp32 residual instead.
"""

import torch
import torch.nn as nn

from ._fused import fast_path_ok
from .SSA import SSAMultiHeadAttention
from .SpikingMLP import SpikingMLP


def bf16_exact(x):
    """True if every element of ``x`` is exactly representable in bf16."""
    if x.dtype == torch.bfloat16:
        return True
    return bool(torch.equal(x.to(torch.bfloat16).to(x.dtype), x))


class EncoderLayer(nn.Module):
    def __init__(self, d_model, n_heads, ff_dim, dropout=0.1, alpha=0.125, n_steps=10):
        super().__init__()
        self.self_attns = SSAMultiHeadAttention(d_model=d_model, n_heads=n_heads, dropout=dropout, alpha=alpha,
                                                n_steps=n_steps)
        self.mlp = SpikingMLP(d_model=d_model, ff_dim=ff_dim, n_steps=n_steps)

    def _fast(self, x, mask=None):
        """In place on the bf16 residual stream ``x [T*B, N, D]``."""
        self.self_attns._fast(x, None, mask)
        self.mlp._fast(x)
        return x

    def forward(self, x, mask=None):
        if fast_path_ok(x, mask, module=self) and bf16_exact(x):
            out = self._fast(x.to(torch.bfloat16).contiguous(), mask)
            return out.to(x.dtype)
        x = x + self.self_attns(x, x, x, attention_mask=mask)
        return x + self.mlp(x)


class Encoder(nn.Module):
    def __init__(self, num_layers, d_model, n_heads, ff_dim, dropout=0.1, alpha=0.125, n_steps=10):
        super().__init__()
        self.layers = nn.ModuleList([
            EncoderLayer(d_model=d_model, n_heads=n_heads, ff_dim=ff_dim, dropout=dropout, alpha=alpha,
                         n_steps=n_steps) for _ in range(num_layers)])

    def _fast(self, x, mask=None):
        for layer in self.layers:
            layer._fast(x, mask)
        return x

    def forward(self, x, mask=None):
        if fast_path_ok(x, mask, module=self) and bf16_exact(x):
            return self._fast(x.to(torch.bfloat16).contiguous(), mask).to(x.dtype)
        for layer in self.layers:
            x = layer(x, mask=mask)
        return x
