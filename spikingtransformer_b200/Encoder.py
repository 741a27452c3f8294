"""Encoder stack: drop-in for ``Triton_Layers/Encoder.py``.

``EncoderLayer``: ``x = x + SSA(x, x, x, mask)``; ``x = x + MLP(x)``
(``Encoder.py:6-24``).  ``Encoder``: ``num_layers`` of them (``:26-41``).

Inference keeps the residual stream as bf16 spike counts (exact: the stream
is a sum of spikes) and the fused kernels add each block's output spikes into
a copy of it in place.  The stream takes that path when it is bf16 or was
produced by this package's spiking modules (known without reading it back to
the host); any other stream takes the per-module path with an fp32 residual.
"""

import torch
import torch.nn as nn

from ._fused import fast_path_ok, mark_spike_counts, spike_counts_bf16
from .SSA import SSAMultiHeadAttention
from .SpikingMLP import SpikingMLP


def stream_copy_bf16(x):
    """A private contiguous bf16 copy of the residual stream ``x`` for the
    in-place fused path, or None when ``x`` may not be exact in bf16."""
    xb = spike_counts_bf16(x)
    if xb is None:
        return None
    return xb.clone(memory_format=torch.contiguous_format)


def stream_out(out_bf16, like):
    """The fused path's result in the caller's dtype, marked as spike counts."""
    if like.dtype == torch.bfloat16:
        return out_bf16
    return mark_spike_counts(out_bf16.to(like.dtype), out_bf16)


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
        xb = stream_copy_bf16(x) if fast_path_ok(x, mask, module=self) else None
        if xb is not None:
            return stream_out(self._fast(xb, mask), x)
        x = self.self_attns.add_to(x, x, x, attention_mask=mask)
        return self.mlp.add_to(x)


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
        xb = stream_copy_bf16(x) if fast_path_ok(x, mask, module=self) else None
        if xb is not None:
            return stream_out(self._fast(xb, mask), x)
        for layer in self.layers:
            x = layer(x, mask=mask)
        return x
