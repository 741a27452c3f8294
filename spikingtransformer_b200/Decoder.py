"""Decoder stack: drop-in for ``Triton_Layers/Decoder.py``.

``DecoderLayer``: masked self-SSA, cross-SSA against the encoder output
(no mask), MLP, each added to the residual stream (``Decoder.py:4-26``).
``Decoder``: ``num_layers`` of them (``:28-43``).
"""

import torch.nn as nn

from ._fused import fast_path_ok, spike_counts_bf16
from .Encoder import stream_copy_bf16, stream_out
from .SSA import SSAMultiHeadAttention
from .SpikingMLP import SpikingMLP


def _fast_inputs(module, x, enc_output, mask):
    """(private bf16 copy of x, bf16 encoder output) for the fused path, or
    (None, None) when either may not be exact in bf16."""
    if not fast_path_ok(x, enc_output, mask, module=module):
        return None, None
    enc = spike_counts_bf16(enc_output)
    if enc is None:
        return None, None
    xb = stream_copy_bf16(x)
    return (xb, enc.contiguous()) if xb is not None else (None, None)


class DecoderLayer(nn.Module):
    def __init__(self, d_model, n_heads, ff_dim, dropout=0.1, alpha=0.125, n_steps=10):
        super().__init__()
        self.self_attns = SSAMultiHeadAttention(d_model=d_model, n_heads=n_heads, dropout=dropout, alpha=alpha,
                                                n_steps=n_steps)
        self.cross_attns = SSAMultiHeadAttention(d_model=d_model, n_heads=n_heads, dropout=dropout, alpha=alpha,
                                                 n_steps=n_steps)
        self.mlp = SpikingMLP(d_model=d_model, ff_dim=ff_dim, n_steps=n_steps)

    def _fast(self, x, enc, mask=None, cross_kv=None):
        """In place on the bf16 residual stream ``x``; ``enc`` bf16 encoder output;
        ``cross_kv``: the cross-attention's (K, V) spikes of ``enc``, if cached."""
        self.self_attns._fast(x, None, mask)
        self.cross_attns._fast(x, enc, None, kv_spikes=cross_kv)
        self.mlp._fast(x)
        return x

    def forward(self, x, enc_output, mask=None):
        xb, enc = _fast_inputs(self, x, enc_output, mask)
        if xb is not None:
            return stream_out(self._fast(xb, enc, mask), x)
        x = self.self_attns.add_to(x, x, x, attention_mask=mask)
        x = self.cross_attns.add_to(x, enc_output, enc_output)
        return self.mlp.add_to(x)


class Decoder(nn.Module):
    def __init__(self, num_layers, d_model, n_heads, ff_dim, dropout=0.1, alpha=0.125, n_steps=10):
        super().__init__()
        self.layers = nn.ModuleList([
            DecoderLayer(d_model=d_model, n_heads=n_heads, ff_dim=ff_dim, dropout=dropout, alpha=alpha,
                         n_steps=n_steps) for _ in range(num_layers)])

    def cross_key_values(self, enc):
        """Per layer, the cross-attention (K, V) spikes of the bf16 encoder output."""
        return [layer.cross_attns.key_value_spikes(enc) for layer in self.layers]

    def _fast(self, x, enc, mask=None, cross_kv=None):
        for i, layer in enumerate(self.layers):
            layer._fast(x, enc, mask, None if cross_kv is None else cross_kv[i])
        return x

    def forward(self, x, enc_output, mask=None):
        xb, enc = _fast_inputs(self, x, enc_output, mask)
        if xb is not None:
            return stream_out(self._fast(xb, enc, mask), x)
        for layer in self.layers:
            x = layer(x, enc_output, mask=mask)
        return x
