"""Spiking OCR seq2seq model: drop-in for ``Triton_Layers/Seq2Seq.py``.

``Seq2Seq(patch_size, d_model, n_heads, ff_dim, num_encoder_layers,
num_decoder_layers, dropout, alpha, tgt_vocab_size, nb_sps_blocks, n_steps)``
with the reference's submodule names (image_encoder, encoder, decoder,
output_layer, lifPE, tgt_tok_emb, positional_encoding) and methods
(``forward -> (logits [T,B,N,V], None)``, ``encode``, ``decode``, mask
helpers, ``greedy_decode``), ``Seq2Seq.py:39-162``.  One added keyword,
``image_encoder="cnn"`` (reference ``CNNBackbone``) or ``"patch"``
(``PatchEmbed``, the 16x16 patch embedding of the OCR benchmark), and
``in_chans`` for the patch encoder.

Inference (no autograd graph) runs the whole forward on the fused kernels:
the image and token inputs repeated over T are computed once and fed to the
LIF at every step; the encoder / decoder residual streams stay bf16 spike
counts on the device; only the logits are fp32.
"""

import math

import torch
import torch.nn as nn
from torch import Tensor

from . import ops
from ._fused import bf16_weight, fast_path_ok, lif_params, mark_spike_counts, spike_counts_bf16
from .Decoder import Decoder
from .Encoder import Encoder
from .ImageEncoder import CNNBackbone, PatchEmbed
from .Lif import LIF


class PositionalEncoding(nn.Module):
    """Sinusoidal positions (``Seq2Seq.py:11-26``), buffer ``pos_embedding [1, maxlen, E]``."""

    def __init__(self, emb_size: int, dropout: float, maxlen: int = 5000):
        super().__init__()
        den = torch.exp(-torch.arange(0, emb_size, 2) * math.log(10000) / emb_size)
        pos = torch.arange(0, maxlen).reshape(maxlen, 1)
        table = torch.zeros((maxlen, emb_size))
        table[:, 0::2] = torch.sin(pos * den)
        table[:, 1::2] = torch.cos(pos * den)
        self.dropout = nn.Dropout(dropout)
        self.register_buffer("pos_embedding", table.unsqueeze(0))

    def forward(self, token_embedding: Tensor):
        return self.dropout(token_embedding + self.pos_embedding[:, : token_embedding.size(1)])


class TokenEmbedding(nn.Module):
    """``Seq2Seq.py:29-36``: ``embedding(tokens) * sqrt(emb_size)``."""

    def __init__(self, vocab_size: int, emb_size: int):
        super().__init__()
        self.embedding = nn.Embedding(vocab_size, emb_size)
        self.emb_size = emb_size

    def forward(self, tokens: Tensor):
        return self.embedding(tokens.long()) * math.sqrt(self.emb_size)


class Seq2Seq(nn.Module):
    def __init__(self, patch_size=16, d_model=512, n_heads=8, ff_dim=2048, num_encoder_layers=6,
                 num_decoder_layers=6, dropout=0.1, alpha=0.125, tgt_vocab_size=1000, nb_sps_blocks=4, n_steps=10,
                 image_encoder="cnn", in_chans=1):
        super().__init__()
        self.n_steps = n_steps
        if image_encoder == "cnn":
            self.image_encoder = CNNBackbone(nb_layers=nb_sps_blocks, patch_size=patch_size, d_model=d_model,
                                             n_steps=n_steps)
        elif image_encoder == "patch":
            self.image_encoder = PatchEmbed(d_model=d_model, patch_size=patch_size, n_steps=n_steps,
                                            in_chans=in_chans)
        else:
            raise ValueError("image_encoder must be 'cnn' or 'patch'")
        self.encoder = Encoder(num_layers=num_encoder_layers, d_model=d_model, n_heads=n_heads, ff_dim=ff_dim,
                               dropout=dropout, alpha=alpha, n_steps=n_steps)
        self.decoder = Decoder(num_layers=num_decoder_layers, d_model=d_model, n_heads=n_heads, ff_dim=ff_dim,
                               dropout=dropout, alpha=alpha, n_steps=n_steps)
        self.output_layer = nn.Linear(d_model, tgt_vocab_size)
        self.lifPE = LIF(n_steps=n_steps)
        self.tgt_tok_emb = TokenEmbedding(tgt_vocab_size, d_model)
        self.positional_encoding = PositionalEncoding(d_model, dropout=dropout)

    # ---------------------------------------------------------------- surrogate selection

    def set_surrogate(self, kind: str, k: float):
        """Select the backward surrogate of every LIF ("superspike" with slope
        k, or "arctan" with alpha k)."""
        for m in self.modules():
            if isinstance(m, LIF):
                m.set_surrogate(kind, k)

    # ---------------------------------------------------------------- fused inference path

    def _fast_ok(self, *ts):
        dropout_active = self.training and self.positional_encoding.dropout.p > 0
        return not dropout_active and fast_path_ok(*ts, module=self)

    def _encode_fast(self, src):
        """bf16 encoder output [T*B, Ns, D] for images src [B, C, H, W]."""
        T = self.n_steps
        if isinstance(self.image_encoder, PatchEmbed):
            x = self.image_encoder.encode_images(src)
        elif self.image_encoder._fast_ok(src):
            x = self.image_encoder.encode_images(src, T)
        else:
            B = src.shape[0]
            src_t = src.unsqueeze(0).expand(T, *src.shape).reshape(T * B, *src.shape[1:])
            x = self.image_encoder(src_t)[0].to(torch.bfloat16).contiguous()
        return self.encoder._fast(x)

    def _decode_fast(self, tgt, enc, look_ahead_mask, cross_kv=None):
        T = self.n_steps
        emb = self.tgt_tok_emb
        p = lif_params(self.lifPE)
        y, _ = ops.embed_pe_lif(tgt, emb.embedding.weight, math.sqrt(emb.emb_size),
                                self.positional_encoding.pos_embedding, p[0:1], p[1:2], p[2:3], T,
                                in_gain=self.lifPE.in_gain)
        mask = None
        if look_ahead_mask is not None:
            B, N = tgt.shape
            H = self.decoder.layers[0].self_attns.n_heads if len(self.decoder.layers) else 1
            mask = ops.mask_to_u8(look_ahead_mask, T, B, H, N, N)
        self.decoder._fast(y, enc, mask, cross_kv)
        D = y.shape[-1]
        logits = ops.linear(y.view(-1, D), bf16_weight(self.output_layer), self.output_layer.bias)
        return logits.view(T, -1, tgt.shape[1], logits.shape[-1])

    # ---------------------------------------------------------------- reference API

    def forward(self, src, tgt, look_ahead_mask: Tensor = None, enc_padding_mask: Tensor = None,
                dec_padding_mask: Tensor = None):
        if self._fast_ok(src, tgt, look_ahead_mask):
            enc = self._encode_fast(src)
            return self._decode_fast(tgt, enc, look_ahead_mask), None
        enc_output, _ = self.encode(src)
        return self.decode(tgt, enc_output, look_ahead_mask, enc_padding_mask, dec_padding_mask)

    def encode(self, src: Tensor):
        if self._fast_ok(src):
            enc = self._encode_fast(src)
            return mark_spike_counts(enc.float(), enc), None
        B = src.shape[0]
        T = self.n_steps
        if isinstance(self.image_encoder, PatchEmbed):
            enc_output, _ = self.image_encoder.forward_repeated(src, T)
        else:
            src = src.unsqueeze(0).expand(T, *src.shape).reshape(T * B, *src.shape[1:])
            enc_output, _ = self.image_encoder(src)
        return self.encoder(enc_output), None

    def decode(self, tgt: Tensor, enc_output: Tensor, look_ahead_mask: Tensor = None,
               enc_padding_mask: Tensor = None, dec_padding_mask: Tensor = None):
        enc = spike_counts_bf16(enc_output) if self._fast_ok(tgt, enc_output, look_ahead_mask) else None
        if enc is not None:
            return self._decode_fast(tgt, enc.contiguous(), look_ahead_mask), None
        T = self.n_steps
        if look_ahead_mask is not None:
            m = look_ahead_mask
            look_ahead_mask = m.unsqueeze(0).repeat(T, 1, 1, 1, 1).reshape(T * m.shape[0], *m.shape[1:])
        y = self.positional_encoding(self.tgt_tok_emb(tgt))
        B, N, D = y.shape
        y = y.unsqueeze(0).expand(T, B, N, D).reshape(T * B, N, D)
        y, _ = self.lifPE(y)
        y = self.decoder(y, enc_output, mask=look_ahead_mask)
        out = self.output_layer(y)
        return out.view(T, out.shape[0] // T, out.shape[1], out.shape[2]), None

    def create_padding_mask(self, seq: Tensor, pad_idx: int, device) -> Tensor:
        return torch.where(seq == pad_idx, 0.0, 1.0).unsqueeze(1).unsqueeze(1).to(device)

    def create_look_ahead_mask(self, size: int, device) -> Tensor:
        return torch.tril(torch.ones((size, size), device=device))

    def create_decoder_mask(self, tgt: Tensor, pad_idx: int, device) -> Tensor:
        look_ahead = self.create_look_ahead_mask(tgt.shape[1], device)
        pad = self.create_padding_mask(tgt, pad_idx, device)
        return torch.minimum(pad, look_ahead)

    @torch.no_grad()
    def greedy_decode(self, src: Tensor, max_len: int, start_symbol: int, eos_idx: int, pad_idx: int,
                      device: str = "cuda"):
        """Greedy decoding as ``Seq2Seq.py:136-162``: re-decodes the prefix each
        step, picks argmax of the T-averaged logits of the last position.

        The whole prefix is decoded every step because the self-attention's
        log-distance bias is normalised by the current length, so earlier
        positions change as the sequence grows.  On the fused path the
        cross-attention K/V spikes of the fixed encoder output are computed
        once and reused by every step (the same values each step would
        compute)."""
        if src.dim() == 3:
            src = src.unsqueeze(0)
        src = src.to(device)
        fast = self._fast_ok(src)
        if fast:
            enc = self._encode_fast(src)
            cross_kv = self.decoder.cross_key_values(enc)
            attention_rec = None
        else:
            memory, attention_rec = self.encode(src)
        ys = torch.full((1, 1), fill_value=start_symbol, dtype=torch.long, device=device)
        out = None
        for _ in range(max_len - 1):
            tgt_mask = self.create_decoder_mask(ys, pad_idx, device)
            if fast:
                out = self._decode_fast(ys, enc, tgt_mask, cross_kv)
            else:
                out, _ = self.decode(ys, memory, tgt_mask)
            prob = out.mean(dim=0)
            next_token_id = torch.argmax(prob[:, -1, :], dim=-1).item()
            ys = torch.cat([ys, torch.tensor([[next_token_id]], device=device, dtype=torch.long)], dim=1)
            if next_token_id == eos_idx:
                break
        return ys, attention_rec, out

    @torch.no_grad()
    def greedy_decode_batch(self, src: Tensor, max_len: int, start_symbol: int, eos_idx: int, pad_idx: int,
                            device: str = "cuda"):
        """Greedy decoding of a batch of images ``src`` [B, C, H, W] in one
        pass per step.

        Every operation is per image and all sequences share the current
        length, so row b of the result is exactly what ``greedy_decode``
        returns for image b alone.  Decoding continues until every row has
        produced ``eos_idx`` (or ``max_len`` tokens); positions after a row's
        eos are set to ``pad_idx``.  Returns ``(ys [B, L], lengths [B])``,
        ``lengths`` counting the start symbol and the eos.
        """
        if src.dim() == 3:
            src = src.unsqueeze(0)
        src = src.to(device)
        B = src.shape[0]
        fast = self._fast_ok(src)
        if fast:
            enc = self._encode_fast(src)
            cross_kv = self.decoder.cross_key_values(enc)
        else:
            memory, _ = self.encode(src)
        ys = torch.full((B, 1), fill_value=start_symbol, dtype=torch.long, device=device)
        done = torch.zeros(B, dtype=torch.bool, device=device)
        lengths = torch.full((B,), max_len, dtype=torch.long, device=device)
        for n in range(1, max_len):
            tgt_mask = self.create_decoder_mask(ys, pad_idx, device)
            if fast:
                out = self._decode_fast(ys, enc, tgt_mask, cross_kv)
            else:
                out, _ = self.decode(ys, memory, tgt_mask)
            nxt = torch.argmax(out.mean(dim=0)[:, -1, :], dim=-1)
            hit = (nxt == eos_idx) & ~done
            lengths = torch.where(hit, torch.full_like(lengths, n + 1), lengths)
            ys = torch.cat([ys, nxt.unsqueeze(1)], dim=1)
            done = done | hit
            if bool(done.all()):
                break
        pos = torch.arange(ys.shape[1], device=device).unsqueeze(0)
        ys = torch.where(pos < lengths.clamp(max=ys.shape[1]).unsqueeze(1), ys, torch.full_like(ys, pad_idx))
        return ys, lengths.clamp(max=ys.shape[1])
