"""CPU fp32 restatement of the reference spiking modules (test infrastructure only).

Each class keeps the reference's submodule, parameter and buffer names so a
state dict moves unchanged between the reference, this oracle and the CUDA
package.  Citations are ``file:line`` inside flofiz/SpikingTransformer.

Only the LIF scan is re-derived (``oracle/lif.py``); everything else in the
reference is stock torch arithmetic (Linear, LayerNorm, einsum, conv), which
is restated here with the same operation order on fp32 CPU tensors.
"""

import math
from typing import Optional

import torch
from torch import nn
import torch.nn.functional as F

from .lif import LIFFunction


def _inverse_sigmoid(p):
    # Lif.py:353-357: clamp to [1e-4, 0.9999], then -log(1/p - 1) in fp32
    p = max(min(p, 0.9999), 0.0001)
    return -torch.log(torch.tensor(1.0 / p - 1.0)).item()


class LIF(nn.Module):
    """Reference ``LIF`` module (``Lif.py:288-441``) over the restated scan.

    Extra keyword ``surrogate`` ("superspike" | "arctan") selects the backward
    surrogate; ``k_superspike`` is used as the arctan ``alpha`` in that case.
    ``in_gain`` scales the input current (1.0 = reference behaviour).
    """

    def __init__(self, beta=0.9, v_th=1.0, v_reset=0.0, k_superspike=4.0,
                 n_steps=4, learn_beta=False, learn_v_th=False,
                 learn_v_reset=False, surrogate="superspike", in_gain=1.0):
        super().__init__()
        self.n_steps = n_steps
        self.learn_beta = learn_beta
        self.learn_v_th = learn_v_th
        self.learn_v_reset = learn_v_reset
        self.surrogate = surrogate
        self.in_gain = float(in_gain)
        if learn_beta:
            self.beta_raw = nn.Parameter(torch.tensor(_inverse_sigmoid(beta)))
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

    def effective_beta(self):
        return torch.sigmoid(self.beta_raw) if self.learn_beta else self.beta

    def forward(self, x):
        # Lif.py:383-427: [T*B, ...] -> [T, B, prod(...)] -> scan -> back
        shape = x.shape
        T = self.n_steps
        if shape[0] % T != 0:
            raise RuntimeError(f"LIF reshape: first dim {shape[0]} not divisible by n_steps={T}")
        x3 = x.reshape(T, shape[0] // T, -1)
        s, vf = LIFFunction.apply(x3, self.effective_beta(), self.v_th, self.v_reset,
                                  float(self.k_superspike), self.surrogate, self.in_gain)
        return s.view(shape), vf.view(shape[0] // T, *shape[1:])


def log_pe_bias(nq, nk):
    """Log-distance bias ``max(0, ceil(log2((max(nq,nk)-1)/(|i-j|+1))))``.

    Restates ``SSA.py:177-201`` (fp32 arithmetic, as the reference).
    """
    iq = torch.arange(nq).unsqueeze(1)
    jk = torch.arange(nk).unsqueeze(0)
    dist = (iq - jk).abs().float()
    L = max(nq, nk)
    return torch.ceil(torch.log2((L - 1) / (dist + 1))).clamp(min=0)


class _SSABase(nn.Module):
    def __init__(self, d_model, n_heads, n_steps, bias):
        super().__init__()
        self.d_model = d_model
        self.n_heads = n_heads
        self.d_head = d_model // n_heads
        self.q_proj = nn.Linear(d_model, d_model, bias=bias)
        self.k_proj = nn.Linear(d_model, d_model, bias=bias)
        self.v_proj = nn.Linear(d_model, d_model, bias=bias)
        self.lnq = nn.LayerNorm(d_model)
        self.lnk = nn.LayerNorm(d_model)
        self.lnv = nn.LayerNorm(d_model)
        self.lno = nn.LayerNorm(d_model)
        self.lifq = LIF(n_steps=n_steps)
        self.lifk = LIF(n_steps=n_steps)
        self.lifv = LIF(n_steps=n_steps)
        self.lifs = LIF(n_steps=n_steps, v_th=0.5)
        self.lifo = LIF(n_steps=n_steps)
        self.out_proj = nn.Linear(d_model, d_model, bias=bias)

    def _project(self, query, key, value):
        # SSA.py:218-232 (and :65-79): Linear -> LayerNorm -> LIF, split heads
        B, N, D = query.shape
        Nk = key.shape[1]
        H, dh = self.n_heads, self.d_head
        q = self.lifq(self.lnq(self.q_proj(query)))[0]
        k = self.lifk(self.lnk(self.k_proj(key)))[0]
        v = self.lifv(self.lnv(self.v_proj(value)))[0]
        q = q.view(B, N, H, dh).transpose(1, 2)
        k = k.view(B, Nk, H, dh).transpose(1, 2)
        v = v.view(B, Nk, H, dh).transpose(1, 2)
        return q, k, v

    def _finish(self, attn, B, N, D):
        # SSA.py:244-251: LIF(v_th=.5), merge heads, out_proj -> LN -> LIF
        s = self.lifs(attn)[0]
        s = s.transpose(1, 2).contiguous().view(B, N, D)
        return self.lifo(self.lno(self.out_proj(s)))[0]


class SSAMultiHeadAttention_(_SSABase):
    """Plain spiking attention, ``SSA.py:10-100``:
    ``((Q K^T) * mask) @ V * 0.125`` then LIF(v_th=0.5)."""

    def __init__(self, d_model, n_heads, alpha=None, causal=False, learnable_alpha=False,
                 dropout=0.0, n_steps=1, bias=True):
        super().__init__(d_model, n_heads, n_steps, bias)

    def attention(self, q, k, v, mask):
        a = q @ k.transpose(-2, -1)
        if mask is not None:
            a = a * mask
        return (a @ v) * 0.125

    def forward(self, query, key=None, value=None, attention_mask=None):
        key = query if key is None else key
        value = query if value is None else value
        B, N, D = query.shape
        q, k, v = self._project(query, key, value)
        return self._finish(self.attention(q, k, v, attention_mask), B, N, D)


class SSAMultiHeadAttention(_SSABase):
    """XNOR spiking attention with log-distance bias, ``SSA.py:103-258``."""

    def __init__(self, d_model, n_heads, alpha=None, causal=False, learnable_alpha=False,
                 dropout=0.0, n_steps=1, bias=True):
        super().__init__(d_model, n_heads, n_steps, bias)
        self.scale = nn.Parameter(torch.sqrt(torch.tensor(1.0 / (d_model // n_heads))))

    @staticmethod
    def xnor_scores(q, k):
        # SSA.py:145-165: Dh - (sum q + sum k - 2 q.k)
        dh = q.shape[-1]
        qk = torch.einsum("bhld,bhmd->bhlm", q, k)
        ham = q.sum(-1, keepdim=True) + k.sum(-1, keepdim=True).transpose(2, 3) - 2 * qk
        return dh - ham

    def attention(self, q, k, v, mask):
        # SSA.py:234-242
        a = self.xnor_scores(q, k)
        a = a + log_pe_bias(q.shape[2], k.shape[2]).to(a.device).unsqueeze(0).unsqueeze(0)
        if mask is not None:
            a = a * mask
        return (a * self.scale) @ v

    def forward(self, query, key=None, value=None, attention_mask=None):
        key = query if key is None else key
        value = query if value is None else value
        B, N, D = query.shape
        q, k, v = self._project(query, key, value)
        return self._finish(self.attention(q, k, v, attention_mask), B, N, D)


class SpikingMLP(nn.Module):
    """``SpikingMLP.py:4-37``: Linear(D,F) -> LN -> LIF -> Linear(F,D) -> LN -> LIF."""

    def __init__(self, d_model, ff_dim, n_steps=1):
        super().__init__()
        self.n_steps = n_steps
        self.expand = nn.Linear(d_model, ff_dim)
        self.compress = nn.Linear(ff_dim, d_model)
        self.lifexpand = LIF(n_steps=n_steps, learn_beta=True)
        self.lifcompress = LIF(n_steps=n_steps, learn_beta=True)
        self.bn_expand = nn.LayerNorm(ff_dim)
        self.bn_compress = nn.LayerNorm(d_model)

    def forward(self, x):
        h = self.lifexpand(self.bn_expand(self.expand(x)))[0]
        return self.lifcompress(self.bn_compress(self.compress(h)))[0]


class EncoderLayer(nn.Module):
    """``Encoder.py:6-24``: x + SSA(x); then + MLP."""

    def __init__(self, d_model, n_heads, ff_dim, dropout=0.1, alpha=0.125, n_steps=10):
        super().__init__()
        self.self_attns = SSAMultiHeadAttention(d_model=d_model, n_heads=n_heads, n_steps=n_steps)
        self.mlp = SpikingMLP(d_model=d_model, ff_dim=ff_dim, n_steps=n_steps)

    def forward(self, x, mask=None):
        x = x + self.self_attns(x, x, x, attention_mask=mask)
        return x + self.mlp(x)


class Encoder(nn.Module):
    """``Encoder.py:26-41``."""

    def __init__(self, num_layers, d_model, n_heads, ff_dim, dropout=0.1, alpha=0.125, n_steps=10):
        super().__init__()
        self.layers = nn.ModuleList(
            [EncoderLayer(d_model, n_heads, ff_dim, dropout, alpha, n_steps) for _ in range(num_layers)])

    def forward(self, x, mask=None):
        for layer in self.layers:
            x = layer(x, mask=mask)
        return x


class DecoderLayer(nn.Module):
    """``Decoder.py:4-26``: masked self-SSA, unmasked cross-SSA, MLP, residuals."""

    def __init__(self, d_model, n_heads, ff_dim, dropout=0.1, alpha=0.125, n_steps=10):
        super().__init__()
        self.self_attns = SSAMultiHeadAttention(d_model=d_model, n_heads=n_heads, n_steps=n_steps)
        self.cross_attns = SSAMultiHeadAttention(d_model=d_model, n_heads=n_heads, n_steps=n_steps)
        self.mlp = SpikingMLP(d_model=d_model, ff_dim=ff_dim, n_steps=n_steps)

    def forward(self, x, enc_output, mask=None):
        x = x + self.self_attns(x, x, x, attention_mask=mask)
        x = x + self.cross_attns(x, enc_output, enc_output)
        return x + self.mlp(x)


class Decoder(nn.Module):
    """``Decoder.py:28-43``."""

    def __init__(self, num_layers, d_model, n_heads, ff_dim, dropout=0.1, alpha=0.125, n_steps=10):
        super().__init__()
        self.layers = nn.ModuleList(
            [DecoderLayer(d_model, n_heads, ff_dim, dropout, alpha, n_steps) for _ in range(num_layers)])

    def forward(self, x, enc_output, mask=None):
        for layer in self.layers:
            x = layer(x, enc_output, mask=mask)
        return x


class PositionalEncoding(nn.Module):
    """Sinusoidal table, ``Seq2Seq.py:11-26``."""

    def __init__(self, emb_size, dropout, maxlen=5000):
        super().__init__()
        den = torch.exp(-torch.arange(0, emb_size, 2) * math.log(10000) / emb_size)
        pos = torch.arange(0, maxlen).reshape(maxlen, 1)
        table = torch.zeros((maxlen, emb_size))
        table[:, 0::2] = torch.sin(pos * den)
        table[:, 1::2] = torch.cos(pos * den)
        self.dropout = nn.Dropout(dropout)
        self.register_buffer("pos_embedding", table.unsqueeze(0))

    def forward(self, tok):
        return self.dropout(tok + self.pos_embedding[:, : tok.size(1)])


class TokenEmbedding(nn.Module):
    """``Seq2Seq.py:29-36``: embedding * sqrt(emb_size)."""

    def __init__(self, vocab_size, emb_size):
        super().__init__()
        self.embedding = nn.Embedding(vocab_size, emb_size)
        self.emb_size = emb_size

    def forward(self, tokens):
        return self.embedding(tokens.long()) * math.sqrt(self.emb_size)


class FusedInvertedBottleneck(nn.Module):
    """``ImageEncoder.py:8-28``."""

    def __init__(self, n_steps=1, threshold=0.5):
        super().__init__()
        self.conv1 = nn.Conv2d(64, 512, kernel_size=3, stride=1, padding=1)
        self.bn1 = nn.BatchNorm2d(512)
        self.lif_1 = LIF(n_steps=n_steps, beta=0.5)
        self.conv2 = nn.Conv2d(512, 64, kernel_size=1, stride=1, padding=0)
        self.bn2 = nn.BatchNorm2d(64)
        self.lif_2 = LIF(n_steps=n_steps, beta=0.5)

    def forward(self, x):
        h = self.lif_1(self.bn1(self.conv1(x)))[0]
        h = self.lif_2(self.bn2(self.conv2(h)))[0]
        return h + x


class ReduceConvBlock(nn.Module):
    """``ImageEncoder.py:31-44``: fold (c h) into channels, 1x1 conv, BN, LIF."""

    def __init__(self, in_channels=1, out_channels=512, n_steps=1, threshold=0.5):
        super().__init__()
        self.conv = nn.Conv2d(64 * 8, out_channels, kernel_size=1)
        self.bn = nn.BatchNorm2d(out_channels)
        self.lif = LIF(n_steps=n_steps, beta=0.5)

    def forward(self, x):
        b, c, h, w = x.shape
        x = x.reshape(b, c * h, w).unsqueeze(-2)
        y = self.bn(self.conv(x)).squeeze(-2)
        return self.lif(y)[0]


class RPE2D(nn.Module):
    """``ImageEncoder.py:47-61``."""

    def __init__(self, d_model, stride=1, n_steps=1, threshold=0.5):
        super().__init__()
        self.conv = nn.Conv1d(d_model, d_model, kernel_size=3, stride=stride, padding=1)
        self.lif = LIF(n_steps=n_steps, beta=0.5)
        self.bn = nn.BatchNorm1d(d_model)

    def forward(self, x):
        return self.lif(self.bn(self.conv(x)))[0]


class CNNBackbone(nn.Module):
    """``ImageEncoder.py:64-102``; returns ``(tokens [T*B, W', D], record)``."""

    def __init__(self, d_model=512, nb_layers=11, patch_size=4, n_steps=1, threshold=0.5):
        super().__init__()
        self.nb_layers = nb_layers
        self.d_model = d_model
        self.layers = nn.ModuleList([FusedInvertedBottleneck(n_steps=n_steps) for _ in range(nb_layers)])
        self.space_to_depth = nn.PixelUnshuffle(patch_size)
        self.conv1 = nn.Conv2d(16, 128, kernel_size=3, stride=1, padding=1)
        self.bn1 = nn.BatchNorm2d(128)
        self.lif_1 = LIF(n_steps=n_steps, beta=0.5)
        self.conv2 = nn.Conv2d(128, 64, kernel_size=1, stride=1, padding=0)
        self.bn2 = nn.BatchNorm2d(64)
        self.lif_2 = LIF(n_steps=n_steps, beta=0.5)
        self.reduce = ReduceConvBlock(64, d_model, n_steps=n_steps)
        self.rpe = RPE2D(d_model, n_steps=n_steps)

    def forward(self, x):
        record = {}
        x = self.lif_1(self.bn1(self.conv1(self.space_to_depth(x))))[0]
        record["conv1"] = x
        x = self.lif_2(self.bn2(self.conv2(x)))[0]
        record["conv2"] = x
        record["FusedInvertedBottleneck"] = []
        for layer in self.layers:
            x = layer(x)
            record["FusedInvertedBottleneck"].append(x)
        x = self.reduce(x)
        r = self.rpe(x)
        x = (x + r).transpose(-1, -2)
        record["RPE2D"] = r
        record["output"] = x
        return x, record


class PatchEmbed(nn.Module):
    """Patch image encoder (no reference counterpart; the 16x16 patch
    embedding of the OCR benchmark): Conv2d(C, D, p, stride p) -> tokens in
    row-major patch order -> LayerNorm(D) -> LIF.  Returns ``(tokens, record)``
    like ``CNNBackbone.forward`` (``ImageEncoder.py:81-102``)."""

    def __init__(self, d_model=384, patch_size=16, n_steps=1, in_chans=1):
        super().__init__()
        self.patch_size = patch_size
        self.d_model = d_model
        self.proj = nn.Conv2d(in_chans, d_model, kernel_size=patch_size, stride=patch_size)
        self.norm = nn.LayerNorm(d_model)
        self.lif = LIF(n_steps=n_steps)

    def forward(self, x):
        y = self.proj(x).flatten(2).transpose(1, 2)
        s = self.lif(self.norm(y))[0]
        return s, {"output": s}


class Seq2Seq(nn.Module):
    """``Seq2Seq.py:39-162``.  ``image_encoder`` selects ``"cnn"`` (the
    reference ``CNNBackbone``) or ``"patch"`` (``PatchEmbed``)."""

    def __init__(self, patch_size=16, d_model=512, n_heads=8, ff_dim=2048,
                 num_encoder_layers=6, num_decoder_layers=6, dropout=0.1, alpha=0.125,
                 tgt_vocab_size=1000, nb_sps_blocks=4, n_steps=10,
                 image_encoder="cnn", in_chans=1):
        super().__init__()
        self.n_steps = n_steps
        if image_encoder == "cnn":
            self.image_encoder = CNNBackbone(nb_layers=nb_sps_blocks, patch_size=patch_size,
                                             d_model=d_model, n_steps=n_steps)
        else:
            self.image_encoder = PatchEmbed(d_model=d_model, patch_size=patch_size,
                                            n_steps=n_steps, in_chans=in_chans)
        self.encoder = Encoder(num_encoder_layers, d_model, n_heads, ff_dim, dropout, alpha, n_steps)
        self.decoder = Decoder(num_decoder_layers, d_model, n_heads, ff_dim, dropout, alpha, n_steps)
        self.output_layer = nn.Linear(d_model, tgt_vocab_size)
        self.lifPE = LIF(n_steps=n_steps)
        self.tgt_tok_emb = TokenEmbedding(tgt_vocab_size, d_model)
        self.positional_encoding = PositionalEncoding(d_model, dropout=dropout)

    def forward(self, src, tgt, look_ahead_mask=None, enc_padding_mask=None, dec_padding_mask=None):
        enc, _ = self.encode(src)
        return self.decode(tgt, enc, look_ahead_mask)

    def encode(self, src):
        # Seq2Seq.py:98-104: repeat the image T times (t-major fold)
        B = src.shape[0]
        T = self.n_steps
        src = src.unsqueeze(0).expand(T, *src.shape).reshape(T * B, *src.shape[1:])
        enc, _ = self.image_encoder(src)
        return self.encoder(enc), None

    def decode(self, tgt, enc_output, look_ahead_mask=None, enc_padding_mask=None, dec_padding_mask=None):
        # Seq2Seq.py:106-119
        T = self.n_steps
        if look_ahead_mask is not None:
            m = look_ahead_mask
            look_ahead_mask = m.unsqueeze(0).repeat(T, 1, 1, 1, 1).reshape(T * m.shape[0], *m.shape[1:])
        y = self.positional_encoding(self.tgt_tok_emb(tgt))
        B, N, D = y.shape
        y = y.unsqueeze(0).expand(T, B, N, D).reshape(T * B, N, D)
        y = self.lifPE(y)[0]
        y = self.decoder(y, enc_output, mask=look_ahead_mask)
        out = self.output_layer(y)
        return out.view(T, out.shape[0] // T, out.shape[1], out.shape[2]), None

    # Seq2Seq.py:121-134: keep = 1, pad = 0; the look-ahead mask combined with the key padding
    def create_decoder_mask(self, tgt, pad_idx, device):
        look_ahead = torch.tril(torch.ones((tgt.shape[1], tgt.shape[1]), device=device))
        pad = torch.where(tgt == pad_idx, 0.0, 1.0).unsqueeze(1).unsqueeze(1).to(device)
        return torch.minimum(pad, look_ahead)

    @torch.no_grad()
    def greedy_decode(self, src, max_len, start_symbol, eos_idx, pad_idx, device="cpu"):
        """Seq2Seq.py:136-162: decode the whole prefix every step, append the
        argmax of the T-averaged logits of the last position, stop at eos."""
        if src.dim() == 3:
            src = src.unsqueeze(0)
        memory, _ = self.encode(src.to(device))
        ys = torch.full((1, 1), fill_value=start_symbol, dtype=torch.long, device=device)
        out = None
        for _ in range(max_len - 1):
            out, _ = self.decode(ys, memory, self.create_decoder_mask(ys, pad_idx, device))
            nxt = int(torch.argmax(out.mean(dim=0)[:, -1, :], dim=-1))
            ys = torch.cat([ys, torch.tensor([[nxt]], dtype=torch.long, device=device)], dim=1)
            if nxt == eos_idx:
                break
        return ys, None, out
