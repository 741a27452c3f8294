"""Image encoders: drop-in for ``Triton_Layers/ImageEncoder.py`` plus the
16x16 patch embedding of the OCR benchmark.

``CNNBackbone`` and its blocks (``ImageEncoder.py:8-102``) keep the reference
structure and names.  In inference (eval mode, no autograd graph) every
convolution runs as a fused tcgen05 GEMM over gathered patches with the
eval-mode BatchNorm as a per-channel affine and the LIF in its epilogue
(``spk_im2col`` + ``spk_linear_affine_lif_fwd``), channels-last, with the
bottleneck identity and the ``x + rpe`` sum added in place; no library
convolution runs.  Training (BatchNorm on batch statistics) keeps the
reference composition: library conv and BatchNorm, this package's LIF.
``PatchEmbed`` (no reference counterpart) is Conv2d(C, D, p, stride p) ->
tokens in row-major patch order -> LayerNorm(D) -> LIF, computed as one fused
tensor-core GEMM over gathered patches: pixels are split into two bf16 terms
against [W | W], which keeps the projection at fp32 accuracy (~2^-17
relative).
"""

import torch
from torch import nn

from . import ops
from ._fused import _key, bf16_weight, fast_path_ok, lif_params, ln_lif, mark_spike_counts
from .Lif import LIF


def _cached(owner, attr, key, make):
    """Derived tensor cached on ``owner`` until ``key`` (storage pointers and
    version counters of its sources) changes."""
    c = getattr(owner, attr, None)
    if c is not None and c[0] == key:
        return c[1]
    with torch.no_grad():
        v = make()
    object.__setattr__(owner, attr, (key, v))
    return v


def conv_bn_operands(conv, bn, weight_order, duplicate=False):
    """GEMM operands of ``bn(conv(x))`` in eval mode: the bf16 weight
    ``[C_out, K]`` with its columns in the patch order ``weight_order(w)``
    returns (``[W | W]`` with ``duplicate``, for split fp32 patches), the conv
    bias, and the BatchNorm as ``y = (conv + bias) * scale + shift`` with
    ``scale = weight / sqrt(running_var + eps)`` and ``shift = bias_bn -
    running_mean * scale`` (the per-channel affine of the reference's eval
    BatchNorm)."""
    key = _key(conv.weight, bn.weight, bn.bias, bn.running_mean, bn.running_var) + (duplicate,)

    def make():
        w = weight_order(conv.weight.detach()).reshape(conv.out_channels, -1).to(torch.bfloat16)
        if duplicate:
            w = torch.cat([w, w], dim=1)
        invstd = 1.0 / torch.sqrt(bn.running_var.detach().float() + bn.eps)
        scale = invstd * bn.weight.detach().float()
        shift = bn.bias.detach().float() - bn.running_mean.detach().float() * scale
        return w.contiguous(), scale.contiguous(), shift.contiguous()

    w, scale, shift = _cached(conv, "_spk_conv_bn", key, make)
    return w, conv.bias, scale, shift


def _conv_affine_lif(A, conv, bn, lif, weight_order, T, duplicate=False, t_broadcast=False, residual=None):
    w, bias, scale, shift = conv_bn_operands(conv, bn, weight_order, duplicate)
    p = lif_params(lif)
    return ops.linear_affine_lif(A, w, bias, scale, shift, p[0:1], p[1:2], p[2:3], T, in_gain=lif.in_gain,
                                 t_broadcast=t_broadcast, residual=residual, want_spikes=residual is None)


def _taps_last(w):
    """Conv weight ``[C_out, C_in, kh, kw]`` -> ``[C_out, kh, kw, C_in]`` (the
    column order of ``spk_im2col`` patches)."""
    return w.permute(0, 2, 3, 1)


class FusedInvertedBottleneck(nn.Module):
    """``ImageEncoder.py:8-28``: conv3x3 64->512, BN, LIF, conv1x1 512->64, BN, LIF, + identity."""

    def __init__(self, n_steps=1, threshold=0.5):
        super().__init__()
        self.conv1 = nn.Conv2d(64, 512, kernel_size=3, stride=1, padding=1)
        self.bn1 = nn.BatchNorm2d(512)
        self.lif_1 = LIF(n_steps=n_steps, beta=0.5)
        self.conv2 = nn.Conv2d(512, 64, kernel_size=1, stride=1, padding=0)
        self.bn2 = nn.BatchNorm2d(64)
        self.lif_2 = LIF(n_steps=n_steps, beta=0.5)

    def _fast(self, x, T):
        """bf16 channels-last ``x [T*B, H, W, 64]`` -> ``lif_2(bn2(conv2(h))) + x``."""
        TB, H, W, C = x.shape
        a = ops.im2col(x, (3, 3), (1, 1), (1, 1))
        h = _conv_affine_lif(a, self.conv1, self.bn1, self.lif_1, _taps_last, T)
        out = x.clone(memory_format=torch.contiguous_format)
        _conv_affine_lif(h, self.conv2, self.bn2, self.lif_2, _taps_last, T, residual=out.view(-1, C))
        return out

    def forward(self, x):
        out = self.lif_1(self.bn1(self.conv1(x)))[0]
        out = self.lif_2(self.bn2(self.conv2(out)))[0]
        return out + x


class ReduceConvBlock(nn.Module):
    """``ImageEncoder.py:31-44``: fold (channel, height) into channels, 1x1 conv, BN, LIF."""

    def __init__(self, in_channels=1, out_channels=512, n_steps=1, threshold=0.5):
        super().__init__()
        self.conv = nn.Conv2d(64 * 8, out_channels, kernel_size=1)
        self.bn = nn.BatchNorm2d(out_channels)
        self.lif = LIF(n_steps=n_steps, beta=0.5)

    def _fast(self, x, T):
        """bf16 channels-last ``x [T*B, H, W, C]`` -> spikes ``[T*B, W, D]``: the
        1x1 convolution over the (channel, height) fold is a gather of each
        column's ``H x C`` block, the weight's input channels ``c*H + h``
        reordered to ``h*C + c``."""
        TB, H, W, C = x.shape
        a = ops.im2col(x, (H, 1), (1, 1), (0, 0))

        def order(w):
            return w.reshape(w.shape[0], C, H).transpose(1, 2)

        s = _conv_affine_lif(a, self.conv, self.bn, self.lif, order, T)
        return s.view(TB, W, -1)

    def forward(self, x):
        b, c, h, w = x.shape
        x = x.reshape(b, c * h, w).unsqueeze(-2)
        out = self.bn(self.conv(x)).squeeze(-2)
        return self.lif(out)[0]


class RPE2D(nn.Module):
    """``ImageEncoder.py:47-61``: conv1d k3 + BN + LIF."""

    def __init__(self, d_model, stride=1, n_steps=1, threshold=0.5):
        super().__init__()
        self.conv = nn.Conv1d(d_model, d_model, kernel_size=3, stride=stride, padding=1)
        self.lif = LIF(n_steps=n_steps, beta=0.5)
        self.bn = nn.BatchNorm1d(d_model)

    def get_mem(self):
        return {"mem": getattr(self.lif, "mem", None)}

    def _fast_sum(self, x, T):
        """bf16 ``x [T*B, W, D]`` (tokens, channels-last) -> ``x + lif(bn(conv(x)))``."""
        TB, W, D = x.shape
        a = ops.im2col(x.view(TB, 1, W, D), (1, 3), (1, 1), (0, 1))
        out = x.clone(memory_format=torch.contiguous_format)
        _conv_affine_lif(a, self.conv, self.bn, self.lif, lambda w: w.permute(0, 2, 1), T, residual=out.view(-1, D))
        return out

    def forward(self, x):
        return self.lif(self.bn(self.conv(x)))[0]


class CNNBackbone(nn.Module):
    """``ImageEncoder.py:64-102``; ``forward(x[T*B,1,32,W]) -> (tokens [T*B, W/4, D], record)``."""

    def __init__(self, d_model=512, nb_layers=11, patch_size=4, n_steps=1, threshold=0.5):
        super().__init__()
        self.nb_layers = nb_layers
        self.d_model = d_model
        self.layers = nn.ModuleList([FusedInvertedBottleneck(n_steps=n_steps, threshold=threshold)
                                     for _ in range(nb_layers)])
        self.space_to_depth = nn.PixelUnshuffle(patch_size)
        self.conv1 = nn.Conv2d(16, 128, kernel_size=3, stride=1, padding=1)
        self.bn1 = nn.BatchNorm2d(128)
        self.lif_1 = LIF(n_steps=n_steps, beta=0.5)
        self.conv2 = nn.Conv2d(128, 64, kernel_size=1, stride=1, padding=0)
        self.bn2 = nn.BatchNorm2d(64)
        self.lif_2 = LIF(n_steps=n_steps, beta=0.5)
        self.reduce = ReduceConvBlock(64, d_model, n_steps=n_steps, threshold=threshold)
        self.rpe = RPE2D(d_model, n_steps=n_steps, threshold=threshold)

    def _fast_ok(self, x):
        p = self.space_to_depth.downscale_factor
        return (not self.training and fast_path_ok(x, module=self) and x.dim() == 4 and x.shape[-2] % p == 0
                and x.shape[-1] % p == 0)

    def _fast(self, images, T, t_broadcast):
        """Fused forward: ``images [n, C, Hi, Wi]`` fp32 -> (bf16 tokens ``[T*B, Wi/p,
        D]``, record).  With ``t_broadcast`` the n images are the B images of a
        T-fold that repeats them (``Seq2Seq.py:98-104``), so the first
        convolution runs once per image and feeds the LIF at every step."""
        p = self.space_to_depth.downscale_factor
        n, Ci, Hi, Wi = images.shape
        H, W = Hi // p, Wi // p
        TB = T * n if t_broadcast else n
        # PixelUnshuffle(p) then conv1 (3x3, padding 1) = one 3p x 3p, stride-p,
        # padding-p gather of the image; unshuffled channel ci*p*p + dy*p + dx
        # at tap (i, j) is image offset (i*p + dy, j*p + dx) of channel ci
        a = ops.im2col(images.permute(0, 2, 3, 1), (3 * p, 3 * p), (p, p), (p, p))

        def order1(w):
            o = w.shape[0]
            return w.reshape(o, Ci, p, p, 3, 3).permute(0, 4, 2, 5, 3, 1)

        x = _conv_affine_lif(a, self.conv1, self.bn1, self.lif_1, order1, T, duplicate=True,
                             t_broadcast=t_broadcast)
        record = {"conv1": x.view(TB, H, W, -1).permute(0, 3, 1, 2)}
        x = _conv_affine_lif(x, self.conv2, self.bn2, self.lif_2, _taps_last, T).view(TB, H, W, -1)
        record["conv2"] = x.permute(0, 3, 1, 2)
        record["FusedInvertedBottleneck"] = []
        for layer in self.layers:
            x = layer._fast(x, T)
            record["FusedInvertedBottleneck"].append(x.permute(0, 3, 1, 2))
        x = self.reduce._fast(x, T)
        out = self.rpe._fast_sum(x, T)
        record["output"] = out
        return out, record

    def encode_images(self, src, T):
        """bf16 tokens ``[T*B, W', D]`` of the T-fold that repeats ``src [B, C, H, W]``
        over T (inference, eval mode)."""
        return self._fast(src.float(), T, t_broadcast=True)[0]

    def forward(self, x):
        if self._fast_ok(x):
            out, record = self._fast(x.float(), self.lif_1.n_steps, t_broadcast=False)
            y = mark_spike_counts(out.float(), out)
            record["output"] = y
            return y, record
        record = {}
        x = self.space_to_depth(x)
        x = self.lif_1(self.bn1(self.conv1(x)))[0]
        record["conv1"] = x
        x = self.lif_2(self.bn2(self.conv2(x)))[0]
        record["conv2"] = x
        record["FusedInvertedBottleneck"] = []
        for layer in self.layers:
            x = layer(x)
            record["FusedInvertedBottleneck"].append(x)
        x = self.reduce(x)
        rpe_value = self.rpe(x)
        x = (x + rpe_value).transpose(-1, -2)
        if not x.requires_grad:
            mark_spike_counts(x)  # sums of two spike trains
        record["RPE2D"] = rpe_value
        record["output"] = x
        return x, record


class PatchEmbed(nn.Module):
    """Patch image encoder: ``forward(x[T*B, C, H, W]) -> (spikes [T*B, (H/p)(W/p), D], record)``."""

    def __init__(self, d_model=384, patch_size=16, n_steps=1, in_chans=1):
        super().__init__()
        self.patch_size = patch_size
        self.d_model = d_model
        self.proj = nn.Conv2d(in_chans, d_model, kernel_size=patch_size, stride=patch_size)
        self.norm = nn.LayerNorm(d_model)
        self.lif = LIF(n_steps=n_steps)

    def _fused(self, images, t_broadcast):
        """images [rows, C, H, W] fp32 -> bf16 spikes [T*B, n_patches, D]."""
        T = self.lif.n_steps
        a = ops.patch_im2col(images, self.patch_size)
        p = lif_params(self.lif)
        s, _ = ops.linear_ln_lif(a, bf16_weight(self.proj, duplicate=True), self.proj.bias, self.norm.weight,
                                 self.norm.bias, self.norm.eps, p[0:1], p[1:2], p[2:3], T,
                                 in_gain=self.lif.in_gain, t_broadcast=t_broadcast)
        n_patch = a.shape[0] // images.shape[0]
        TB = T * images.shape[0] if t_broadcast else images.shape[0]
        return s.view(TB, n_patch, self.d_model)

    def encode_images(self, src):
        """The T-fold of ``src [B, C, H, W]`` repeated over T, computed once per image."""
        return self._fused(src, t_broadcast=True)

    def _project(self, x):
        """The 16x16 / stride-16 convolution without its bias as one GEMM:
        ``[N, C, H, W]`` -> ``[N, (H/p)(W/p), D]`` in the order of
        ``proj(x).flatten(2).transpose(1, 2)`` (H and W multiples of p)."""
        p = self.patch_size
        N, C, H, W = x.shape
        a = x.reshape(N, C, H // p, p, W // p, p).permute(0, 2, 4, 1, 3, 5).reshape(N * (H // p) * (W // p), -1)
        y = torch.nn.functional.linear(a, self.proj.weight.reshape(self.d_model, -1))
        return y.view(N, (H // p) * (W // p), self.d_model)

    def _tiles(self, x):
        p = self.patch_size
        return x.is_cuda and x.shape[-2] % p == 0 and x.shape[-1] % p == 0

    def forward(self, x):
        if fast_path_ok(x, module=self):
            sb = self._fused(x, t_broadcast=False)
            s = mark_spike_counts(sb.float(), sb)
            return s, {"output": s}
        if self._tiles(x):
            # conv bias handed to the LayerNorm->LIF kernels
            s = ln_lif(self._project(x), self.norm, self.lif, bias=self.proj.bias)
        else:
            s = ln_lif(self.proj(x).flatten(2).transpose(1, 2), self.norm, self.lif)
        return s, {"output": s}

    def forward_repeated(self, src, T):
        """``forward`` of ``src [B, C, H, W]`` repeated T times along dim 0 (the
        encoder input of ``Seq2Seq.py:98-104``), with the projection computed once
        per image; its gradient sums over the T copies as the repeat's does."""
        if not self._tiles(src):
            B = src.shape[0]
            return self(src.unsqueeze(0).expand(T, *src.shape).reshape(T * B, *src.shape[1:]))
        y = self._project(src)
        y = y.unsqueeze(0).expand(T, *y.shape).reshape(T * y.shape[0], *y.shape[1:])
        s = ln_lif(y, self.norm, self.lif, bias=self.proj.bias)
        return s, {"output": s}
