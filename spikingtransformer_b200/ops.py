"""Tensor-level wrappers over the C ABI (no autograd; see Lif.py for that).

Every function requires CUDA tensors and raises on CPU input: there is no
CPU implementation in this package.
"""

import torch

from . import _lib


def _cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("spikingtransformer_b200 ops need CUDA tensors (got %s)" % t.device)


def _scalar_f32(v, device):
    """A one-element fp32 device tensor holding ``v`` (tensor or number)."""
    if isinstance(v, torch.Tensor):
        if v.device != device:
            v = v.to(device)
        if v.dtype != torch.float32:
            v = v.float()
        return v.reshape(1).contiguous()
    return torch.full((1,), float(v), dtype=torch.float32, device=device)


def lif_fwd(x, beta, v_th, v_reset, in_gain=1.0, spike_dtype=torch.float32, want_v_final=True):
    """LIF scan over dim 0 of ``x`` ([T, ...]); returns ``(spikes, v_final)``.

    ``x`` may be fp32/fp16/bf16; spikes are ``spike_dtype`` (fp32, bf16,
    uint8 or float8_e4m3fn, shaped like ``x``) or ``"bits"``: packed bits,
    uint8 ``[T, ceil(N/8)]`` with neuron n of step t at bit n % 8 of byte
    ``[t, n // 8]`` (N = ``x[0].numel()``); ``v_final`` is fp32 shaped like
    ``x[0]`` (or None).
    """
    _cuda(x)
    x = x.contiguous()
    T = x.shape[0]
    N = x[0].numel()
    dev = x.device
    if spike_dtype == "bits":
        s = torch.empty((T, (N + 7) // 8), dtype=torch.uint8, device=dev)
        code, out_bytes = _lib.BIT, s.numel()
    else:
        s = torch.empty(x.shape, dtype=spike_dtype, device=dev)
        code, out_bytes = _lib.dtype_code(s), s.numel() * s.element_size()
    vf = torch.empty(x.shape[1:], dtype=torch.float32, device=dev) if want_v_final else None
    b, th, vr = (_scalar_f32(v, dev) for v in (beta, v_th, v_reset))
    nbytes = T * N * x.element_size() + out_bytes + (4 * N if vf is not None else 0)
    _lib.call("spk_lif_fwd", _lib.ptr(x), _lib.dtype_code(x), _lib.ptr(s), code, _lib.ptr(vf),
              _lib.ptr(b), _lib.ptr(th), _lib.ptr(vr), float(in_gain), T, N, _lib.stream_ptr(dev),
              tag="lif_fwd", work=dict(bytes=nbytes))
    return s, vf


def unpack_spike_bits(bits, N):
    """Packed spike bits ``[T, ceil(N/8)]`` (``lif_fwd(..., spike_dtype="bits")``)
    -> float 0/1 ``[T, N]`` (a plain tensor op, for checks and inspection)."""
    shifts = torch.arange(8, device=bits.device, dtype=torch.uint8)
    b = (bits.unsqueeze(-1) >> shifts) & 1
    return b.reshape(bits.shape[0], -1)[:, :N].float()


def lif_bwd(g_spikes, g_vfinal, x, spikes, beta, v_th, v_reset, in_gain=1.0, surrogate="superspike", k=4.0,
            need_beta_grad=True, spikes_packed=False):
    """Backward of ``lif_fwd``; returns ``(grad_x in x.dtype, grad_beta fp32 [1] or None)``.
    ``spikes_packed``: ``spikes`` holds packed bits (``spike_dtype="bits"``)."""
    _cuda(g_spikes, g_vfinal, x, spikes)
    x = x.contiguous()
    spikes = spikes.contiguous()
    g_spikes = g_spikes.contiguous().to(torch.float32)
    if g_vfinal is not None:
        g_vfinal = g_vfinal.contiguous().to(torch.float32)
    T = x.shape[0]
    N = x[0].numel()
    dev = x.device
    gx = torch.empty_like(x)
    b, th, vr = (_scalar_f32(v, dev) for v in (beta, v_th, v_reset))
    gb = ws = None
    wsb = 0
    if need_beta_grad:
        gb = torch.empty(1, dtype=torch.float32, device=dev)
        wsb = int(_lib.load().spk_lif_bwd_workspace_bytes(T, N))
        ws = torch.empty(wsb // 4, dtype=torch.float32, device=dev)
    s_code = _lib.BIT if spikes_packed else _lib.dtype_code(spikes)
    _lib.call("spk_lif_bwd", _lib.ptr(g_spikes), _lib.ptr(g_vfinal), _lib.ptr(x), _lib.dtype_code(x),
              _lib.ptr(spikes), s_code, _lib.ptr(b), _lib.ptr(th), _lib.ptr(vr), float(in_gain),
              _lib.SURROGATE[surrogate], float(k), _lib.ptr(gx), _lib.ptr(gb), _lib.ptr(ws), wsb, T, N,
              _lib.stream_ptr(dev), tag="lif_bwd",
              work=dict(bytes=T * N * (4 + 2 * x.element_size()) + spikes.numel() * spikes.element_size(),
                        launches=2))
    return gx, gb


def linear_ln_lif(A, W, bias, ln_gamma, ln_beta, ln_eps, lif_beta, lif_vth, lif_vr, T, in_gain=1.0,
                  t_broadcast=False, spike_dtype=torch.bfloat16, residual=None, want_spikes=True,
                  want_ln_out=False):
    """Fused ``LIF(LayerNorm(A @ W.T + bias))`` over the t-major fold.

    ``A``: bf16 ``[T*R, K]`` (or ``[R, K]`` with ``t_broadcast``); ``W``: bf16
    ``[N, K]``.  Returns ``(spikes [T*R, N] or None, ln_out fp32 or None)``.
    With ``residual`` (bf16 ``[T*R, N]``) the spikes are also added into it.
    """
    _cuda(A, W, residual)
    if A.dtype != torch.bfloat16 or W.dtype != torch.bfloat16:
        raise TypeError("linear_ln_lif expects bf16 A and W")
    A = A.contiguous()
    W = W.contiguous()
    K = A.shape[-1]
    N = W.shape[0]
    rows = A.numel() // K
    R = rows if t_broadcast else rows // T
    if not t_broadcast and rows % T:
        raise RuntimeError("rows %d not divisible by T=%d" % (rows, T))
    dev = A.device
    out_rows = T * R
    spikes = torch.empty((out_rows, N), dtype=spike_dtype, device=dev) if want_spikes else None
    ln_out = torch.empty(((R if t_broadcast else out_rows), N), dtype=torch.float32, device=dev) \
        if want_ln_out else None
    if residual is not None and (residual.dtype != torch.bfloat16 or not residual.is_contiguous()):
        raise TypeError("residual must be a contiguous bf16 tensor")
    f = lambda t: None if t is None else t.float().contiguous()  # noqa: E731
    bias, ln_gamma, ln_beta = f(bias), f(ln_gamma), f(ln_beta)
    b, th, vr = (_scalar_f32(v, dev) for v in (lif_beta, lif_vth, lif_vr))
    _lib.call("spk_linear_ln_lif_fwd", _lib.ptr(A), _lib.ptr(W), _lib.ptr(bias), _lib.ptr(ln_gamma),
              _lib.ptr(ln_beta), float(ln_eps), _lib.ptr(b), _lib.ptr(th), _lib.ptr(vr), float(in_gain), T, R, K, N,
              1 if t_broadcast else 0, _lib.ptr(spikes), _lib.DTYPE_CODE[spike_dtype], _lib.ptr(residual),
              _lib.ptr(ln_out), _lib.stream_ptr(dev),
              tag="linear_ln_lif K=%d N=%d rows=%d%s" % (K, N, rows, " +residual" if residual is not None else ""),
              work=dict(flops=2.0 * rows * K * N,
                        bytes=(rows * K + N * K) * 2 + out_rows * N * (spikes.element_size() if want_spikes else 0)
                        + (4 * out_rows * N if residual is not None else 0)))
    return spikes, ln_out


def linear_affine_lif(A, W, bias, scale, shift, lif_beta, lif_vth, lif_vr, T, in_gain=1.0, t_broadcast=False,
                      spike_dtype=torch.bfloat16, residual=None, want_spikes=True):
    """Fused ``LIF((A @ W.T + bias) * scale + shift)`` over the t-major fold
    (per-feature affine, e.g. an eval-mode BatchNorm; no row statistics).

    ``A``: bf16 ``[T*R, K]`` (or ``[R, K]`` with ``t_broadcast``); ``W``: bf16
    ``[N, K]``.  Returns the spikes ``[T*R, N]`` (or None when only the
    ``residual`` (bf16 ``[T*R, N]``) is updated, in place)."""
    _cuda(A, W, residual)
    if A.dtype != torch.bfloat16 or W.dtype != torch.bfloat16:
        raise TypeError("linear_affine_lif expects bf16 A and W")
    A = A.contiguous()
    W = W.contiguous()
    K = A.shape[-1]
    N = W.shape[0]
    rows = A.numel() // K
    R = rows if t_broadcast else rows // T
    if not t_broadcast and rows % T:
        raise RuntimeError("rows %d not divisible by T=%d" % (rows, T))
    dev = A.device
    spikes = torch.empty((T * R, N), dtype=spike_dtype, device=dev) if want_spikes else None
    if residual is not None and (residual.dtype != torch.bfloat16 or not residual.is_contiguous()):
        raise TypeError("residual must be a contiguous bf16 tensor")
    f = lambda t: None if t is None else t.float().contiguous()  # noqa: E731
    bias, scale, shift = f(bias), f(scale), f(shift)
    b, th, vr = (_scalar_f32(v, dev) for v in (lif_beta, lif_vth, lif_vr))
    _lib.call("spk_linear_affine_lif_fwd", _lib.ptr(A), _lib.ptr(W), _lib.ptr(bias), _lib.ptr(scale), _lib.ptr(shift),
              _lib.ptr(b), _lib.ptr(th), _lib.ptr(vr), float(in_gain), T, R, K, N, 1 if t_broadcast else 0,
              _lib.ptr(spikes), _lib.DTYPE_CODE[spike_dtype], _lib.ptr(residual), _lib.stream_ptr(dev),
              tag="linear_affine_lif K=%d N=%d rows=%d%s" % (K, N, rows, " +residual" if residual is not None else ""),
              work=dict(flops=2.0 * rows * K * N,
                        bytes=(rows * K + N * K) * 2 + T * R * N * (spikes.element_size() if want_spikes else 0)
                        + (4 * T * R * N if residual is not None else 0)))
    return spikes


def im2col(x, kernel, stride=(1, 1), padding=(0, 0)):
    """Patches of a channels-last ``x`` ``[N, H, W, C]`` (bf16, or fp32 split
    into hi | lo bf16 terms) for a ``kernel = (kh, kw)`` convolution: bf16
    ``[N*Ho*Wo, kh*kw*C]`` (``2*kh*kw*C`` for fp32), column ``(i*kw + j)*C + c``."""
    _cuda(x)
    if x.dtype not in (torch.float32, torch.bfloat16):
        x = x.float()
    x = x.contiguous()
    N, H, W, C = x.shape
    kh, kw = kernel
    sh, sw = stride
    ph, pw = padding
    Ho = (H + 2 * ph - kh) // sh + 1
    Wo = (W + 2 * pw - kw) // sw + 1
    K = kh * kw * C * (2 if x.dtype == torch.float32 else 1)
    out = torch.empty((N * Ho * Wo, K), dtype=torch.bfloat16, device=x.device)
    _lib.call("spk_im2col", _lib.ptr(x), _lib.dtype_code(x), N, H, W, C, kh, kw, sh, sw, ph, pw, _lib.ptr(out),
              _lib.stream_ptr(x.device), tag="im2col",
              work=dict(bytes=x.numel() * x.element_size() + out.numel() * 2))
    return out


def ln_lif_ok(T, D):
    """Shapes the fused LayerNorm -> LIF training kernels take."""
    return 1 <= T <= 4 and D % 32 == 0 and 32 <= D <= 2048 and (D <= 512 or D % 128 == 0)


def _row_stride(t):
    """Row stride (elements) of ``t`` viewed as ``[rows, t.shape[-1]]`` with unit
    column stride (a column slice of a wider tensor qualifies), else None."""
    if t.dim() < 2 or t.stride(-1) != 1:
        return None
    ld = t.stride(-2)
    expected = ld
    for i in range(t.dim() - 2, 0, -1):
        expected *= t.shape[i]
        if t.stride(i - 1) != expected:
            return None
    return ld


def ln_lif_fwd(pre, ln_gamma, ln_beta, ln_eps, lif_beta, lif_vth, lif_vr, T, in_gain=1.0,
               spike_dtype=torch.float32, bias=None, heads=None):
    """``LIF(LayerNorm(pre + bias))`` over the t-major fold; ``pre`` ``[T*R, ..., D]``,
    ``bias`` ``[D]`` or None (the preceding Linear's bias, taken out of its GEMM).
    ``heads=(head_dim, seq_len)``: spikes written head-major, ``[T*R/seq_len,
    D/head_dim, seq_len, head_dim]`` (the per-head layout the attention reads).
    ``pre`` may be a column slice of a wider tensor (row stride > D, read in
    place).  Returns ``(spikes like pre in spike_dtype, stats fp32 [T*R', 2]
    (mean, rstd))``."""
    _cuda(pre)
    D = pre.shape[-1]
    ld = _row_stride(pre)
    if ld is None or ld < D or (ld != D and (D % 128 or ld % 4)):
        pre, ld = pre.contiguous(), D
    rows = pre.numel() // D
    if rows % T:
        raise RuntimeError("rows %d not divisible by T=%d" % (rows, T))
    R = rows // T
    dev = pre.device
    hd, sl = heads if heads is not None else (0, 1)
    shape = pre.shape if heads is None else (rows // sl, D // hd, sl, hd)
    spikes = torch.empty(shape, dtype=spike_dtype, device=dev)
    stats = torch.empty((rows, 2), dtype=torch.float32, device=dev)
    g = None if ln_gamma is None else ln_gamma.detach().float().contiguous()
    bt = None if ln_beta is None else ln_beta.detach().float().contiguous()
    pb = None if bias is None else bias.detach().float().contiguous()
    b, th, vr = (_scalar_f32(v, dev) for v in (lif_beta, lif_vth, lif_vr))
    _lib.call("spk_ln_lif_fwd", _lib.ptr(pre), _lib.dtype_code(pre), _lib.ptr(pb), _lib.ptr(g), _lib.ptr(bt),
              float(ln_eps),
              _lib.ptr(b), _lib.ptr(th), _lib.ptr(vr), float(in_gain), T, R, D, ld, hd, sl, _lib.ptr(spikes),
              _lib.DTYPE_CODE[spike_dtype], _lib.ptr(stats), _lib.stream_ptr(dev), tag="ln_lif_fwd D=%d" % D,
              work=dict(bytes=rows * D * (pre.element_size() + spikes.element_size()) + rows * 8))
    return spikes, stats


def ln_lif_residual_ok(pre, residual):
    """Whether ``ln_lif_fwd_residual`` takes these tensors: D = 384, 768 or
    1536, fp32 residual ``[rows, D]`` laid out like the output, 16-byte aligned
    rows."""
    D = pre.shape[-1]
    ld = _row_stride(pre)
    return (D in (384, 768, 1536) and pre.is_cuda and residual.is_cuda and residual.dtype == torch.float32
            and residual.is_contiguous() and residual.numel() == pre.numel() and ld is not None and ld % 4 == 0
            and pre.data_ptr() % 16 == 0 and residual.data_ptr() % 16 == 0)


def ln_lif_fwd_residual(pre, ln_gamma, ln_beta, ln_eps, lif_beta, lif_vth, lif_vr, T, residual, in_gain=1.0,
                        bias=None, want_bf16=False):
    """``residual + LIF(LayerNorm(pre + bias))`` in one kernel: the residual
    connection of a transformer layer (``Encoder.py:19-22``,
    ``Decoder.py:18-24``) fused into the LayerNorm->LIF forward.  Returns
    ``(out fp32 like residual, stats [T*R, 2], out in bf16 or None)``; the
    backward is ``ln_lif_bwd`` with ``g_spikes = dL/dout``.  Callers check
    ``ln_lif_residual_ok`` first."""
    _cuda(pre, residual)
    D = pre.shape[-1]
    ld = _row_stride(pre)
    rows = pre.numel() // D
    if rows % T:
        raise RuntimeError("rows %d not divisible by T=%d" % (rows, T))
    dev = pre.device
    out = torch.empty(residual.shape, dtype=torch.float32, device=dev)
    outb = torch.empty(residual.shape, dtype=torch.bfloat16, device=dev) if want_bf16 else None
    stats = torch.empty((rows, 2), dtype=torch.float32, device=dev)
    g = None if ln_gamma is None else ln_gamma.detach().float().contiguous()
    bt = None if ln_beta is None else ln_beta.detach().float().contiguous()
    pb = None if bias is None else bias.detach().float().contiguous()
    b, th, vr = (_scalar_f32(v, dev) for v in (lif_beta, lif_vth, lif_vr))
    _lib.call("spk_ln_lif_fwd_residual", _lib.ptr(pre), _lib.dtype_code(pre), _lib.ptr(pb), _lib.ptr(g),
              _lib.ptr(bt), float(ln_eps), _lib.ptr(b), _lib.ptr(th), _lib.ptr(vr), float(in_gain), T, rows // T,
              D, ld, _lib.ptr(residual), _lib.ptr(out), _lib.ptr(outb), _lib.ptr(stats), _lib.stream_ptr(dev),
              tag="ln_lif_fwd_residual D=%d" % D,
              work=dict(bytes=rows * D * (pre.element_size() + 8 + (2 if want_bf16 else 0)) + rows * 8))
    return out, stats, outb


def ln_lif_bwd(g_spikes, pre, stats, ln_gamma, ln_beta, lif_beta, lif_vth, lif_vr, T, in_gain=1.0,
               surrogate="superspike", k=4.0, need_gamma=True, need_beta=True, need_lif_beta=True, bias=None,
               need_bias=False, heads=None, g_pre_out=None):
    """Backward of ``ln_lif_fwd``: ``(g_pre like pre, g_gamma [D] or None, g_beta [D] or None,
    g_lif_beta [1] or None, g_bias [D] or None)``; ``bias`` and ``heads`` are the
    forward's (with ``heads``, ``g_spikes`` is head-major like the spikes).
    ``g_pre_out``: where to write g_pre, with pre's shape and row stride (e.g.
    the matching column slice of a wider gradient buffer)."""
    _cuda(g_spikes, pre, stats)
    D = pre.shape[-1]
    ld = _row_stride(pre)
    strided_ok = ld is not None and ld >= D and (ld == D or (D % 128 == 0 and ld % 4 == 0))
    if g_pre_out is not None:
        if not strided_ok or _row_stride(g_pre_out) != ld or g_pre_out.shape != pre.shape \
                or g_pre_out.dtype != pre.dtype:
            raise RuntimeError("g_pre_out must match pre's shape, dtype and row stride")
    elif not strided_ok or ld != D:
        pre, ld = pre.contiguous(), D
    g_spikes = g_spikes.contiguous()
    if g_spikes.dtype not in (torch.float32, torch.float16, torch.bfloat16):
        g_spikes = g_spikes.float()
    rows = pre.numel() // D
    R = rows // T
    dev = pre.device
    g_pre = g_pre_out if g_pre_out is not None else torch.empty(pre.shape, dtype=pre.dtype, device=dev)
    gg = torch.empty(D, dtype=torch.float32, device=dev) if need_gamma else None
    gb = torch.empty(D, dtype=torch.float32, device=dev) if need_beta else None
    glb = torch.empty(1, dtype=torch.float32, device=dev) if need_lif_beta else None
    gpb = torch.empty(D, dtype=torch.float32, device=dev) if need_bias else None
    pb = None if bias is None else bias.detach().float().contiguous()
    hd, sl = heads if heads is not None else (0, 1)
    wsb = int(_lib.load().spk_ln_lif_bwd_workspace_bytes(T, R, D))
    ws = torch.empty(wsb // 4, dtype=torch.float32, device=dev)
    g = None if ln_gamma is None else ln_gamma.detach().float().contiguous()
    bt = None if ln_beta is None else ln_beta.detach().float().contiguous()
    b, th, vr = (_scalar_f32(v, dev) for v in (lif_beta, lif_vth, lif_vr))
    _lib.call("spk_ln_lif_bwd", _lib.ptr(g_spikes), _lib.dtype_code(g_spikes), _lib.ptr(pre), _lib.dtype_code(pre),
              _lib.ptr(pb), _lib.ptr(stats), _lib.ptr(g), _lib.ptr(bt), _lib.ptr(b), _lib.ptr(th), _lib.ptr(vr),
              float(in_gain), _lib.SURROGATE[surrogate], float(k), T, R, D, ld, hd, sl, _lib.ptr(g_pre), _lib.ptr(gg),
              _lib.ptr(gb), _lib.ptr(gpb), _lib.ptr(glb), _lib.ptr(ws), wsb, _lib.stream_ptr(dev),
              tag="ln_lif_bwd D=%d" % D,
              work=dict(bytes=rows * D * (g_spikes.element_size() + 2 * pre.element_size()) + rows * 8))
    return g_pre, gg, gb, glb, gpb


def linear(A, W, bias=None):
    """``A @ W.T + bias`` in fp32 from bf16 ``A [M, K]`` and ``W [N, K]``."""
    _cuda(A, W)
    A = A.contiguous()
    W = W.contiguous()
    M, K = A.numel() // A.shape[-1], A.shape[-1]
    N = W.shape[0]
    out = torch.empty((M, N), dtype=torch.float32, device=A.device)
    bias = None if bias is None else bias.float().contiguous()
    _lib.call("spk_linear_fwd", _lib.ptr(A), _lib.ptr(W), _lib.ptr(bias), _lib.ptr(out), M, K, N,
              _lib.stream_ptr(A.device), tag="linear K=%d N=%d" % (K, N), work=dict(flops=2.0 * M * K * N))
    return out


def linear_grads_ok(g, w_or_x):
    """Shapes the training Linear gradient kernels take: 2-D-able bf16
    tensors whose feature sizes are multiples of 8, 16-byte aligned."""
    return (g.is_cuda and g.dtype == torch.bfloat16 and w_or_x.dtype == torch.bfloat16 and g.shape[-1] % 8 == 0
            and w_or_x.shape[-1] % 8 == 0 and g.data_ptr() % 16 == 0 and w_or_x.data_ptr() % 16 == 0)


def linear_dgrad(G, W):
    """``G @ W`` in fp32 for ``G`` bf16 ``[M, N]`` and the Linear weight ``W`` bf16
    ``[N, K]``: the input gradient of ``x @ W.T``."""
    _cuda(G, W)
    G = G.reshape(-1, G.shape[-1]).contiguous()
    W = W.contiguous()
    M, N = G.shape
    K = W.shape[1]
    out = torch.empty((M, K), dtype=torch.float32, device=G.device)
    _lib.call("spk_linear_dgrad", _lib.ptr(G), _lib.ptr(W), _lib.ptr(out), M, N, K, _lib.stream_ptr(G.device),
              tag="linear_dgrad N=%d K=%d" % (N, K),
              work=dict(flops=2.0 * M * N * K, bytes=(M * N + N * K) * 2 + M * K * 4))
    return out


def linear_wgrad(G, X):
    """``G.T @ X`` in fp32 for ``G`` bf16 ``[M, N]`` and ``X`` bf16 ``[M, K]``: the
    weight gradient of ``x @ W.T``, summed over the M rows."""
    _cuda(G, X)
    G = G.reshape(-1, G.shape[-1]).contiguous()
    X = X.reshape(-1, X.shape[-1]).contiguous()
    M, N = G.shape
    K = X.shape[1]
    out = torch.empty((N, K), dtype=torch.float32, device=G.device)
    wsb = int(_lib.load().spk_linear_wgrad_workspace_bytes(M, N, K))
    ws = torch.empty(max(wsb, 16) // 4, dtype=torch.float32, device=G.device)
    _lib.call("spk_linear_wgrad", _lib.ptr(G), _lib.ptr(X), _lib.ptr(out), _lib.ptr(ws), wsb, M, N, K,
              _lib.stream_ptr(G.device), tag="linear_wgrad N=%d K=%d" % (N, K),
              work=dict(flops=2.0 * M * N * K, bytes=(M * N + M * K) * 2 + N * K * 4))
    return out


def ssa(q, k, v, T, B, H, variant, scale, lif_beta, lif_vth, lif_vr, in_gain=1.0, mask=None, causal=False,
        out_dtype=torch.bfloat16, want_attn=False):
    """Spiking attention core + output LIF on head-merged bf16 spikes.

    ``q``: ``[T*B, Nq, H*dh]``, ``k``/``v``: ``[T*B, Nk, H*dh]``.  ``mask``:
    None, or a tensor broadcastable to ``[T, B, H, Nq, Nk]`` (nonzero = keep);
    ``causal=True`` uses the built-in key <= query mask instead.
    Returns ``(spikes [T*B, Nq, H*dh], attn fp32 [T*B, H, Nq, dh] or None)``.
    """
    _cuda(q, k, v, mask)
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    Nq, D = q.shape[-2], q.shape[-1]
    Nk = k.shape[-2]
    dh = D // H
    dev = q.device
    out = torch.empty(q.shape, dtype=out_dtype, device=dev)
    attn = torch.empty((T * B, H, Nq, dh), dtype=torch.float32, device=dev) if want_attn else None
    mask_mode, mptr, strides = 0, None, (0, 0, 0, 0)
    m8 = None
    if causal:
        mask_mode = 1
    elif mask is not None:
        m8 = mask_to_u8(mask, T, B, H, Nq, Nk)
        mask_mode, mptr = 2, m8.data_ptr()
        strides = tuple(m8.stride(i) for i in range(4))
    sc, b, th, vr = (_scalar_f32(x, dev) for x in (scale, lif_beta, lif_vth, lif_vr))
    _lib.call("spk_ssa_fwd", _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), int(variant), mask_mode, mptr, *strides,
              _lib.ptr(sc), _lib.ptr(b), _lib.ptr(th), _lib.ptr(vr), float(in_gain), T, B, H, Nq, Nk, dh,
              _lib.ptr(out), _lib.DTYPE_CODE[out_dtype], _lib.ptr(attn), _lib.stream_ptr(dev),
              tag="ssa Nq=%d Nk=%d" % (Nq, Nk),
              work=dict(flops=4.0 * T * B * H * Nq * Nk * dh,
                        bytes=(q.numel() + k.numel() + v.numel()) * 2 + out.numel() * out.element_size()
                        + (attn.numel() * 4 if attn is not None else 0)
                        + (_distinct_bytes(m8) if m8 is not None else 0)))
    return out, attn


def ssa_heads(q, k, v, T, variant, scale, lif_beta, lif_vth, lif_vr, in_gain=1.0, out_dtype=torch.bfloat16,
              want_attn=False):
    """Unmasked attention core + output LIF on head-split bf16 spikes (any
    strides with a unit stride along the head dimension): ``q`` ``[T*B, H, Nq,
    dh]``, ``k``/``v`` ``[T*B, H, Nk, dh]``, Nq, Nk <= 256.  Returns ``(spikes
    [T*B, Nq, H*dh], a fp32 [T*B, Nq, H*dh] or None)``: ``a`` is the LIF input
    ``scale * O``, token-major like the spikes."""
    _cuda(q, k, v)
    q, k, v = (t if t.dtype == torch.bfloat16 else t.to(torch.bfloat16) for t in (q, k, v))
    TB, H, Nq, dh = q.shape
    Nk = k.shape[2]
    dev = q.device
    out = torch.empty((TB, Nq, H * dh), dtype=out_dtype, device=dev)
    attn = torch.empty((TB, Nq, H * dh), dtype=torch.float32, device=dev) if want_attn else None
    sc, b, th, vr = (_scalar_f32(x, dev) for x in (scale, lif_beta, lif_vth, lif_vr))
    _lib.call("spk_ssa_fwd_heads", _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _head_strides(q, k, v), int(variant),
              _lib.ptr(sc), _lib.ptr(b), _lib.ptr(th), _lib.ptr(vr), float(in_gain), T, TB // T, H, Nq, Nk, dh,
              _lib.ptr(out), _lib.DTYPE_CODE[out_dtype], _lib.ptr(attn), _lib.stream_ptr(dev),
              tag="ssa Nq=%d Nk=%d" % (Nq, Nk),
              work=dict(flops=4.0 * TB * H * Nq * Nk * dh,
                        bytes=(q.numel() + k.numel() + v.numel()) * 2 + out.numel() * out.element_size()
                        + (attn.numel() * 4 if attn is not None else 0)))
    return out, attn


def _distinct_bytes(t):
    """Bytes of memory behind a (possibly broadcast, stride-0) tensor."""
    return t.untyped_storage().nbytes()


def _head_strides(*ts):
    """(t*b, head, position) element strides of [TB, H, N, d] tensors, packed
    as a ctypes int64 array; the d stride must be 1."""
    import ctypes
    vals = []
    for t in ts:
        if t.stride(-1) != 1:
            raise RuntimeError("attention operands need unit stride along the head dimension")
        vals += [t.stride(0), t.stride(1), t.stride(2)]
    return (ctypes.c_int64 * len(vals))(*vals)


def _masked_short_args(q, k, v, mask, T):
    TB, H, Nq, dh = q.shape
    Nk = k.shape[2]
    B = TB // T
    m8, ms = None, (0, 0, 0, 0)
    if mask is not None:
        m8 = mask_to_u8(mask, T, B, H, Nq, Nk)
        ms = tuple(m8.stride(i) for i in range(4))
    return TB, H, Nq, Nk, dh, B, m8, ms


def attn_masked_train_fwd(q, k, v, mask, scale, T, variant):
    """``scale * ((S * M) V)`` token-major fp32 ``[TB, Nq, H*dh]`` for head-major
    spikes ``q [TB, H, Nq, dh]``, ``k / v [TB, H, Nk, dh]`` (one dtype), Nq, Nk,
    dh <= 64; ``mask`` None or broadcastable as for ``ssa``; ``variant`` 1 XNOR
    with the log-distance bias, 0 plain."""
    _cuda(q, k, v, mask)
    TB, H, Nq, Nk, dh, B, m8, ms = _masked_short_args(q, k, v, mask, T)
    a = torch.empty((TB, Nq, H * dh), dtype=torch.float32, device=q.device)
    sc = _scalar_f32(scale.detach() if isinstance(scale, torch.Tensor) else scale, q.device)
    _lib.call("spk_attn_masked_train_fwd", _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.dtype_code(q),
              _head_strides(q, k, v), _lib.ptr(m8), *ms, int(variant), _lib.ptr(sc), T, B, H, Nq, Nk, dh,
              _lib.ptr(a), _lib.stream_ptr(q.device), tag="attn_masked_train_fwd",
              work=dict(flops=4.0 * TB * H * Nq * Nk * dh))
    return a


def attn_masked_train_bwd(q, k, v, mask, scale, T, variant, g):
    """Backward of ``attn_masked_train_fwd`` from ``g = dL/da`` (fp32, token-major):
    ``(dq, dk, dv)`` shaped and typed like q, k, v, and dL/dscale."""
    _cuda(q, k, v, mask, g)
    TB, H, Nq, Nk, dh, B, m8, ms = _masked_short_args(q, k, v, mask, T)
    g = g.float().contiguous()
    # the gradients are written with the operands' own strides
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    if (dq.stride(), dk.stride(), dv.stride()) != (q.stride(), k.stride(), v.stride()):
        raise RuntimeError("attn_masked_train_bwd needs dense q, k, v (contiguous in some dimension order)")
    part = torch.empty(TB * H, dtype=torch.float32, device=q.device)
    sc = _scalar_f32(scale.detach() if isinstance(scale, torch.Tensor) else scale, q.device)
    _lib.call("spk_attn_masked_train_bwd", _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.dtype_code(q),
              _head_strides(q, k, v), _lib.ptr(m8), *ms, int(variant), _lib.ptr(sc), T, B, H, Nq, Nk, dh,
              _lib.ptr(g), _lib.ptr(dq),
              _lib.ptr(dk), _lib.ptr(dv), _lib.ptr(part), _lib.stream_ptr(q.device), tag="attn_masked_train_bwd",
              work=dict(flops=10.0 * TB * H * Nq * Nk * dh))
    return dq, dk, dv, part.sum()


def mask_to_u8(mask, T, B, H, Nq, Nk):
    """uint8 view of an attention mask, expanded (stride 0) to [T, B, H, Nq, Nk].

    Accepts the reference's T-folded masks ``[T*B, 1|H, Nq, Nk]`` and any mask
    broadcastable to ``[B, H, Nq, Nk]``.
    """
    if mask.dtype == torch.uint8 and mask.dim() == 5 and tuple(mask.shape) == (T, B, H, Nq, Nk):
        return mask  # already converted
    m = (mask != 0).to(torch.uint8)
    if m.dim() == 4 and m.shape[0] == T * B and T * B != B:
        m = m.reshape(T, B, *m.shape[1:])
    else:
        while m.dim() < 4:
            m = m.unsqueeze(0)
        m = m.unsqueeze(0)
    m = m.expand(T, B, H, Nq, Nk)
    if m.stride(-1) != 1:
        m = m.contiguous()
    return m


def embed_pe_lif(tokens, emb, emb_scale, pe, lif_beta, lif_vth, lif_vr, T, in_gain=1.0, out_dtype=torch.bfloat16):
    """``LIF(T-fold(emb[tokens]*emb_scale + pe[:N]))`` -> spikes ``[T*B, N, D]``."""
    _cuda(tokens, emb, pe)
    tokens = tokens.to(torch.int64).contiguous()
    B, N = tokens.shape
    V, D = emb.shape
    emb = emb.float().contiguous()
    pe = pe.reshape(-1, D).float().contiguous()
    dev = tokens.device
    out = torch.empty((T * B, N, D), dtype=out_dtype, device=dev)
    bad = torch.zeros(1, dtype=torch.int32, device=dev)
    b, th, vr = (_scalar_f32(x, dev) for x in (lif_beta, lif_vth, lif_vr))
    _lib.call("spk_embed_pe_lif_fwd", _lib.ptr(tokens), _lib.ptr(emb), float(emb_scale), _lib.ptr(pe), _lib.ptr(b),
              _lib.ptr(th), _lib.ptr(vr), float(in_gain), T, B, N, D, V, _lib.ptr(out), _lib.DTYPE_CODE[out_dtype],
              _lib.ptr(bad), _lib.stream_ptr(dev), tag="embed_pe_lif",
              work=dict(bytes=B * N * (8 + 8 * D) + T * B * N * D * out.element_size()))
    return out, bad


def patch_im2col(img, patch):
    """``[B, C, H, W]`` fp32 -> bf16 ``[B*(H/p)*(W/p), 2*C*p*p]`` (hi | lo split)."""
    _cuda(img)
    img = img.float().contiguous()
    B, C, H, W = img.shape
    K = C * patch * patch
    out = torch.empty((B * (H // patch) * (W // patch), 2 * K), dtype=torch.bfloat16, device=img.device)
    _lib.call("spk_patch_im2col", _lib.ptr(img), B, C, H, W, patch, _lib.ptr(out), _lib.stream_ptr(img.device),
              tag="patch_im2col", work=dict(bytes=img.numel() * 4 + out.numel() * 2))
    return out


def synth_text_lines(B, seed, H=64, W=1024, L=None, V=256, device="cuda"):
    """On-device synthetic text-line batch: images ``[B, 1, H, W]`` fp32
    (U(0, 0.2) background, 5-40 black rectangles of side 8-20 px each) and,
    with ``L``, byte targets ``[B, L]`` int64 in ``[0, V)``; a function of
    ``seed`` only (counter-based hash), reproducible on the CPU."""
    dev = torch.device(device)
    if dev.type != "cuda":
        raise RuntimeError("synth_text_lines runs on a CUDA device")
    img = torch.empty((B, 1, H, W), dtype=torch.float32, device=dev)
    tok = torch.empty((B, L), dtype=torch.int64, device=dev) if L else None
    _lib.call("spk_synth_text_lines", _lib.ptr(img), B, H, W, int(seed) & 0xFFFFFFFFFFFFFFFF, _lib.ptr(tok),
              int(L or 0), V, _lib.stream_ptr(dev), tag="synth_text_lines",
              work=dict(bytes=img.numel() * 4 + (tok.numel() * 8 if tok is not None else 0)))
    return img, tok


class _CEOverT(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, targets, ignore_index, label_smoothing, bad):
        T, V = logits.shape[0], logits.shape[-1]
        rows = logits[0].numel() // V
        dev = logits.device
        out = torch.empty(3, dtype=torch.float32, device=dev)
        grad = torch.empty_like(logits) if ctx.needs_input_grad[0] else None
        ws = torch.empty(int(_lib.load().spk_ce_over_t_workspace_bytes(rows)), dtype=torch.uint8, device=dev)
        _lib.call("spk_ce_over_t", _lib.ptr(logits), _lib.DTYPE_CODE[logits.dtype], _lib.ptr(targets), T, rows, V,
                  int(ignore_index), float(label_smoothing), _lib.ptr(out), _lib.ptr(grad), _lib.ptr(ws), ws.numel(),
                  _lib.ptr(bad), _lib.stream_ptr(dev), tag="ce_over_t",
                  work=dict(bytes=logits.numel() * logits.element_size() * (2 if grad is not None else 1)))
        ctx.save_for_backward(grad, out)
        loss, acc = out[0], out[1]
        ctx.mark_non_differentiable(acc)
        return loss, acc

    @staticmethod
    def backward(ctx, g_loss, g_acc):
        grad, out = ctx.saved_tensors
        return grad * (g_loss * out[2]).to(grad.dtype), None, None, None, None


def ce_over_t(logits, targets, ignore_index=-100, label_smoothing=0.0):
    """Training loss and metric of the OCR seq2seq in one pass: the mean over
    the T steps of ``CrossEntropyLoss(ignore_index, label_smoothing)`` of each
    step's logits, and the token accuracy of the argmax of the T-averaged
    logits over non-ignored targets.  ``logits``: ``[T, ..., V]`` fp32 or
    bf16; ``targets``: ``[...]`` int64.  Returns ``(loss, accuracy, bad)``;
    ``loss`` is differentiable, ``bad`` a device flag set by out-of-range
    targets."""
    _cuda(logits, targets)
    if logits.dtype not in (torch.float32, torch.bfloat16):
        logits = logits.float()
    logits = logits.contiguous()
    targets = targets.to(torch.int64).contiguous()
    if targets.numel() * logits.shape[-1] * logits.shape[0] != logits.numel():
        raise RuntimeError("targets %s do not match logits %s" % (tuple(targets.shape), tuple(logits.shape)))
    bad = torch.zeros(1, dtype=torch.int32, device=logits.device)
    loss, acc = _CEOverT.apply(logits, targets, ignore_index, label_smoothing, bad)
    return loss, acc, bad


def device_error_check(device=None):
    """Synchronise and raise if a kernel's bounded wait gave up."""
    _lib.call("spk_device_error_check", _lib.stream_ptr(device))


# ------------------------------------------------- training-path XNOR attention core


def xnor_train_combine(qm, rv, w, scale, TB, H):
    """``(qm + rv + w) * scale`` -> token-major ``[TB, Nq, H*dh]`` fp32; ``qm``
    ``[B, Nq, dh]``, ``rv`` ``[Nq, B*dh]``, ``w`` ``[B, 1, dh]`` fp32, ``B = TB*H``."""
    _cuda(qm, rv, w)
    B, Nq, dh = qm.shape
    qm, rv, w = qm.contiguous(), rv.contiguous(), w.contiguous()
    sc = _scalar_f32(scale.detach() if isinstance(scale, torch.Tensor) else scale, qm.device)
    out = torch.empty((TB, Nq, H * dh), dtype=torch.float32, device=qm.device)
    _lib.call("spk_xnor_train_combine", _lib.ptr(qm), _lib.ptr(rv), _lib.ptr(w), _lib.ptr(sc), _lib.ptr(out), TB, H,
              Nq, dh, _lib.stream_ptr(qm.device), tag="xnor_train_combine",
              work=dict(bytes=3 * out.numel() * 4))
    return out


def xnor_train_grad_prep(g, out, scale, H, dh):
    """From the token-major gradient ``g`` and forward output ``out``
    (``[TB, Nq, H*dh]`` fp32): ``(g_heads [B, Nq, 2dh] bf16, g_rows [Nq, 2, B, dh]
    bf16, gcol [B, dh] fp32, sum(g * out))`` with ``gs = g * scale`` split hi | lo."""
    _cuda(g, out)
    g = g.float().contiguous()
    out = out.contiguous()
    TB, Nq, D = g.shape
    B = TB * H
    dev = g.device
    C = int(_lib.load().spk_xnor_train_prep_chunks(Nq))
    g_heads = torch.empty((B, Nq, 2 * dh), dtype=torch.bfloat16, device=dev)
    g_rows = torch.empty((Nq, 2, B, dh), dtype=torch.bfloat16, device=dev)
    gcol_part = torch.empty((C, B, dh), dtype=torch.float32, device=dev)
    gsc_part = torch.empty((C, B * dh // 4), dtype=torch.float32, device=dev)
    sc = _scalar_f32(scale.detach() if isinstance(scale, torch.Tensor) else scale, dev)
    _lib.call("spk_xnor_train_grad_prep", _lib.ptr(g), _lib.ptr(out), _lib.ptr(sc), _lib.ptr(g_heads),
              _lib.ptr(g_rows), _lib.ptr(gcol_part), _lib.ptr(gsc_part), TB, H, Nq, dh, _lib.stream_ptr(dev),
              tag="xnor_train_grad_prep", work=dict(bytes=g.numel() * 16))
    return g_heads, g_rows, gcol_part.sum(0), gsc_part.sum()


def xnor_train_grad_finish(ke, rg, u, dk32, TB, H, out_dtype):
    """``(dk, dv)`` head-major ``[B, Nk, dh]`` in ``out_dtype``: ``dv = ke + rg^P + u``,
    ``dk = dk32``; ``rg`` ``[Nk, B*dh]``, ``u`` ``[B, dh]``."""
    _cuda(ke, rg, u, dk32)
    B, Nk, dh = ke.shape
    ke, rg, u, dk32 = ke.contiguous(), rg.contiguous(), u.contiguous(), dk32.contiguous()
    dk = torch.empty((B, Nk, dh), dtype=out_dtype, device=ke.device)
    dv = torch.empty((B, Nk, dh), dtype=out_dtype, device=ke.device)
    _lib.call("spk_xnor_train_grad_finish", _lib.ptr(ke), _lib.ptr(rg), _lib.ptr(u), _lib.ptr(dk32), _lib.ptr(dk),
              _lib.ptr(dv), _lib.DTYPE_CODE[out_dtype], TB, H, Nk, dh, _lib.stream_ptr(ke.device),
              tag="xnor_train_grad_finish", work=dict(bytes=ke.numel() * 20))
    return dk, dv


def xnor_train_n_major(x):
    """``x`` ``[B, N, d]`` -> ``[N, B*d]`` with ``out[n, b*d:(b+1)*d] = x[b, n]``
    (the n-major operand of ``R @ V``).  Rows of ``d`` elements must span a
    multiple of 16 bytes."""
    _cuda(x)
    B, N, d = x.shape
    row_bytes = d * x.element_size()
    if row_bytes % 16:
        raise ValueError(f"xnor_train_n_major: rows of {row_bytes} bytes are not a multiple of 16")
    x = x.contiguous()
    out = torch.empty((N, B * d), dtype=x.dtype, device=x.device)
    _lib.call("spk_xnor_train_n_major", _lib.ptr(x), _lib.ptr(out), B, N, row_bytes, _lib.stream_ptr(x.device),
              tag="xnor_train_n_major", work=dict(bytes=2 * x.numel() * x.element_size()))
    return out


def xnor_train_combine_lif(qm, rv, w, scale, TB, H, T, lif_beta, lif_vth, lif_vr, in_gain=1.0,
                           spike_dtype=torch.float32):
    """``xnor_train_combine`` followed by the output LIF over the T-major fold:
    ``(a [TB, Nq, H*dh] fp32, spikes like a in spike_dtype)``."""
    _cuda(qm, rv, w)
    B, Nq, dh = qm.shape
    dev = qm.device
    qm, rv, w = qm.contiguous(), rv.contiguous(), w.contiguous()
    sc = _scalar_f32(scale.detach() if isinstance(scale, torch.Tensor) else scale, dev)
    b, th, vr = (_scalar_f32(v, dev) for v in (lif_beta, lif_vth, lif_vr))
    a = torch.empty((TB, Nq, H * dh), dtype=torch.float32, device=dev)
    s = torch.empty((TB, Nq, H * dh), dtype=spike_dtype, device=dev)
    _lib.call("spk_xnor_train_combine_lif", _lib.ptr(qm), _lib.ptr(rv), _lib.ptr(w), _lib.ptr(sc), _lib.ptr(b),
              _lib.ptr(th), _lib.ptr(vr), float(in_gain), _lib.ptr(a), _lib.ptr(s), _lib.DTYPE_CODE[spike_dtype], T, TB,
              H, Nq, dh, _lib.stream_ptr(dev), tag="xnor_train_combine_lif",
              work=dict(bytes=a.numel() * (16 + s.element_size())))
    return a, s


def xnor_train_grad_prep_lif(g_spikes, a, scale, H, dh, T, lif_beta, lif_vth, lif_vr, in_gain=1.0,
                             surrogate="superspike", k=4.0, need_lif_beta=False):
    """``xnor_train_grad_prep`` after the output LIF's backward: from dL/dspikes
    and the pre-activation ``a``; returns ``(g_heads, g_rows, gcol [B, dh],
    sum(dL/da * a), LIF beta gradient [1] or None)``."""
    _cuda(g_spikes, a)
    if g_spikes.dtype not in (torch.float32, torch.float16, torch.bfloat16):
        g_spikes = g_spikes.float()
    g_spikes = g_spikes.contiguous()
    a = a.contiguous()
    TB, Nq, D = a.shape
    B = TB * H
    dev = a.device
    C = int(_lib.load().spk_xnor_train_prep_chunks(Nq))
    X = TB // T * H * dh // 4
    g_heads = torch.empty((B, Nq, 2 * dh), dtype=torch.bfloat16, device=dev)
    g_rows = torch.empty((Nq, 2, B, dh), dtype=torch.bfloat16, device=dev)
    gcol_part = torch.empty((C, B, dh), dtype=torch.float32, device=dev)
    gsc_part = torch.empty((C, X), dtype=torch.float32, device=dev)
    gb_part = torch.empty((C, X), dtype=torch.float32, device=dev) if need_lif_beta else None
    sc = _scalar_f32(scale.detach() if isinstance(scale, torch.Tensor) else scale, dev)
    b, th, vr = (_scalar_f32(v, dev) for v in (lif_beta, lif_vth, lif_vr))
    _lib.call("spk_xnor_train_grad_prep_lif", _lib.ptr(g_spikes), _lib.dtype_code(g_spikes), _lib.ptr(a), _lib.ptr(sc),
              _lib.ptr(b), _lib.ptr(th), _lib.ptr(vr), float(in_gain), _lib.SURROGATE[surrogate], float(k),
              _lib.ptr(g_heads), _lib.ptr(g_rows), _lib.ptr(gcol_part), _lib.ptr(gsc_part), _lib.ptr(gb_part), T, TB,
              H, Nq, dh, _lib.stream_ptr(dev), tag="xnor_train_grad_prep_lif",
              work=dict(bytes=a.numel() * (4 + g_spikes.element_size() + 8)))
    return g_heads, g_rows, gcol_part.sum(0), gsc_part.sum(), None if gb_part is None else gb_part.sum().reshape(1)
