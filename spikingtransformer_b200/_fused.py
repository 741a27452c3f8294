"""Plumbing shared by the module classes: cached bf16 weight copies, packed
device-side LIF parameters and the Linear -> LayerNorm -> LIF call.

Derived state only (never saved in the state dict): caches are keyed on the
source tensor's storage pointer and version counter, so an optimizer step or
``load_state_dict`` invalidates them without a host synchronisation.
"""

import weakref

import torch

from . import ops


def _key(*ts):
    return tuple((t.data_ptr(), t._version, t.device, t.dtype) for t in ts)


def bf16_weight(lin, duplicate=False):
    """bf16 copy of ``lin.weight`` ([N, K]); with ``duplicate`` the columns are
    repeated, [W | W] ([N, 2K]), for split-precision inputs."""
    w = lin.weight
    attr = "_spk_w2" if duplicate else "_spk_w"
    k = _key(w)
    cached = getattr(lin, attr, None)
    if cached is not None and cached[0] == k:
        return cached[1]
    with torch.no_grad():
        wb = w.detach().reshape(w.shape[0], -1).to(torch.bfloat16)
        if duplicate:
            wb = torch.cat([wb, wb], dim=1)
        wb = wb.contiguous()
    object.__setattr__(lin, attr, (k, wb))
    return wb


def lif_params(lif):
    """fp32 device tensor [beta, v_th, v_reset] of a LIF module (cached)."""
    beta_src = lif.beta_raw if lif.learn_beta else lif.beta
    k = _key(beta_src, lif.v_th, lif.v_reset)
    cached = getattr(lif, "_spk_params", None)
    if cached is not None and cached[0] == k:
        return cached[1]
    with torch.no_grad():
        b = torch.sigmoid(beta_src.detach()) if lif.learn_beta else beta_src.detach()
        p = torch.stack([b.float().reshape(()), lif.v_th.detach().float().reshape(()),
                         lif.v_reset.detach().float().reshape(())]).contiguous()
    object.__setattr__(lif, "_spk_params", (k, p))
    return p


def split_bf16(x):
    """fp32 ``[..., K]`` -> bf16 ``[..., 2K]`` = [hi | lo] with hi + lo ~ x."""
    x = x.float()
    hi = x.to(torch.bfloat16)
    lo = (x - hi.float()).to(torch.bfloat16)
    return torch.cat([hi, lo], dim=-1)


def lin_ln_lif(x, lin, ln, lif, T, t_broadcast=False, residual=None, spike_dtype=torch.bfloat16,
               want_spikes=True, want_ln_out=False):
    """``lif(ln(lin(x)))`` through the fused kernel.

    ``x``: bf16 (used as is: exact for spike counts) or fp32 (split into two
    bf16 terms against [W | W]).  Returns ``(spikes [rows, N], ln_out)``.
    """
    if x.dtype == torch.bfloat16:
        A, W = x, bf16_weight(lin)
    else:
        A, W = split_bf16(x), bf16_weight(lin, duplicate=True)
    K = A.shape[-1]
    p = lif_params(lif)
    return ops.linear_ln_lif(A.reshape(-1, K), W, lin.bias, ln.weight, ln.bias, ln.eps, p[0:1], p[1:2], p[2:3], T,
                             in_gain=lif.in_gain, t_broadcast=t_broadcast, spike_dtype=spike_dtype,
                             residual=residual, want_spikes=want_spikes, want_ln_out=want_ln_out)


_SPIKE_COUNTS = {}


# the residual connections of the training path go through LNLIFResidualFunction
# (False: spikes and a separate add, the composition the fused form is tested against)
RESIDUAL_FUSION = True


def mark_spike_counts(t, bf16=None):
    """Record that ``t`` holds spike counts (small non-negative integers, exact
    in bf16), with its bf16 copy if one exists; returns ``t``.  The record
    lasts while ``t`` lives and is ignored once ``t`` is modified in place."""
    key = id(t)

    def drop(_ref, key=key):
        entry = _SPIKE_COUNTS.get(key)
        if entry is not None and entry[0] is _ref:
            del _SPIKE_COUNTS[key]

    _SPIKE_COUNTS[key] = (weakref.ref(t, drop), t._version, bf16)
    return t


def spike_counts_bf16(t):
    """The bf16 form of a residual-stream tensor without a host
    synchronisation: ``t`` when it is bf16, the recorded copy (or a cast) when
    ``t`` was produced by this package's spiking modules and has not been
    modified since; None when exactness cannot be known without reading ``t``
    back (the caller then takes the per-module path, which works on any
    values)."""
    if t.dtype == torch.bfloat16:
        return t
    entry = _SPIKE_COUNTS.get(id(t))
    if entry is None or entry[0]() is not t or entry[1] != t._version:
        return None
    return entry[2] if entry[2] is not None else t.to(torch.bfloat16)


def fast_path_ok(*tensors, module=None):
    """Inference fast path: CUDA tensors and no autograd graph to build."""
    if not all(t is None or t.is_cuda for t in tensors):
        return False
    if torch.is_grad_enabled():
        if any(t is not None and t.requires_grad for t in tensors):
            return False
        if module is not None and any(p.requires_grad for p in module.parameters()):
            return False
    return True


class LNLIFFunction(torch.autograd.Function):
    """``lif(ln(pre + bias))`` for training in two kernels (``ops.ln_lif_fwd`` /
    ``ops.ln_lif_bwd``): the LayerNorm, the LIF scan and both backwards fused
    over the T steps of each token.  ``bias`` is the preceding Linear's (or
    None): its GEMM runs without one and the bias gradient comes out of the
    backward kernel.  Gradients: pre, the Linear bias, the LayerNorm weight and
    bias, and the LIF beta.  Spikes are written in ``spike_dtype`` (0/1 are
    exact in every float type), head-major when ``heads = (head_dim, seq_len)``."""

    @staticmethod
    def forward(ctx, pre, bias, ln_weight, ln_bias, lif_beta, v_th, v_reset, eps, k, surrogate, in_gain, T,
                spike_dtype, heads=None):
        spikes, stats = ops.ln_lif_fwd(pre, ln_weight, ln_bias, eps, lif_beta, v_th, v_reset, T, in_gain,
                                       spike_dtype=spike_dtype, bias=bias, heads=heads)
        ctx.save_for_backward(pre, stats, bias, ln_weight, ln_bias, lif_beta, v_th, v_reset)
        ctx.k, ctx.surrogate, ctx.in_gain, ctx.T, ctx.heads = float(k), surrogate, float(in_gain), int(T), heads
        return spikes

    @staticmethod
    def backward(ctx, g_spikes):
        pre, stats, pb, w, b, lb, vth, vr = ctx.saved_tensors
        need = ctx.needs_input_grad
        g_pre, gw, gb, glb, gpb = ops.ln_lif_bwd(g_spikes, pre, stats, w, b, lb, vth, vr, ctx.T, ctx.in_gain,
                                                 ctx.surrogate, ctx.k, need_gamma=need[2], need_beta=need[3],
                                                 need_lif_beta=need[4], bias=pb,
                                                 need_bias=pb is not None and need[1], heads=ctx.heads)
        gpb = gpb.to(pb.dtype) if gpb is not None else None
        gw = gw.to(w.dtype) if gw is not None else None
        gb = gb.to(b.dtype) if gb is not None else None
        glb = glb.reshape(lb.shape).to(lb.dtype) if glb is not None else None
        return g_pre, gpb, gw, gb, glb, None, None, None, None, None, None, None, None, None


class LNLIFResidualFunction(torch.autograd.Function):
    """``residual + lif(ln(pre + bias))`` for training: the residual connection
    of a transformer layer (``Encoder.py:19-22``, ``Decoder.py:18-24``) fused
    into the LayerNorm->LIF forward kernel (``ops.ln_lif_fwd_residual``), which
    under bf16 autocast also writes the bf16 copy the next layer's GEMMs read
    (recorded with ``mark_spike_counts``).  Backward: ``dL/dresidual =
    dL/dout``, and ``ops.ln_lif_bwd`` with ``g_spikes = dL/dout``."""

    @staticmethod
    def forward(ctx, pre, bias, ln_weight, ln_bias, lif_beta, v_th, v_reset, eps, k, surrogate, in_gain, T,
                residual):
        want_bf16 = _autocast_bf16(residual)
        out, stats, outb = ops.ln_lif_fwd_residual(pre, ln_weight, ln_bias, eps, lif_beta, v_th, v_reset, T,
                                                   residual.detach(), in_gain, bias=bias, want_bf16=want_bf16)
        ctx.save_for_backward(pre, stats, bias, ln_weight, ln_bias, lif_beta, v_th, v_reset)
        ctx.k, ctx.surrogate, ctx.in_gain, ctx.T = float(k), surrogate, float(in_gain), int(T)
        if outb is not None:
            mark_spike_counts(out, bf16=outb)
        return out

    @staticmethod
    def backward(ctx, g_out):
        pre, stats, pb, w, b, lb, vth, vr = ctx.saved_tensors
        need = ctx.needs_input_grad
        g_pre, gw, gb, glb, gpb = ops.ln_lif_bwd(g_out, pre, stats, w, b, lb, vth, vr, ctx.T, ctx.in_gain,
                                                 ctx.surrogate, ctx.k, need_gamma=need[2], need_beta=need[3],
                                                 need_lif_beta=need[4], bias=pb,
                                                 need_bias=pb is not None and need[1])
        gpb = gpb.to(pb.dtype) if gpb is not None else None
        gw = gw.to(w.dtype) if gw is not None else None
        gb = gb.to(b.dtype) if gb is not None else None
        glb = glb.reshape(lb.shape).to(lb.dtype) if glb is not None else None
        return g_pre, gpb, gw, gb, glb, None, None, None, None, None, None, None, g_out if need[12] else None


class QKVLNLIF(torch.autograd.Function):
    """The Q, K and V LayerNorm->LIF passes of a self-attention over the column
    slices of one ``[rows, 3D]`` GEMM output (``x [Wq; Wk; Wv]^T``).  Each pass
    reads its slice in place, and the backward writes the three input
    gradients into one ``[rows, 3D]`` buffer, so the GEMM before it has a
    single input gradient (one dgrad GEMM over K = 3D, accumulated in fp32).
    ``per`` holds, for Q, K and V, ``(eps, k, surrogate, in_gain)``; the
    tensors are, for Q, K and V, ``(bias, ln weight, ln bias, lif beta, v_th,
    v_reset)``."""

    @staticmethod
    def forward(ctx, pre3, T, per, spike_dtype, heads, *tensors):
        D = pre3.shape[-1] // 3
        outs, stats = [], []
        for i in range(3):
            pb, w, b, lb, vth, vr = tensors[6 * i:6 * i + 6]
            eps, _, _, gain = per[i]
            s, st = ops.ln_lif_fwd(pre3[..., i * D:(i + 1) * D], w, b, eps, lb, vth, vr, T, gain,
                                   spike_dtype=spike_dtype, bias=pb, heads=heads)
            outs.append(s)
            stats.append(st)
        ctx.save_for_backward(pre3, *stats, *tensors)
        ctx.T, ctx.per, ctx.heads = int(T), per, heads
        return tuple(outs)

    @staticmethod
    def backward(ctx, *g_spikes):
        pre3, st0, st1, st2 = ctx.saved_tensors[:4]
        tensors = ctx.saved_tensors[4:]
        stats = (st0, st1, st2)
        need = ctx.needs_input_grad
        D = pre3.shape[-1] // 3
        g3 = torch.empty_like(pre3)
        grads = []
        for i in range(3):
            pb, w, b, lb, vth, vr = tensors[6 * i:6 * i + 6]
            _, k, surrogate, gain = ctx.per[i]
            n = 5 + 6 * i  # index of this pass's bias among forward's inputs
            gs = g_spikes[i]
            if gs is None:
                shape = (pre3.shape[0] * pre3.shape[1] // ctx.heads[1], D // ctx.heads[0], ctx.heads[1],
                         ctx.heads[0]) if ctx.heads is not None else pre3[..., :D].shape
                gs = torch.zeros(shape, dtype=pre3.dtype, device=pre3.device)
            _, gw, gb, glb, gpb = ops.ln_lif_bwd(gs, pre3[..., i * D:(i + 1) * D], stats[i], w, b, lb, vth, vr,
                                                 ctx.T, gain, surrogate, k, need_gamma=need[n + 1],
                                                 need_beta=need[n + 2], need_lif_beta=need[n + 3], bias=pb,
                                                 need_bias=pb is not None and need[n], heads=ctx.heads,
                                                 g_pre_out=g3[..., i * D:(i + 1) * D])
            grads += [gpb.to(pb.dtype) if gpb is not None else None, gw.to(w.dtype) if gw is not None else None,
                      gb.to(b.dtype) if gb is not None else None,
                      glb.reshape(lb.shape).to(lb.dtype) if glb is not None else None, None, None]
        return (g3, None, None, None, None, *grads)


def qkv_ln_lif_train(x, projs, lns, lifs, heads, xb=None):
    """Q, K, V spikes (head-major ``[TB, H, N, dh]``) of a self-attention on the
    autograd path from one GEMM: under bf16 autocast and with D % 128 == 0,
    ``x [Wq; Wk; Wv]^T`` in one ``LinearBF16`` and the three LayerNorm->LIF
    passes in ``QKVLNLIF``; None when that path does not apply (the caller
    then projects separately)."""
    D = projs[0].out_features
    if xb is None:
        xb = bf16_input(x)
    if (xb is None or D % 128 or heads[0] % 4 or D % heads[0]
            or any(p.out_features != D or p.weight.dtype != torch.float32 for p in projs)
            or not all(_ln_lif_fusable(x, D, ln, lif) for ln, lif in zip(lns, lifs))
            or len({lif.n_steps for lif in lifs}) != 1):
        return None
    w3 = torch.cat([p.weight for p in projs], dim=0)
    pre3 = LinearBF16.apply(x, w3, xb, w3.detach().to(torch.bfloat16))
    per = [(ln.eps, lif._k_host, lif.surrogate, lif.in_gain) for ln, lif in zip(lns, lifs)]
    tensors = []
    for p, ln, lif in zip(projs, lns, lifs):
        tensors += [p.bias, ln.weight, ln.bias, lif.effective_beta(), lif.v_th, lif.v_reset]
    dt = torch.get_autocast_dtype(x.device.type)
    return QKVLNLIF.apply(pre3, lifs[0].n_steps, per, dt, heads, *tensors)


def _ln_lif_fusable(x, D, ln, lif):
    return (x.is_cuda and isinstance(ln, torch.nn.LayerNorm) and ln.elementwise_affine
            and tuple(ln.normalized_shape) == (D,) and x.shape[0] % lif.n_steps == 0
            and ops.ln_lif_ok(lif.n_steps, D))


def _lif_args(ln, lif):
    return (ln.weight, ln.bias, lif.effective_beta(), lif.v_th, lif.v_reset, ln.eps, lif._k_host, lif.surrogate,
            lif.in_gain, lif.n_steps)


def ln_lif(x, ln, lif, bias=None):
    """``lif(ln(x + bias))[0]`` on the autograd path: the fused training kernels
    when the shapes allow (CUDA, affine LayerNorm over the last dimension), the
    module composition otherwise (``Lif.py:288-441`` over torch's LayerNorm)."""
    if _ln_lif_fusable(x, x.shape[-1], ln, lif):
        return LNLIFFunction.apply(x, bias, *_lif_args(ln, lif), torch.float32)
    return lif(ln(x if bias is None else x + bias))[0]


class LinearBF16(torch.autograd.Function):
    """``x W^T`` (no bias) for the bf16-autocast training path: bf16 operands,
    fp32 accumulation, bf16 output.  ``xb`` / ``wb`` are bf16 copies of x and W
    made once and shared by every GEMM that reads them (Q, K and V read the same
    x).  The backward GEMMs write the input and weight gradients directly in
    x's and W's dtypes (fp32 output from fp32 accumulation), so no cast kernel
    runs in either direction and fp32 gradients are summed in fp32.  They are
    torch's (cuBLAS): this package's tcgen05 gradient GEMMs
    (``ops.linear_dgrad`` / ``ops.linear_wgrad``) compute the same products
    but take 1.1-1.6x cuBLAS's time at the training shapes."""

    @staticmethod
    def forward(ctx, x, w, xb, wb):
        with torch.autocast(x.device.type, enabled=False):
            y = torch.nn.functional.linear(xb, wb)
        ctx.save_for_backward(xb, wb)
        ctx.dtypes = (x.dtype, w.dtype)
        return y

    @staticmethod
    def backward(ctx, gy):
        xb, wb = ctx.saved_tensors
        tx, tw = ctx.dtypes
        g2 = gy.reshape(-1, gy.shape[-1]).to(torch.bfloat16)
        dx = dw = None
        with torch.autocast(gy.device.type, enabled=False):
            if ctx.needs_input_grad[0]:
                dx = torch.mm(g2, wb) if tx == torch.bfloat16 else torch.mm(g2, wb, out_dtype=torch.float32).to(tx)
                dx = dx.view(*gy.shape[:-1], wb.shape[1])
            if ctx.needs_input_grad[1]:
                dw = torch.mm(g2.t(), xb.reshape(-1, xb.shape[-1]), out_dtype=torch.float32).to(tw)
        return dx, dw, None, None


def _autocast_bf16(x):
    return x.is_cuda and torch.is_autocast_enabled(x.device.type) and \
        torch.get_autocast_dtype(x.device.type) == torch.bfloat16


def bf16_input(x):
    """The bf16 copy of an activation that ``lin_ln_lif_train`` GEMMs read under
    bf16 autocast (None otherwise); made once and passed to every consumer.  A
    residual-stream tensor written by ``LNLIFResidualFunction`` already has
    one (recorded with ``mark_spike_counts``)."""
    if _autocast_bf16(x):
        if x.dtype == torch.bfloat16:
            return x.detach()
        entry = _SPIKE_COUNTS.get(id(x))
        if entry is not None and entry[0]() is x and entry[1] == x._version and entry[2] is not None:
            return entry[2]
        return x.detach().to(torch.bfloat16)
    return None


def _linear_nobias(x, lin, xb):
    if xb is None:
        xb = bf16_input(x)
    if xb is None or lin.weight.dtype not in (torch.float32, torch.bfloat16):
        return torch.nn.functional.linear(x, lin.weight)
    return LinearBF16.apply(x, lin.weight, xb, bf16_weight(lin))


def lin_ln_lif_train(x, lin, ln, lif, narrow=False, heads=None, xb=None, residual=None):
    """``lif(ln(lin(x)))[0]`` on the autograd path.  With the fused kernels the
    GEMM runs without the bias, which the LayerNorm->LIF kernels add and
    differentiate; under bf16 autocast it is ``LinearBF16`` on ``xb`` (the
    shared bf16 copy of x from ``bf16_input``, made here if not given).
    ``narrow``: under autocast, write the spikes in the autocast dtype; meant
    for spikes whose consumer is a GEMM that reads that dtype.  ``heads =
    (head_dim, n)`` for ``x`` ``[TB, n, D]``: return the spikes as ``[TB,
    D/head_dim, n, head_dim]``, written in that layout by the kernel where it
    can.  ``residual``: return ``residual + lif(ln(lin(x)))[0]`` instead (the
    residual connection of a transformer layer), fused into the LayerNorm->LIF
    kernel where it applies."""
    D = lin.out_features
    if residual is not None:
        if not narrow and heads is None and _ln_lif_fusable(x, D, ln, lif) and RESIDUAL_FUSION:
            pre = _linear_nobias(x, lin, xb)
            if ops.ln_lif_residual_ok(pre, residual) and residual.shape[-1] == D:
                return LNLIFResidualFunction.apply(pre, lin.bias, *_lif_args(ln, lif), residual)
            return residual + LNLIFFunction.apply(pre, lin.bias, *_lif_args(ln, lif), torch.float32, None)
        return residual + lin_ln_lif_train(x, lin, ln, lif, narrow=narrow, heads=heads, xb=xb)
    if _ln_lif_fusable(x, D, ln, lif):
        pre = _linear_nobias(x, lin, xb)
        dt = torch.float32
        if narrow and torch.is_autocast_enabled(x.device.type):
            dt = torch.get_autocast_dtype(x.device.type)
        direct = heads is not None and D % 128 == 0 and heads[0] % 4 == 0 and D % heads[0] == 0
        out = LNLIFFunction.apply(pre, lin.bias, *_lif_args(ln, lif), dt, heads if direct else None)
        if heads is None or direct:
            return out
    else:
        out = ln_lif(lin(x), ln, lif)
    hd, n = heads
    return out.view(-1, n, D // hd, hd).transpose(1, 2)
