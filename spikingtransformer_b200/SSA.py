"""Spiking self-attention: drop-in for ``Triton_Layers/SSA.py``.

``SSAMultiHeadAttention`` (XNOR scores + log-distance bias + learnable scale,
``SSA.py:103-258``) and ``SSAMultiHeadAttention_`` (plain ``Q K^T``, fixed
0.125 scale after ``@ V``, ``SSA.py:10-100``) keep the reference constructor
arguments, submodule names (q_proj, k_proj, v_proj, lnq..lno, lifq..lifo,
out_proj, scale) and ``forward(query, key=None, value=None,
attention_mask=None) -> [B', N, D]`` fp32 spikes.

Inference (no autograd graph needed): three fused Linear->LN->LIF kernels
produce Q, K, V spikes, ``spk_ssa_fwd`` computes the attention core and the
``lifs`` LIF, and a fourth fused kernel applies out_proj->lno->lifo.
Training: the reference composition (torch Linear / LayerNorm / einsum) over
the LIF kernels of this package, so autograd sees the same graph as the
reference.
"""

from typing import Optional

import torch
import torch.nn as nn

from . import ops
from ._fused import (bf16_input, fast_path_ok, lif_params, lin_ln_lif, lin_ln_lif_train, mark_spike_counts,
                     qkv_ln_lif_train)
from .Lif import LIF


class _SSACore(nn.Module):
    variant = 1

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

    # ---------------------------------------------------------------- fused path

    def _scale_tensor(self, device):
        raise NotImplementedError

    def _attend(self, q, k, v, T, mask, out_dtype=torch.bfloat16):
        """q [T*B, Nq, D], k/v [T*B, Nk, D] bf16 spikes -> lifs spikes."""
        TB = q.shape[0]
        p = lif_params(self.lifs)
        causal = False
        if isinstance(mask, str) and mask == "causal":
            causal, mask = True, None
        out, _ = ops.ssa(q, k, v, T, TB // T, self.n_heads, self.variant, self._scale_tensor(q.device),
                         p[0:1], p[1:2], p[2:3], in_gain=self.lifs.in_gain, mask=mask, causal=causal,
                         out_dtype=out_dtype)
        return out

    def key_value_spikes(self, src):
        """K and V spikes (bf16 [T*B, Nk, D]) of a bf16 key/value source; a
        cross-attention over a fixed source (the encoder output during
        decoding) can compute them once and pass them to ``_fast``."""
        T = self.lifq.n_steps
        TB, Nk, D = src.shape
        k = lin_ln_lif(src, self.k_proj, self.lnk, self.lifk, T)[0].view(TB, Nk, D)
        v = lin_ln_lif(src, self.v_proj, self.lnv, self.lifv, T)[0].view(TB, Nk, D)
        return k, v

    def _fast(self, x, kv=None, mask=None, kv_spikes=None):
        """Residual step on bf16 spike counts: ``x += SSA(x, kv, kv)`` in place.

        ``x``: [T*B, Nq, D] bf16; ``kv``: [T*B, Nk, D] bf16 or None (self);
        ``mask``: None, "causal", or a mask accepted by ``ops.ssa``;
        ``kv_spikes``: (K, V) from ``key_value_spikes(kv)``, used instead of
        projecting ``kv`` again.
        """
        T = self.lifq.n_steps
        TB, Nq, D = x.shape
        q = lin_ln_lif(x, self.q_proj, self.lnq, self.lifq, T)[0].view(TB, Nq, D)
        k, v = self.key_value_spikes(x if kv is None else kv) if kv_spikes is None else kv_spikes
        a = self._attend(q, k, v, T, mask)
        lin_ln_lif(a, self.out_proj, self.lno, self.lifo, T, residual=x.view(-1, D), want_spikes=False)
        return x

    def _fast_public(self, query, key, value, attention_mask):
        T = self.lifq.n_steps
        TB, N, D = query.shape
        Nk = key.shape[1]
        q = lin_ln_lif(query, self.q_proj, self.lnq, self.lifq, T)[0].view(TB, N, D)
        k = lin_ln_lif(key, self.k_proj, self.lnk, self.lifk, T)[0].view(TB, Nk, D)
        v = lin_ln_lif(value, self.v_proj, self.lnv, self.lifv, T)[0].view(TB, Nk, D)
        a = self._attend(q, k, v, T, attention_mask)
        out = lin_ln_lif(a, self.out_proj, self.lno, self.lifo, T, spike_dtype=torch.float32)[0]
        return mark_spike_counts(out.view(TB, N, D))

    # ---------------------------------------------------------------- autograd path

    def _scores(self, q, k):
        raise NotImplementedError

    def _reference_forward(self, query, key, value, attention_mask, residual=None):
        TB, N, D = query.shape
        Nk = key.shape[1]
        # Q, K, V spikes feed only the attention products, so under autocast
        # they are written in its dtype (0/1 exact), per head [TB, H, N, dh]
        hd = self.d_head
        # one bf16 copy of each distinct input for all the GEMMs that read it
        qb = bf16_input(query)
        kb = qb if key is query else bf16_input(key)
        vb = kb if value is key else (qb if value is query else bf16_input(value))
        qkv = None
        if key is query and value is query:
            # self-attention: one GEMM for Q, K and V
            qkv = qkv_ln_lif_train(query, (self.q_proj, self.k_proj, self.v_proj), (self.lnq, self.lnk, self.lnv),
                                   (self.lifq, self.lifk, self.lifv), (hd, N), xb=qb)
        if qkv is not None:
            q, k, v = qkv
        else:
            q = lin_ln_lif_train(query, self.q_proj, self.lnq, self.lifq, narrow=True, heads=(hd, N), xb=qb)
            k = lin_ln_lif_train(key, self.k_proj, self.lnk, self.lifk, narrow=True, heads=(hd, Nk), xb=kb)
            v = lin_ln_lif_train(value, self.v_proj, self.lnv, self.lifv, narrow=True, heads=(hd, Nk), xb=vb)
        # token-major [TB, N, D]; the lifs LIF is per neuron, so it commutes with
        # the reference's transpose back from heads (SSA.py:242-247)
        s = self._combine_lif(q, k, v, attention_mask)
        return lin_ln_lif_train(s, self.out_proj, self.lno, self.lifo, residual=residual)

    def _combine_lif(self, q, k, v, mask):
        """lifs(attention core) -> token-major spikes [TB, N, H*dh]."""
        return self.lifs(self._combine(q, k, v, mask))[0]

    def add_to(self, x, key=None, value=None, attention_mask=None):
        """``x + self(x, key, value, attention_mask)``, the residual connection of
        an encoder / decoder layer (``Encoder.py:19``, ``Decoder.py:18-21``); on
        the autograd path the add is fused into the output LayerNorm->LIF kernel."""
        key = x if key is None else key
        value = x if value is None else value
        if fast_path_ok(x, key, value, attention_mask, module=self):
            return x + self._fast_public(x, key, value, attention_mask)
        return self._reference_forward(x, key, value, attention_mask, residual=x)

    def forward(self, query: torch.Tensor, key: Optional[torch.Tensor] = None, value: Optional[torch.Tensor] = None,
                attention_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        key = query if key is None else key
        value = query if value is None else value
        if fast_path_ok(query, key, value, attention_mask, module=self):
            return self._fast_public(query, key, value, attention_mask)
        return self._reference_forward(query, key, value, attention_mask)

    def extra_repr(self) -> str:
        return f"d_model={self.d_model}, n_heads={self.n_heads}, d_head={self.d_head}"


class SSAMultiHeadAttention(_SSACore):
    """XNOR spiking attention (``SSA.py:103-258``).

    ``S = Dh - (sum q + sum k - 2 q.k) + R``, ``R[i,j] = max(0,
    ceil(log2((max(Nq,Nk)-1)/(|i-j|+1))))``, ``S *= mask``,
    ``out = LIF_{v_th=.5}((S * scale) @ V)``; ``alpha``, ``causal``,
    ``learnable_alpha`` and ``dropout`` are accepted and unused, as in the
    reference.
    """

    variant = 1

    def __init__(self, d_model: int, n_heads: int, alpha: Optional[float] = None, causal: bool = False,
                 learnable_alpha: bool = False, dropout: float = 0.0, n_steps: int = 1, bias: bool = True):
        super().__init__(d_model, n_heads, n_steps, bias)
        self.scale = nn.Parameter(torch.sqrt(torch.tensor(1.0 / (d_model // n_heads))), requires_grad=True)

    def _scale_tensor(self, device):
        return self.scale.detach()

    @staticmethod
    def xnor_attention_scores(q, k):
        dh = q.shape[-1]
        qk = torch.einsum("bhld,bhmd->bhlm", q, k)
        return dh - (q.sum(-1, keepdim=True) + k.sum(-1, keepdim=True).transpose(2, 3) - 2 * qk)

    def xnor_attention(self, Q, K):
        """``Dh - Hamming(Q, K)`` as in ``SSA.py:145-165``."""
        return self.xnor_attention_scores(Q, K)

    def get_log_pe_bias(self, seq_len, device):
        """Self-attention log-distance bias (``SSA.py:167-175``)."""
        return self.get_log_pe_bias_cross(seq_len, seq_len, device)

    def get_log_pe_bias_cross(self, seq_len_q, seq_len_k, device):
        """``max(0, ceil(log2((max(Lq,Lk)-1)/(|i-j|+1))))``, ``SSA.py:177-201``."""
        iq = torch.arange(seq_len_q, device=device).unsqueeze(1)
        jk = torch.arange(seq_len_k, device=device).unsqueeze(0)
        dist = (iq - jk).abs().float()
        L = max(seq_len_q, seq_len_k)
        return torch.ceil(torch.log2((L - 1) / (dist + 1))).clamp(min=0)

    def _log_pe_bias(self, seq_len_q, seq_len_k, device):
        """``get_log_pe_bias_cross`` for this package's own kernels, built once
        per (Lq, Lk, device) and shared: they only read it."""
        key = (seq_len_q, seq_len_k, device)
        R = _LOG_PE_CACHE.get(key)
        if R is None:
            R = _LOG_PE_CACHE[key] = self.get_log_pe_bias_cross(seq_len_q, seq_len_k, device)
        return R

    def _combine_lif(self, q, k, v, mask):
        lifs = self.lifs
        TB, H, Nq, dh = q.shape
        if (mask is None and q.is_cuda and k.shape[2] <= 256 and dh <= 256 and dh % 4 == 0
                and 1 <= lifs.n_steps <= 4 and TB % lifs.n_steps == 0):
            # the core and the lifs LIF in the same kernels; spikes feed only
            # the output projection, so under autocast they take its dtype
            dt = torch.float32
            if torch.is_autocast_enabled(q.device.type):
                dt = torch.get_autocast_dtype(q.device.type)
            R = self._log_pe_bias(Nq, k.shape[2], q.device)
            return XnorLIF.apply(q, k, v, R, self.scale, lifs.effective_beta(), lifs.v_th, lifs.v_reset,
                                 lifs.in_gain, lifs.surrogate, lifs._k_host, lifs.n_steps, dt)
        return super()._combine_lif(q, k, v, mask)

    def _combine(self, q, k, v, mask):
        """Attention core before the lifs LIF: q [TB, H, Nq, dh], k / v [TB, H,
        Nk, dh] -> token-major [TB, Nq, H*dh]."""
        if mask is not None and masked_short_ok(q, k, self.lifs.n_steps):
            return MaskedShortAttention.apply(q, k, v, self.scale, mask, self.lifs.n_steps, 1)
        if mask is not None:
            a = self.xnor_attention(q, k)
            a = a + self.get_log_pe_bias_cross(q.shape[2], k.shape[2], q.device).unsqueeze(0).unsqueeze(0)
            return _token_major((a * mask * self.scale) @ v)
        # Without a mask the score matrix regroups exactly (spikes are 0/1):
        #   S V = 2 Q (K^T V) + (dh - |q|) (1^T V) - 1 (s^T V) + R V,  s_j = |k_j|,
        # so neither S nor its gradient is formed.
        dh = q.shape[-1]
        R = self._log_pe_bias(q.shape[2], k.shape[2], q.device)
        if q.is_cuda and k.shape[2] <= 256 and dh <= 256:
            return XnorScoreFree.apply(q, k, v, R, self.scale)
        # fp32 matmuls keep every integer term exact (sums below 2^24), whatever
        # the autocast state
        with torch.autocast(q.device.type, enabled=False):
            qf, kf, vf = q.float(), k.float(), v.float()
            m = 2.0 * (qf @ (kf.transpose(-2, -1) @ vf))
            m = m + (dh - qf.sum(-1, keepdim=True)) * vf.sum(-2, keepdim=True)
            m = m - kf.sum(-1).unsqueeze(-2) @ vf
            m = m + R @ vf
            return _token_major(m * self.scale)


def masked_short_ok(q, k, T):
    """The masked short-sequence attention kernels take this call: CUDA, Nq,
    Nk, dh <= 64, the T-fold divisible by T."""
    return (q.is_cuda and q.dim() == 4 and q.shape[2] <= 64 and k.shape[2] <= 64 and q.shape[3] <= 64
            and q.shape[0] % T == 0)


def _dense(t, dtype):
    """``t`` in ``dtype``, contiguous in some dimension order (one copy if not)."""
    if t.dtype != dtype:
        t = t.to(dtype)
    if not (t.is_contiguous() or t.transpose(1, 2).is_contiguous()):
        t = t.contiguous()
    return t


class MaskedShortAttention(torch.autograd.Function):
    """Masked attention core for sequences of at most 64 positions (the
    decoder's masked self-attention, ``SSA.py:234-242``; plain form
    ``SSA.py:81-84``): ``scale * ((S * mask) @ V)`` token-major fp32, with S
    the XNOR score plus the log-distance bias (``variant`` 1) or ``Q K^T``
    (0).  Forward and backward each run one kernel
    (``spk_attn_masked_train_fwd`` / ``_bwd``) with the score matrix in shared
    memory; gradients of Q, K, V (in their dtype) and of a learnable scale."""

    @staticmethod
    def forward(ctx, q, k, v, scale, mask, T, variant):
        dt = q.dtype if q.dtype in (torch.float32, torch.float16, torch.bfloat16) else torch.float32
        q, k, v = _dense(q, dt), _dense(k, dt), _dense(v, dt)
        with torch.autocast(q.device.type, enabled=False):
            a = ops.attn_masked_train_fwd(q, k, v, mask, scale, T, variant)
        ctx.save_for_backward(q, k, v, scale if isinstance(scale, torch.Tensor) else None)
        ctx.scale_value, ctx.mask, ctx.T, ctx.variant = scale, mask, T, variant
        return a

    @staticmethod
    def backward(ctx, g):
        q, k, v, scale_t = ctx.saved_tensors
        scale = scale_t if scale_t is not None else ctx.scale_value
        with torch.autocast(q.device.type, enabled=False):
            dq, dk, dv, gscale = ops.attn_masked_train_bwd(q, k, v, ctx.mask, scale, ctx.T, ctx.variant, g)
        if scale_t is not None and ctx.needs_input_grad[3]:
            gscale = gscale.reshape(scale_t.shape).to(scale_t.dtype)
        else:
            gscale = None
        return dq, dk, dv, gscale, None, None, None


def _token_major(a):
    """[TB, H, N, dh] -> [TB, N, H*dh]."""
    TB, H, N, dh = a.shape
    return a.transpose(1, 2).reshape(TB, N, H * dh)


def _split_bf16(x):
    """fp32 -> (hi, lo) bf16 with hi + lo equal to x to about 2^-16 relative."""
    hi = x.to(torch.bfloat16)
    return hi, (x - hi.float()).to(torch.bfloat16)


def _flat_bf16(t):
    """[TB, H, N, d] of any strides -> contiguous bf16 [TB*H, N, d] (no copy when
    it already is, else one pass)."""
    if t.dtype != torch.bfloat16 or not t.is_contiguous():
        out = torch.empty(t.shape, dtype=torch.bfloat16, device=t.device)
        out.copy_(t)
        t = out
    return t.view(-1, t.shape[-2], t.shape[-1])


_ONES = {}


def _ones_bf16(r, c, device):
    key = (r, c, device)
    t = _ONES.get(key)
    if t is None:
        t = _ONES[key] = torch.ones((r, c), dtype=torch.bfloat16, device=device)
    return t


# log-distance bias matrices of the attention kernels, by (Lq, Lk, device)
_LOG_PE_CACHE = {}


def _bmm32(a, b):
    """bf16 x bf16 -> fp32 batched product on the tensor cores."""
    return torch.bmm(a, b, out_dtype=torch.float32)


def _score_free_kernel_ok(q, k, v):
    """The score-free forward kernel takes these head-split operands: Nq, Nk <=
    256, a head width of 8..64 in steps of 8, unit stride along it and the
    other strides multiples of 8 elements, 16-byte aligned bf16 data."""
    if not (q.is_cuda and q.dim() == 4 and q.shape[2] <= 256 and k.shape[2] <= 256):
        return False
    dh = q.shape[3]
    if not (8 <= dh <= 64 and dh % 8 == 0):
        return False
    for t in (q, k, v):
        if t.dtype != torch.bfloat16 or t.stride(3) != 1 or t.data_ptr() % 16:
            return False
        if any(st <= 0 or st % 8 for st in t.stride()[:3]):
            return False
    return True


def _xnor_m(kb, vb):
    """``M = 2 K^T V - 1 (1^T V)^T`` in bf16 (exact: ``|M| <= Nk``), the small
    operand of the regrouped core's products."""
    kv = _bmm32(kb.transpose(1, 2), vb)
    cv = vb.sum(1, keepdim=True, dtype=torch.float32)
    return (2.0 * kv - cv).to(torch.bfloat16)


def _xnor_products(q, k, v, R):
    """Forward products of the regrouped core: ``(qb, kb, vb, Mb, Rb, qm, rv, w)``
    with ``m / scale = qm + rv^P + w`` (see ``XnorScoreFree``)."""
    TB, H, Nq, dh = q.shape
    Nk = k.shape[2]
    qb, kb, vb = (_flat_bf16(t) for t in (q, k, v))
    B = qb.shape[0]
    Rb = R.to(torch.bfloat16)
    kv = _bmm32(kb.transpose(1, 2), vb)                           # [B, dh, dh]
    # |k_j| as a product with a ones vector; then [1; dh - |k|]^T V gives
    # 1^T V and w in one product (all exact)
    sk = torch.mm(kb.view(-1, dh), _ones_bf16(dh, 1, kb.device), out_dtype=torch.float32).view(B, 1, Nk)
    lw = torch.cat([torch.ones_like(sk), dh - sk], dim=1).to(torch.bfloat16)   # [B, 2, Nk]
    cw = _bmm32(lw, vb)                                            # [B, 2, dh]
    cv, w = cw[:, :1], cw[:, 1:]
    Mb = (2.0 * kv - cv).to(torch.bfloat16)                        # exact: |M| <= Nk
    qm = _bmm32(qb, Mb)                                            # [B, Nq, dh]
    vn = ops.xnor_train_n_major(vb) if (dh * 2) % 16 == 0 else vb.permute(1, 0, 2).reshape(Nk, B * dh)
    rv = torch.mm(Rb, vn, out_dtype=torch.float32)
    return qb, kb, vb, Mb, Rb, qm, rv, w


def _xnor_backward(qb, kb, vb, Mb, Rb, g_heads, g_rows, gcol, meta):
    """dQ, dK, dV of the regrouped core from the prepared gradient."""
    (tq, sq), (tk, sk_), (tv, sv) = meta
    TB, H, Nq, dh = sq
    B = kb.shape[0]
    # dQ = G M^T with G = hi | lo against [M^T; M^T]: one fp32-accumulated
    # product, rounded once to q's dtype
    mt = Mb.transpose(1, 2)
    mt2 = torch.cat([mt, mt], dim=1)                               # [B, 2dh, dh]
    dq = torch.bmm(g_heads, mt2) if tq == torch.bfloat16 else _bmm32(g_heads, mt2).to(tq)
    # dM = Q^T G, E = 2 dM - 1 gcol^T, u = -1^T dM + dh gcol
    dm2 = _bmm32(qb.transpose(1, 2), g_heads)                      # [B, dh, 2dh]
    dm = dm2[..., :dh] + dm2[..., dh:]
    e = 2.0 * dm - gcol.unsqueeze(1)
    u = dh * gcol - dm.sum(1)
    eh, el = _split_bf16(e)
    # second split term accumulated in place into the first product's output
    bf = torch.ops.aten.baddbmm.dtype_out
    dk32 = _bmm32(vb, eh.transpose(1, 2))
    bf(dk32, vb, el.transpose(1, 2), torch.float32, out=dk32)      # V E^T
    ke = _bmm32(kb, eh)
    bf(ke, kb, el, torch.float32, out=ke)                          # K E
    rt = Rb.t()
    rg = torch.mm(rt, g_rows[:, 0].reshape(Nq, B * dh), out_dtype=torch.float32)
    torch.ops.aten.addmm.dtype_out(rg, rt, g_rows[:, 1].reshape(Nq, B * dh), torch.float32, out=rg)  # R^T G
    dk, dv = ops.xnor_train_grad_finish(ke, rg, u, dk32, TB, H, tk)
    return dq.view(sq), dk.view(sk_), dv.to(tv).view(sv)


class XnorScoreFree(torch.autograd.Function):
    """Score-free XNOR attention core on the tensor cores, for training.

    ``m = scale * [2 Q (K^T V) + (dh - |q|) (1^T V) - 1 (s^T V) + R V]`` with
    ``s_j = |k_j|``, which equals ``(S * scale) @ V`` for the reference's
    ``S = dh - (|q_i| + |k_j| - 2 q_i.k_j) + R`` (``SSA.py:145-165``,
    ``:177-201``, ``:235-240``) when Q, K, V are 0/1.  Grouped as
    ``m / scale = Q M + R V + 1 w^T`` with the small ``M = 2 K^T V - 1 (1^T V)^T``
    and ``w = (dh - s)^T V``.

    Forward: every operand is an integer that bf16 holds exactly (spikes,
    ``|M| <= Nk <= 256``, ``dh - s_j <= dh``, ``R <= 8``) and every product
    accumulates in fp32, so ``m / scale`` is exact and the output equals the
    fp32 formulation bit for bit.  Backward: the real-valued gradient operands
    are split into two bf16 terms (hi + lo, about 2^-16 relative); with
    ``E = 2 dM - 1 gcol^T`` (``gcol`` the column sums of the scaled gradient)
    the rank-one terms fold into the products: ``dQ = G M^T``,
    ``dK = V E^T``, ``dV = K E + R^T G + 1 u^T``.  Everything between the
    library GEMMs runs in three memory-bound kernels (``xnor_train.cu``).

    Inputs: q [TB, H, Nq, dh], k and v [TB, H, Nk, dh] (0/1 in any float
    dtype, any strides), R [Nq, Nk] fp32, scale a 0-d parameter.  Output: fp32
    token-major [TB, Nq, H*dh] (the layout the output projection reads).
    """

    @staticmethod
    def forward(ctx, q, k, v, R, scale):
        with torch.autocast("cuda", enabled=False):
            TB, H = q.shape[:2]
            qb, kb, vb, Mb, Rb, qm, rv, w = _xnor_products(q, k, v, R)
            out = ops.xnor_train_combine(qm, rv, w, scale, TB, H)
        ctx.save_for_backward(qb, kb, vb, Mb, Rb, out, scale)
        ctx.meta = ((q.dtype, q.shape), (k.dtype, k.shape), (v.dtype, v.shape))
        return out

    @staticmethod
    def backward(ctx, g):
        qb, kb, vb, Mb, Rb, out, scale = ctx.saved_tensors
        TB, H, Nq, dh = ctx.meta[0][1]
        with torch.autocast("cuda", enabled=False):
            g_heads, g_rows, gcol, gdot = ops.xnor_train_grad_prep(g, out, scale, H, dh)
            gscale = (gdot / scale.float()).reshape(scale.shape).to(scale.dtype)   # sum(g * m)
            dq, dk, dv = _xnor_backward(qb, kb, vb, Mb, Rb, g_heads, g_rows, gcol, ctx.meta)
        return dq, dk, dv, None, gscale


class XnorLIF(torch.autograd.Function):
    """``XnorScoreFree`` followed by the attention's output LIF (``lifs``,
    ``SSA.py:242``), both passes fused into the core's kernels: spikes come out
    token-major in ``spike_dtype`` (they feed only the output projection), and
    the backward runs the LIF's BPTT inside the gradient preparation.  Equal
    to ``lifs(XnorScoreFree(...))`` (the LIF kernels' arithmetic).  Gradients:
    Q, K, V, scale and the LIF beta."""

    @staticmethod
    def forward(ctx, q, k, v, R, scale, lif_beta, v_th, v_reset, in_gain, surrogate, k_sg, T, spike_dtype):
        with torch.autocast("cuda", enabled=False):
            TB, H = q.shape[:2]
            if spike_dtype in (torch.bfloat16, torch.float32) and _score_free_kernel_ok(q, k, v):
                # the forward kernel of the unmasked core (score-free, exact, the
                # LIF in its epilogue) reads the head-split operands in place and
                # writes the spikes and the LIF input a; the backward's small
                # product M is formed there
                spikes, a = ops.ssa_heads(q, k, v, T, 1, scale, lif_beta, v_th, v_reset, in_gain,
                                          out_dtype=spike_dtype, want_attn=True)
                qb, kb, vb = (_flat_bf16(t) for t in (q, k, v))
                Mb, Rb = None, R.to(torch.bfloat16)
            else:
                qb, kb, vb, Mb, Rb, qm, rv, w = _xnor_products(q, k, v, R)
                a, spikes = ops.xnor_train_combine_lif(qm, rv, w, scale, TB, H, T, lif_beta, v_th, v_reset,
                                                       in_gain, spike_dtype)
        ctx.save_for_backward(qb, kb, vb, Mb, Rb, a, scale, lif_beta, v_th, v_reset)
        ctx.meta = ((q.dtype, q.shape), (k.dtype, k.shape), (v.dtype, v.shape))
        ctx.lif = (float(in_gain), surrogate, float(k_sg), int(T))
        return spikes

    @staticmethod
    def backward(ctx, g):
        qb, kb, vb, Mb, Rb, a, scale, lb, vth, vr = ctx.saved_tensors
        TB, H, Nq, dh = ctx.meta[0][1]
        gain, surrogate, k_sg, T = ctx.lif
        need_lb = ctx.needs_input_grad[5]
        with torch.autocast("cuda", enabled=False):
            if Mb is None:
                Mb = _xnor_m(kb, vb)
            g_heads, g_rows, gcol, gdot, glb = ops.xnor_train_grad_prep_lif(
                g, a, scale, H, dh, T, lb, vth, vr, gain, surrogate, k_sg, need_lif_beta=need_lb)
            gscale = (gdot / scale.float()).reshape(scale.shape).to(scale.dtype)
            dq, dk, dv = _xnor_backward(qb, kb, vb, Mb, Rb, g_heads, g_rows, gcol, ctx.meta)
        glb = glb.reshape(lb.shape).to(lb.dtype) if glb is not None else None
        return dq, dk, dv, None, gscale, glb, None, None, None, None, None, None, None


class SSAMultiHeadAttention_(_SSACore):
    """Plain spiking attention (``SSA.py:10-100``):
    ``out = LIF_{v_th=.5}(((Q K^T) * mask) @ V * 0.125)``."""

    variant = 0

    def __init__(self, d_model: int, n_heads: int, alpha: Optional[float] = None, causal: bool = False,
                 learnable_alpha: bool = False, dropout: float = 0.0, n_steps: int = 1, bias: bool = True):
        super().__init__(d_model, n_heads, n_steps, bias)

    def _scale_tensor(self, device):
        c = getattr(self, "_spk_scale", None)
        if c is None or c.device != device:
            c = torch.full((1,), 0.125, dtype=torch.float32, device=device)
            object.__setattr__(self, "_spk_scale", c)
        return c

    def _combine(self, q, k, v, mask):
        if masked_short_ok(q, k, self.lifs.n_steps):
            return MaskedShortAttention.apply(q, k, v, self._scale_tensor(q.device), mask, self.lifs.n_steps, 0)
        a = q @ k.transpose(-2, -1)
        if mask is not None:
            a = a * mask
        return _token_major((a @ v) * 0.125)

