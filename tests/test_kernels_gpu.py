"""Kernel-level parity: libspk.so (through the C ABI) against the CPU oracle
and the golden fixtures made from the reference.

Rules (tests/parity.py): spikes bit-exact outside the 1e-4 near-threshold
band; membrane / LayerNorm outputs within 1e-3 relative; SSA spike-count
products bit-exact.
"""

import os

import pytest
import torch
import torch.nn.functional as F

import oracle
from oracle import modules as om
from parity import assert_spikes_match, assert_close_rel, membrane_history

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module")
def ops():
    from spikingtransformer_b200 import ops as o
    return o


def gen(seed):
    return torch.Generator().manual_seed(seed)


# ------------------------------------------------------------------ LIF


@pytest.mark.parametrize("spike_dtype", [torch.float32, torch.bfloat16, torch.uint8])
def test_lif_fwd_cfg1_bit_exact(ops, spike_dtype):
    # LIF forward at the CPU benchmark shape [T=4, B=8, N=128, D=256], tau=2
    g = gen(0)
    x = torch.randn(4, 8, 128, 256, generator=g) + 0.5
    x3 = x.reshape(4, 8, -1)
    s_ref, vf_ref = oracle.lif_forward(x3, 0.5, 1.0, 0.0, in_gain=0.5)
    s, vf = ops.lif_fwd(x3.to(DEV), 0.5, 1.0, 0.0, in_gain=0.5, spike_dtype=spike_dtype)
    assert torch.equal(s.float().cpu(), s_ref)
    assert torch.equal(vf.cpu(), vf_ref)


@pytest.mark.parametrize("N", [4 * 8 * 128 * 256 // 4, 1001, 8, 3])
def test_lif_fp8_and_packed_bit_spikes(ops, N):
    """fp8 (e4m3) and packed-bit spike outputs: the same trains as fp32 spikes,
    and the backward reads them back bit-exactly (vector path for N % 8 == 0,
    per-element path for a ragged last byte)."""
    T = 4
    g = gen(N)
    x = torch.randn(T, N, generator=g) + 0.5
    gs = torch.randn(T, N, generator=g)
    s_ref, vf_ref = oracle.lif_forward(x, 0.5, 1.0, 0.0, in_gain=0.5)
    xd = x.to(DEV)
    s8, vf8 = ops.lif_fwd(xd, 0.5, 1.0, 0.0, in_gain=0.5, spike_dtype=torch.float8_e4m3fn)
    assert s8.dtype == torch.float8_e4m3fn and torch.equal(s8.float().cpu(), s_ref)
    assert torch.equal(vf8.cpu(), vf_ref)
    sb, vfb = ops.lif_fwd(xd, 0.5, 1.0, 0.0, in_gain=0.5, spike_dtype="bits")
    assert sb.shape == (T, (N + 7) // 8) and sb.dtype == torch.uint8
    assert torch.equal(ops.unpack_spike_bits(sb, N).cpu(), s_ref)
    assert torch.equal(vfb.cpu(), vf_ref)
    if N % 8:  # bits past N in the last byte stay 0
        assert int(sb[:, -1].cpu().max()) < (1 << (N % 8))
    gx_ref, gb_ref = oracle.lif_backward(gs, None, x, s_ref, 0.5, 1.0, 0.0, in_gain=0.5)
    for spikes, packed in ((s8, False), (sb, True)):
        gx, gb = ops.lif_bwd(gs.to(DEV), None, xd, spikes, 0.5, 1.0, 0.0, in_gain=0.5, spikes_packed=packed)
        assert torch.equal(gx.cpu(), gx_ref)
        assert torch.allclose(gb.cpu().reshape(()), gb_ref, rtol=1e-4, atol=1e-4)


def test_lif_golden(ops, golden_dir):
    for c in torch.load(os.path.join(golden_dir, "lif.pt"), weights_only=False):
        x = c["x_in"].to(DEV)
        s, vf = ops.lif_fwd(x, c["beta"], c["v_th"], c["v_reset"])
        assert torch.equal(s.cpu(), c["spikes"]), c["dtype"]
        assert torch.equal(vf.cpu(), c["v_final"]), c["dtype"]
        gx, gb = ops.lif_bwd(c["g_spikes"].to(DEV), None, x, s, c["beta"], c["v_th"], c["v_reset"])
        assert torch.equal(gx.cpu(), c["grad_x"].to(gx.dtype))
        assert torch.allclose(gb.cpu().reshape(()), c["grad_beta"], rtol=1e-5, atol=1e-5)
        gx, gb = ops.lif_bwd(c["g_spikes"].to(DEV), c["g_vfinal"].to(DEV), x, s, c["beta"], c["v_th"], c["v_reset"])
        assert torch.equal(gx.cpu(), c["grad_x_vf"].to(gx.dtype))
        assert torch.allclose(gb.cpu().reshape(()), c["grad_beta_vf"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("T,N", [(1, 5), (3, 1023), (8, 4096), (13, 77), (20, 640), (64, 33)])
@pytest.mark.parametrize("surrogate", ["superspike", "arctan"])
def test_lif_shapes_and_surrogates(ops, T, N, surrogate):
    g = gen(T * 1000 + N)
    x = torch.randn(T, N, generator=g) + 0.3
    gs = torch.randn(T, N, generator=g)
    gvf = torch.randn(N, generator=g)
    s_ref, vf_ref = oracle.lif_forward(x, 0.8, 0.9, -0.1)
    s, vf = ops.lif_fwd(x.to(DEV), 0.8, 0.9, -0.1)
    assert torch.equal(s.cpu(), s_ref)
    assert torch.equal(vf.cpu(), vf_ref)
    gx_ref, gb_ref = oracle.lif_backward(gs, gvf, x, s_ref, 0.8, 0.9, -0.1, k=2.0, surrogate=surrogate)
    gx, gb = ops.lif_bwd(gs.to(DEV), gvf.to(DEV), x.to(DEV), s, 0.8, 0.9, -0.1, surrogate=surrogate, k=2.0)
    if surrogate == "superspike":
        assert torch.equal(gx.cpu(), gx_ref)
    else:
        assert torch.allclose(gx.cpu(), gx_ref, rtol=1e-6, atol=1e-7)
    assert torch.allclose(gb.cpu().reshape(()), gb_ref, rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("T,N", [(1, 128), (3, 5 * 1024 + 384), (4, 600 * 1024)])
@pytest.mark.parametrize("surrogate", ["superspike", "arctan"])
def test_lif_bwd_staged_inputs(ops, T, N, surrogate):
    """The backward that stages its inputs through shared memory with bulk
    copies (fp32 currents, T <= 4, N a multiple of 128): every spike format it
    reads, with and without g_vfinal, a partial last tile of 1024 neurons and
    more tiles than blocks."""
    g = gen(7 * N + T)
    x = torch.randn(T, N, generator=g) + 0.4
    gs = torch.randn(T, N, generator=g)
    gvf = torch.randn(N, generator=g)
    s_ref, _ = oracle.lif_forward(x, 0.7, 1.0, 0.0, in_gain=0.5)
    xd = x.to(DEV)
    for sd in (torch.bfloat16, torch.uint8, torch.float8_e4m3fn, "bits"):
        s, _ = ops.lif_fwd(xd, 0.7, 1.0, 0.0, in_gain=0.5, spike_dtype=sd)
        for gv in (None, gvf):
            gx_ref, gb_ref = oracle.lif_backward(gs, gv, x, s_ref, 0.7, 1.0, 0.0, k=2.0, in_gain=0.5,
                                                 surrogate=surrogate)
            gx, gb = ops.lif_bwd(gs.to(DEV), None if gv is None else gv.to(DEV), xd, s, 0.7, 1.0, 0.0,
                                 in_gain=0.5, surrogate=surrogate, k=2.0, spikes_packed=sd == "bits")
            what = "%s spikes, g_vfinal %s" % (sd, gv is not None)
            if surrogate == "superspike":
                assert torch.equal(gx.cpu(), gx_ref), what
            else:
                assert torch.allclose(gx.cpu(), gx_ref, rtol=1e-6, atol=1e-7), what
            assert torch.allclose(gb.cpu().reshape(()), gb_ref, rtol=1e-4, atol=1e-4), what


def test_lif_empty(ops):
    x = torch.empty(4, 0, device=DEV)
    s, vf = ops.lif_fwd(x, 0.9, 1.0, 0.0)
    assert s.shape == (4, 0)


def test_lif_rejects_cpu(ops):
    with pytest.raises(RuntimeError):
        ops.lif_fwd(torch.zeros(2, 3), 0.9, 1.0, 0.0)


def test_lif_rejects_long_T(ops):
    with pytest.raises(RuntimeError):
        ops.lif_fwd(torch.zeros(65, 8, device=DEV), 0.9, 1.0, 0.0)


# ------------------------------------------------------------------ Linear -> LN -> LIF


def ref_linear_ln_lif(A, W, bias, gamma, beta_ln, T, lif_beta, vth, vr, gain=1.0, t_broadcast=False, eps=1e-5):
    pre = A.float() @ W.float().t() + bias
    y = F.layer_norm(pre, (W.shape[0],), gamma, beta_ln, eps)
    if t_broadcast:
        y3 = y.unsqueeze(0).expand(T, *y.shape).reshape(T, -1)
    else:
        y3 = y.reshape(T, -1)
    s, _ = oracle.lif_forward(y3, lif_beta, vth, vr, in_gain=gain)
    vh = membrane_history(y3, lif_beta, vth, vr, gain)
    return s.reshape(-1, W.shape[0]), y, vh


def make_lin(seed, R, K, N, T, t_broadcast=False, counts=1, p=0.15):
    g = gen(seed)
    rows = R if t_broadcast else T * R
    A = torch.zeros(rows, K)
    for _ in range(counts):
        A += (torch.rand(rows, K, generator=g) < p).float()
    bound = 1.0 / K ** 0.5
    W = ((torch.rand(N, K, generator=g) * 2 - 1) * bound).to(torch.bfloat16)
    bias = (torch.rand(N, generator=g) * 2 - 1) * 0.01
    gamma = 1.0 + 0.1 * torch.randn(N, generator=g)
    beta_ln = 0.1 * torch.randn(N, generator=g)
    return A.to(torch.bfloat16), W, bias, gamma, beta_ln


@pytest.mark.parametrize("T,R,K,N", [
    (4, 256, 384, 384),     # QKV / out_proj shape
    (4, 96, 384, 1536),     # MLP expand (cluster of 4 CTAs)
    (4, 64, 1536, 384),     # MLP compress
    (2, 24, 32, 32),        # small model
    (3, 50, 64, 128),       # T not dividing 128, partial tiles
    (1, 300, 128, 64),
    (10, 37, 96, 512),
])
def test_linear_ln_lif(ops, T, R, K, N):
    A, W, bias, gamma, beta_ln = make_lin(T * 7 + R + K + N, R, K, N, T, counts=2)
    s_ref, y_ref, vh = ref_linear_ln_lif(A, W, bias, gamma, beta_ln, T, 0.9, 1.0, 0.0)
    s, y = ops.linear_ln_lif(A.to(DEV), W.to(DEV), bias.to(DEV), gamma.to(DEV), beta_ln.to(DEV), 1e-5, 0.9, 1.0,
                             0.0, T, want_ln_out=True, spike_dtype=torch.float32)
    assert_close_rel(y, y_ref, what="layernorm out")
    assert_spikes_match(s.reshape(T, -1), s_ref.reshape(T, -1), vh, 1.0, what="spikes")


@pytest.mark.parametrize("T,R,K,N,gain,vr,res", [
    (4, 256, 384, 384, 1.0, 0.0, False),
    (4, 256, 384, 384, 0.5, 0.0, True),     # out_proj with the residual add
    (4, 96, 384, 1536, 0.5, 0.0, False),    # MLP expand (cluster split)
    (4, 64, 1536, 384, 1.0, -0.25, True),   # MLP compress, non-zero reset
    (4, 50, 128, 128, 0.5, 0.0, True),      # token count not a multiple of 8
    (2, 100, 128, 256, 0.7, 0.125, True),
    (8, 40, 64, 128, 1.0, 0.0, False),
    (1, 300, 128, 64, 1.0, 0.0, True),
    (16, 20, 64, 64, 1.0, 0.0, True),
])
def test_linear_ln_lif_fast(ops, T, R, K, N, gain, vr, res):
    # bf16 spikes without the LayerNorm output: the kernel variant the model runs
    A, W, bias, gamma, beta_ln = make_lin(T * 13 + R + K + N, R, K, N, T, counts=2)
    s_ref, _, vh = ref_linear_ln_lif(A, W, bias, gamma, beta_ln, T, 0.9, 1.0, vr, gain=gain)
    resid = torch.randint(0, 5, (T * R, N), generator=gen(R)).to(torch.bfloat16) if res else None
    r_dev = resid.to(DEV) if res else None
    s, y = ops.linear_ln_lif(A.to(DEV), W.to(DEV), bias.to(DEV), gamma.to(DEV), beta_ln.to(DEV), 1e-5, 0.9, 1.0,
                             vr, T, in_gain=gain, residual=r_dev, spike_dtype=torch.bfloat16)
    assert y is None and s.dtype == torch.bfloat16
    assert_spikes_match(s.float().cpu().reshape(T, -1), s_ref.reshape(T, -1), vh, 1.0, what="spikes")
    if res:
        assert torch.equal(r_dev.float().cpu(), resid.float() + s.float().cpu())


@pytest.mark.parametrize("R,K,N,gain,vr,res", [
    (256, 384, 384, 1.0, 0.0, False),
    (256, 384, 384, 0.5, 0.0, True),     # out_proj: residual only, as the model calls it
    (96, 384, 1536, 0.5, 0.0, False),    # MLP expand, 6-CTA cluster
    (64, 1536, 384, 1.0, -0.25, True),   # MLP compress into the residual, non-zero reset
    (200, 256, 128, 0.5, 0.0, True),     # last tile holds one group of 8 tokens
    (104, 128, 64, 1.0, 0.0, False),     # one 32-column chunk per warp
    (72, 192, 512, 0.8, 0.1, True),      # 2-CTA cluster of 256 columns, K not a multiple of 64
    (40, 384, 256, 1.0, 0.0, False),
    (48, 768, 384, 0.5, 0.0, False),     # K > 512: the 8-warp epilogue without a residual
])
def test_linear_ln_lif_t4_transposed_epilogue(ops, R, K, N, gain, vr, res):
    """T = 4 with a token count divisible by 8 and one bf16 output (the spikes,
    or the residual stream without the spikes): the epilogue that reads TMEM
    transposed and writes through TMA stores."""
    T = 4
    A, W, bias, gamma, beta_ln = make_lin(T * 17 + R + K + N, R, K, N, T, counts=2)
    s_ref, _, vh = ref_linear_ln_lif(A, W, bias, gamma, beta_ln, T, 0.9, 1.0, vr, gain=gain)
    args = (A.to(DEV), W.to(DEV), bias.to(DEV), gamma.to(DEV), beta_ln.to(DEV), 1e-5, 0.9, 1.0, vr, T)
    if res:
        resid = torch.randint(0, 5, (T * R, N), generator=gen(R + 1)).to(torch.bfloat16)
        r_dev = resid.to(DEV)
        s, y = ops.linear_ln_lif(*args, in_gain=gain, residual=r_dev, want_spikes=False)
        assert s is None and y is None
        s = r_dev.float().cpu() - resid.float()
        assert set(s.unique().tolist()) <= {0.0, 1.0}
    else:
        s, y = ops.linear_ln_lif(*args, in_gain=gain, spike_dtype=torch.bfloat16)
        s = s.float().cpu()
    assert_spikes_match(s.reshape(T, -1), s_ref.reshape(T, -1), vh, 1.0, what="spikes")


@pytest.mark.parametrize("T,R,K,N,gain,vr", [
    (4, 300, 512, 384, 1.0, 0.0),    # patch embedding (split-bf16 pixels, K = 2 x 256)
    (4, 200, 256, 1536, 0.5, 0.0),   # 6-CTA cluster, last tile partial
    (3, 129, 128, 128, 0.7, 0.1),    # T not a power of two, non-zero reset
    (1, 64, 64, 64, 1.0, 0.0),
    (8, 150, 192, 512, 0.5, -0.25),
])
def test_linear_ln_lif_t_broadcast_bf16(ops, T, R, K, N, gain, vr):
    """t-broadcast rows with bf16 spikes: one pre-activation per token drives
    the LIF at every step (the patch-embedding path)."""
    A, W, bias, gamma, beta_ln = make_lin(T * 3 + R + K + N, R, K, N, T, t_broadcast=True)
    s_ref, _, vh = ref_linear_ln_lif(A, W, bias, gamma, beta_ln, T, 0.9, 1.0, vr, gain=gain, t_broadcast=True)
    s, y = ops.linear_ln_lif(A.to(DEV), W.to(DEV), bias.to(DEV), gamma.to(DEV), beta_ln.to(DEV), 1e-5, 0.9, 1.0, vr,
                             T, in_gain=gain, t_broadcast=True, spike_dtype=torch.bfloat16)
    assert y is None and s.shape == (T * R, N)
    assert_spikes_match(s.float().cpu().reshape(T, -1), s_ref.reshape(T, -1), vh, 1.0, what="spikes")


def test_linear_ln_lif_cfg2_tau(ops):
    # fused Linear->LN->LIF at the cfg-2 feature sizes (tau=2 neuron), fewer rows
    T, R, K, N = 4, 2048, 384, 1536
    A, W, bias, _, _ = make_lin(2, R, K, N, T)
    gamma, beta_ln = torch.ones(N), torch.zeros(N)
    s_ref, y_ref, vh = ref_linear_ln_lif(A, W, bias, gamma, beta_ln, T, 0.5, 1.0, 0.0, gain=0.5)
    s, y = ops.linear_ln_lif(A.to(DEV), W.to(DEV), bias.to(DEV), gamma.to(DEV), beta_ln.to(DEV), 1e-5, 0.5, 1.0,
                             0.0, T, in_gain=0.5, want_ln_out=True)
    assert_close_rel(y, y_ref, what="layernorm out")
    assert_spikes_match(s.reshape(T, -1), s_ref.reshape(T, -1), vh, 1.0, what="spikes")


def test_linear_ln_lif_residual_and_tbcast(ops):
    T, R, K, N = 4, 200, 256, 384
    A, W, bias, gamma, beta_ln = make_lin(5, R, K, N, T, t_broadcast=True)
    s_ref, y_ref, vh = ref_linear_ln_lif(A, W, bias, gamma, beta_ln, T, 0.9, 1.0, 0.0, t_broadcast=True)
    resid = torch.randint(0, 5, (T * R, N)).to(torch.bfloat16)
    r_dev = resid.to(DEV)
    s, y = ops.linear_ln_lif(A.to(DEV), W.to(DEV), bias.to(DEV), gamma.to(DEV), beta_ln.to(DEV), 1e-5, 0.9, 1.0,
                             0.0, T, t_broadcast=True, residual=r_dev, want_ln_out=True)
    assert_close_rel(y, y_ref, what="layernorm out")
    assert_spikes_match(s.reshape(T, -1), s_ref.reshape(T, -1), vh, 1.0, what="spikes")
    assert torch.equal(r_dev.float().cpu(), resid.float() + s.float().cpu())


def test_linear_plain(ops):
    # N % 4 == 0 takes the staged 16-byte stores, the others the per-row stores
    for M, K, N in [(300, 384, 256), (77, 64, 40), (1000, 128, 600), (129, 64, 37), (260, 96, 258)]:
        g = gen(M + N)
        A = torch.randint(0, 4, (M, K), generator=g).to(torch.bfloat16)
        W = torch.randn(N, K, generator=g).to(torch.bfloat16)
        b = torch.randn(N, generator=g)
        out = ops.linear(A.to(DEV), W.to(DEV), b.to(DEV))
        ref = A.float() @ W.float().t() + b
        assert torch.allclose(out.cpu(), ref, rtol=1e-5, atol=1e-4)


@pytest.mark.parametrize("M,N,K", [
    (65536, 384, 384),     # q/k/v, out_proj at 64 images (T = 4)
    (4096, 1152, 384),     # the stacked Q/K/V projection
    (2048, 1536, 384),     # MLP expand
    (3000, 384, 1536),     # MLP compress, rows not a multiple of 128
    (77, 32, 40),          # small model: partial tiles in every dimension
    (129, 96, 200),
])
def test_linear_training_gradients(ops, M, N, K):
    """Input and weight gradients of a bias-free Linear from bf16 operands
    against the fp64 products of the same bf16 values: within 1e-5 of the
    largest element (fp32 accumulation)."""
    g = gen(M + N + K)
    G = torch.randn(M, N, generator=g).to(torch.bfloat16)
    W = (torch.randn(N, K, generator=g) * 0.05).to(torch.bfloat16)
    X = (torch.rand(M, K, generator=g) < 0.2).to(torch.bfloat16)
    dx = ops.linear_dgrad(G.to(DEV), W.to(DEV)).cpu()
    dw = ops.linear_wgrad(G.to(DEV), X.to(DEV)).cpu()
    dx_ref = G.double() @ W.double()
    dw_ref = G.double().t() @ X.double()
    assert dx.dtype == torch.float32 and dx.shape == (M, K) and dw.shape == (N, K)
    assert (dx.double() - dx_ref).abs().max() <= 1e-5 * dx_ref.abs().max()
    assert (dw.double() - dw_ref).abs().max() <= 1e-5 * dw_ref.abs().max()
    # the same call twice gives the same bits (fixed-order split sums)
    assert torch.equal(ops.linear_wgrad(G.to(DEV), X.to(DEV)).cpu(), dw)


@pytest.mark.parametrize("B,C,H,W,p", [(3, 1, 32, 64, 16), (2, 3, 12, 18, 6), (2, 2, 8, 24, 4)])
def test_patch_im2col_matches_unfold(ops, B, C, H, W, p):
    """Patch rows [hi | lo] in bf16 against torch's unfold of the same image
    (vector kernel for p % 4 == 0 and W % 4 == 0, scalar kernel otherwise)."""
    g = gen(B * 100 + p)
    img = torch.rand(B, C, H, W, generator=g)
    a = ops.patch_im2col(img.to(DEV), p).cpu()
    ref = F.unfold(img, p, stride=p).transpose(1, 2).reshape(-1, C * p * p)
    hi = ref.to(torch.bfloat16)
    lo = (ref - hi.float()).to(torch.bfloat16)
    assert torch.equal(a, torch.cat([hi, lo], dim=1))


@pytest.mark.parametrize("B,N,d,dtype", [(2048, 256, 48, torch.bfloat16), (37, 19, 8, torch.bfloat16),
                                         (5, 300, 4, torch.float32), (3, 1, 64, torch.uint8)])
def test_xnor_n_major_matches_permute(ops, B, N, d, dtype):
    """The n-major copy of V ([B, N, d] -> [N, B*d]) equals torch's permute
    bit for bit; rows that are not a multiple of 16 bytes are refused."""
    g = gen(B + N + d)
    x = (torch.rand(B, N, d, generator=g) * 200).to(dtype)
    out = ops.xnor_train_n_major(x.to(DEV)).cpu()
    assert torch.equal(out, x.permute(1, 0, 2).reshape(N, B * d))
    with pytest.raises(ValueError):
        ops.xnor_train_n_major(torch.zeros(2, 3, 5, dtype=torch.bfloat16, device=DEV))


def test_patch_embed_split(ops):
    g = gen(3)
    img = torch.rand(3, 1, 32, 64, generator=g)
    Wc = (torch.randn(64, 1, 16, 16, generator=g) * 0.05).to(torch.bfloat16).float()
    a = ops.patch_im2col(img.to(DEV), 16)
    W2 = torch.cat([Wc.reshape(64, -1), Wc.reshape(64, -1)], 1).to(torch.bfloat16)
    out = ops.linear(a, W2.to(DEV))
    ref = F.conv2d(img, Wc, stride=16).flatten(2).transpose(1, 2).reshape(-1, 64)
    assert torch.allclose(out.cpu(), ref, rtol=2e-5, atol=2e-5)


# ------------------------------------------------------------------ convolution patches, affine -> LIF


@pytest.mark.parametrize("N,H,W,C,k,s,pd,dtype", [
    (3, 8, 20, 64, (3, 3), (1, 1), (1, 1), torch.bfloat16),   # bottleneck 3x3 (16-byte chunks)
    (2, 32, 40, 1, (12, 12), (4, 4), (4, 4), torch.float32),  # PixelUnshuffle(4) + 3x3 on the image, split
    (4, 8, 9, 64, (8, 1), (1, 1), (0, 0), torch.bfloat16),    # the (channel, height) fold of the reduce block
    (5, 1, 33, 32, (1, 3), (1, 1), (0, 1), torch.bfloat16),   # Conv1d k=3 of the position encoding
    (2, 5, 7, 3, (3, 2), (2, 1), (1, 0), torch.bfloat16),     # odd channels: per-element path
])
def test_im2col_matches_unfold(ops, N, H, W, C, k, s, pd, dtype):
    g = gen(N * H + C)
    x = (torch.rand(N, C, H, W, generator=g) * 3).floor() if dtype == torch.bfloat16 else \
        torch.rand(N, C, H, W, generator=g)
    out = ops.im2col(x.permute(0, 2, 3, 1).to(dtype).to(DEV), k, s, pd).cpu()
    cols = F.unfold(x, k, padding=pd, stride=s)                          # [N, C*kh*kw, L], (c, i, j)
    L = cols.shape[-1]
    ref = cols.view(N, C, k[0] * k[1], L).permute(0, 3, 2, 1).reshape(N * L, -1)  # (i, j, c) columns
    if dtype == torch.float32:
        hi = ref.to(torch.bfloat16)
        ref = torch.cat([hi, (ref - hi.float()).to(torch.bfloat16)], dim=1)
    assert torch.equal(out, ref.to(torch.bfloat16))


@pytest.mark.parametrize("T,R,K,N,tb,res", [
    (4, 300, 576, 512, False, False),   # bottleneck 3x3 64 -> 512 (2-CTA cluster, no statistics exchange)
    (4, 200, 512, 64, False, True),     # bottleneck 1x1 512 -> 64 + identity
    (4, 150, 288, 128, True, False),    # first convolution, once per image, LIF at every step
    (3, 77, 96, 32, False, True),
])
def test_linear_affine_lif(ops, T, R, K, N, tb, res):
    g = gen(T * R + K + N)
    rows = R if tb else T * R
    A = (torch.rand(rows, K, generator=g) < 0.3).to(torch.bfloat16)
    W = (torch.randn(N, K, generator=g) / K ** 0.5).to(torch.bfloat16)
    bias = 0.1 * torch.randn(N, generator=g)
    scale = 1.0 + 0.3 * torch.randn(N, generator=g)
    shift = 0.2 * torch.randn(N, generator=g) + 0.5
    pre = (A.float() @ W.float().t() + bias) * scale + shift
    y3 = pre.unsqueeze(0).expand(T, *pre.shape).reshape(T, -1) if tb else pre.reshape(T, -1)
    s_ref, _ = oracle.lif_forward(y3, 0.5, 1.0, 0.0)
    vh = membrane_history(y3, 0.5, 1.0, 0.0)
    resid = torch.randint(0, 3, (T * R, N), generator=g).to(torch.bfloat16) if res else None
    r_dev = resid.to(DEV) if res else None
    s = ops.linear_affine_lif(A.to(DEV), W.to(DEV), bias.to(DEV), scale.to(DEV), shift.to(DEV), 0.5, 1.0, 0.0, T,
                              t_broadcast=tb, residual=r_dev, want_spikes=not res)
    if res:
        assert s is None
        s = r_dev.float().cpu() - resid.float()
    assert_spikes_match(s.float().cpu().reshape(T, -1), s_ref, vh, 1.0, what="affine lif spikes")


# ------------------------------------------------------------------ SSA


def ref_ssa(q, k, v, T, H, variant, scale, mask, vth=0.5, beta=0.9, gain=1.0):
    """q,k,v [T*B, N, D] float spikes -> (spikes, attn, exact integer O)."""
    TB, Nq, D = q.shape
    Nk = k.shape[1]
    dh = D // H
    qh = q.view(TB, Nq, H, dh).transpose(1, 2)
    kh = k.view(TB, Nk, H, dh).transpose(1, 2)
    vh = v.view(TB, Nk, H, dh).transpose(1, 2)
    if variant == 1:
        m = om.SSAMultiHeadAttention(D, H, n_steps=T)
        with torch.no_grad():
            m.scale.fill_(scale)
            attn = m.attention(qh, kh, vh, mask)
        s_int = om.SSAMultiHeadAttention.xnor_scores(qh.double(), kh.double()) + \
            om.log_pe_bias(Nq, Nk).double()
    else:
        attn = om.SSAMultiHeadAttention_.attention(None, qh, kh, vh, mask)
        s_int = qh.double() @ kh.double().transpose(-2, -1)
    if mask is not None:
        s_int = s_int * mask.double()
    o_int = s_int @ vh.double()
    x3 = attn.reshape(T, -1)
    s, _ = oracle.lif_forward(x3, beta, vth, 0.0, in_gain=gain)
    vhist = membrane_history(x3, beta, vth, 0.0, gain)
    spikes = s.reshape(TB, H, Nq, dh).transpose(1, 2).reshape(TB, Nq, D)
    return spikes, attn, o_int, vhist


def spikes_qkv(seed, TB, Nq, Nk, D, p=0.15):
    g = gen(seed)
    q = (torch.rand(TB, Nq, D, generator=g) < p).float()
    k = (torch.rand(TB, Nk, D, generator=g) < p).float()
    v = (torch.rand(TB, Nk, D, generator=g) < p).float()
    return q, k, v


@pytest.mark.parametrize("variant", [0, 1])
@pytest.mark.parametrize("T,B,H,Nq,Nk,dh,maskkind", [
    (2, 2, 4, 12, 12, 8, None),
    (2, 3, 2, 40, 40, 48, "causal"),
    (4, 2, 8, 256, 256, 48, None),     # encoder shape (two key blocks)
    (4, 2, 8, 64, 64, 48, "causal"),   # decoder self-attention
    (4, 2, 8, 64, 256, 48, None),      # decoder cross-attention
    (2, 3, 2, 200, 130, 64, None),     # two query blocks, the second partial; head width 64
    (1, 2, 3, 300, 40, 16, None),      # more than two query blocks (dense kernel)
    (2, 2, 2, 130, 70, 64, "dense"),
    (1, 1, 1, 200, 300, 16, "dense"),
    # short sequences (two (batch, head) pairs per tile): odd pair count,
    # Nq != Nk, keys < 32, head width 8 / 16 / 32
    (3, 5, 3, 33, 50, 32, "dense"),
    (2, 3, 3, 64, 20, 16, "dense"),
    (2, 2, 4, 12, 12, 8, "causal"),
    (2, 3, 2, 48, 48, 64, "causal"),  # head width 64: the slots' V tiles fill both atoms of P V
    (1, 3, 1, 64, 64, 64, "dense"),
])
def test_ssa(ops, variant, T, B, H, Nq, Nk, dh, maskkind):
    D = H * dh
    q, k, v = spikes_qkv(Nq * 31 + Nk + dh + variant, T * B, Nq, Nk, D, p=0.2 if variant == 0 else 0.15)
    scale = 0.125 if variant == 0 else (1.0 / dh) ** 0.5
    mask = None
    if maskkind == "causal":
        mask = torch.tril(torch.ones(Nq, Nk)).expand(T * B, 1, Nq, Nk)
    elif maskkind == "dense":
        mask = (torch.rand(T * B, 1, Nq, Nk, generator=gen(9)) < 0.7).float()
    s_ref, attn_ref, o_int, vhist = ref_ssa(q, k, v, T, H, variant, scale, mask)
    s, attn = ops.ssa(q.to(DEV).bfloat16(), k.to(DEV).bfloat16(), v.to(DEV).bfloat16(), T, B, H, variant, scale,
                      0.9, 0.5, 0.0, mask=None if maskkind == "causal" else (mask.to(DEV) if mask is not None else None),
                      causal=maskkind == "causal", out_dtype=torch.float32, want_attn=True)
    # spike-count products: a = fl(scale * O) with O the exact integer product
    expect = (o_int.float() * torch.tensor(scale, dtype=torch.float32))
    assert torch.equal(attn.cpu(), expect), "attention products differ from the exact integer product"
    assert_close_rel(attn, attn_ref, tol=1e-5, what="attention vs reference rounding")
    s_ours = s.cpu().reshape(T * B, Nq, H, dh).transpose(1, 2).reshape(T, -1)
    s_want = s_ref.reshape(T * B, Nq, H, dh).transpose(1, 2).reshape(T, -1)
    if variant == 0:
        # plain: a = 0.125 * integer is computed exactly on both sides, so the
        # spike trains must agree bit for bit (values sit exactly on v_th often)
        assert torch.equal(s_ours, s_want)
    else:
        assert_spikes_match(s_ours, s_want, vhist.reshape(T, -1), 0.5, what="ssa spikes")


# ------------------------------------------------------------------ embedding


@pytest.mark.parametrize("variant", [0, 1])
@pytest.mark.parametrize("T,B,H,Nq,Nk,dh", [(4, 2, 8, 256, 256, 48), (4, 3, 2, 64, 256, 48), (2, 2, 3, 40, 70, 64)])
def test_ssa_heads_equals_token_major(ops, variant, T, B, H, Nq, Nk, dh):
    """The head-split entry point (operands as strided [T*B, H, N, dh] views,
    the layout of the training forward) gives the token-major entry point's
    spikes and LIF input bit for bit."""
    D = H * dh
    q, k, v = spikes_qkv(Nq * 13 + Nk + dh + variant, T * B, Nq, Nk, D, p=0.15)
    q, k, v = (t.to(DEV).bfloat16() for t in (q, k, v))
    scale = 0.125 if variant == 0 else (1.0 / dh) ** 0.5
    s_ref, a_ref = ops.ssa(q, k, v, T, B, H, variant, scale, 0.9, 0.5, 0.0, in_gain=0.5, want_attn=True)
    heads = [t.view(T * B, t.shape[1], H, dh).transpose(1, 2) for t in (q, k, v)]  # strided views
    s, a = ops.ssa_heads(*heads, T, variant, scale, 0.9, 0.5, 0.0, in_gain=0.5, want_attn=True)
    assert torch.equal(s, s_ref)
    assert torch.equal(a, a_ref.transpose(1, 2).reshape(T * B, Nq, D))


def test_embed_pe_lif(ops):
    g = gen(4)
    V, D, B, N, T = 50, 32, 3, 7, 4
    pe_mod = om.PositionalEncoding(D, 0.0, maxlen=64)
    emb = torch.randn(V, D, generator=g).to(torch.bfloat16).float()
    tok = torch.randint(0, V, (B, N), generator=g)
    x = emb[tok] * (D ** 0.5) + pe_mod.pos_embedding[:, :N]
    x3 = x.unsqueeze(0).expand(T, B, N, D).reshape(T, -1)
    s_ref, _ = oracle.lif_forward(x3, 0.9, 1.0, 0.0)
    s, bad = ops.embed_pe_lif(tok.to(DEV), emb.to(DEV), D ** 0.5, pe_mod.pos_embedding.to(DEV), 0.9, 1.0, 0.0, T,
                              out_dtype=torch.float32)
    assert int(bad.item()) == 0
    assert torch.equal(s.cpu().reshape(T, -1), s_ref)
    _, bad = ops.embed_pe_lif((tok + V).to(DEV), emb.to(DEV), D ** 0.5, pe_mod.pos_embedding.to(DEV), 0.9, 1.0, 0.0,
                              T)
    assert int(bad.item()) == 1


def test_no_device_timeouts(ops):
    ops.device_error_check()


def test_bounded_wait_gives_up_and_reports_timeout(ops):
    """A device-side wait that nothing satisfies ends after its limit (50 ms
    here instead of the kernels' 2 s): the kernel returns, the context stays
    usable, and the host sees SPK_ERR_TIMEOUT once, after which the flag is
    clear."""
    from spikingtransformer_b200 import _lib
    lib = _lib.load()
    ops.device_error_check()
    st = _lib.stream_ptr(torch.device(DEV))
    assert lib.spk_test_bounded_wait(50_000_000, st) == 0
    with pytest.raises(RuntimeError, match="timed out"):
        ops.device_error_check()
    ops.device_error_check()  # cleared
    x = torch.ones(2, 8, device=DEV)
    s, _ = ops.lif_fwd(x, 0.5, 0.75, 0.0)  # the device still runs work: v = 1 > 0.75 fires at both steps
    assert s.sum().item() == 16.0
    assert lib.spk_test_bounded_wait(0, st) == 1  # SPK_ERR_INVALID


# ------------------------------------------------------------------ LayerNorm -> LIF (training)


@pytest.mark.parametrize("T,R,D,pre_dtype,surrogate,gain", [
    (4, 64, 384, torch.float32, "superspike", 1.0),
    (4, 48, 384, torch.bfloat16, "arctan", 0.5),
    (4, 8, 1536, torch.bfloat16, "arctan", 1.0),    # four warps per token
    (2, 50, 64, torch.float32, "superspike", 0.7),
    (3, 17, 96, torch.float32, "arctan", 1.0),
    (1, 5, 512, torch.float32, "superspike", 1.0),
    (2, 9, 1536, torch.float32, "superspike", 1.0),
    (4, 30, 256, torch.float16, "arctan", 1.0),
    (4, 12, 768, torch.bfloat16, "superspike", 1.0),  # two warps per token
    (1, 7, 768, torch.float32, "arctan", 0.5),
    (3, 10, 384, torch.bfloat16, "superspike", 1.0),
    (4, 301, 384, torch.bfloat16, "arctan", 1.0),     # several tokens per warp
])
def test_ln_lif_train_fwd_bwd(ops, T, R, D, pre_dtype, surrogate, gain):
    g = gen(T * 100 + R + D)
    pre = (torch.randn(T * R, D, generator=g) * 1.5 + 0.3).to(pre_dtype)
    gamma = (1.0 + 0.2 * torch.randn(D, generator=g))
    beta_ln = 0.3 * torch.randn(D, generator=g)
    lif_beta = torch.tensor(0.8)
    k = 2.0 if surrogate == "arctan" else 4.0
    gs = torch.randn(T * R, D, generator=g)
    # the Linear's bias handed to the kernels on every other case
    bias = 0.2 * torch.randn(D, generator=g) if R % 2 == 0 else None
    # reference: torch LayerNorm (fp32) composed with the oracle's autograd LIF
    x = pre.float().clone().requires_grad_(True)
    w = gamma.clone().requires_grad_(True)
    b = beta_ln.clone().requires_grad_(True)
    lb = lif_beta.clone().requires_grad_(True)
    pb = None if bias is None else bias.clone().requires_grad_(True)
    y = F.layer_norm(x if pb is None else x + pb, (D,), w, b, 1e-5)
    s_ref, _ = oracle.lif.LIFFunction.apply(y.view(T, R, D), lb, torch.tensor(1.0), torch.tensor(0.0), k, surrogate,
                                            gain)
    (s_ref * gs.view(T, R, D)).sum().backward()
    # ours
    bias_dev = None if bias is None else bias.to(DEV)
    s, stats = ops.ln_lif_fwd(pre.to(DEV), gamma.to(DEV), beta_ln.to(DEV), 1e-5, lif_beta, 1.0, 0.0, T,
                              in_gain=gain, bias=bias_dev)
    g_pre, g_w, g_b, g_lb, g_pb = ops.ln_lif_bwd(gs.to(DEV), pre.to(DEV), stats, gamma.to(DEV), beta_ln.to(DEV),
                                                 lif_beta, 1.0, 0.0, T, gain, surrogate, k, bias=bias_dev,
                                                 need_bias=bias is not None)
    vh = membrane_history(y.detach().view(T, -1), lif_beta, 1.0, 0.0, gain)
    assert_spikes_match(s.cpu().view(T, -1), s_ref.detach().view(T, -1), vh, 1.0, what="ln_lif spikes")
    mean = (x.detach() if bias is None else x.detach() + bias).mean(-1)
    assert torch.allclose(stats[:, 0].cpu(), mean, rtol=1e-4, atol=1e-5)
    # gradients on the rows whose spike train matches (a flipped near-threshold spike changes the
    # backward of its token)
    same = (s.cpu().view(T, R, D) == s_ref.detach().view(T, R, D)).all(dim=0).all(dim=-1)  # [R]
    assert same.float().mean() > 0.9
    rows = same.repeat(T)
    tol = 2e-2 if pre_dtype == torch.bfloat16 else 2e-3
    gp, gp_ref = g_pre.float().cpu()[rows], x.grad[rows]
    assert_close_rel(gp, gp_ref, tol=tol, what="g_pre")
    if bool(same.all()):
        assert_close_rel(g_w.cpu(), w.grad, tol=tol, what="g_gamma")
        assert_close_rel(g_b.cpu(), b.grad, tol=tol, what="g_beta")
        assert abs(g_lb.item() - lb.grad.item()) <= tol * max(1.0, abs(lb.grad.item()))
        if bias is not None:
            assert_close_rel(g_pb.cpu(), pb.grad, tol=tol, what="g_bias")


@pytest.mark.parametrize("pre_dtype,gs_dtype", [(torch.bfloat16, torch.bfloat16), (torch.float32, torch.float32)])
def test_ln_lif_train_head_major_spikes(ops, pre_dtype, gs_dtype):
    """Spikes written per head, [T*B, H, N, dh] (the layout the attention reads),
    and their gradient read in that layout, equal the row-major results
    transposed."""
    g = gen(21)
    T, B, N, H, dh = 4, 3, 20, 8, 48
    D = H * dh
    pre = (torch.randn(T * B * N, D, generator=g) * 1.3 + 0.2).to(pre_dtype).to(DEV)
    bias = (0.1 * torch.randn(D, generator=g)).to(DEV)
    gamma = (1.0 + 0.2 * torch.randn(D, generator=g)).to(DEV)
    s_rm, st_rm = ops.ln_lif_fwd(pre, gamma, None, 1e-5, 0.8, 1.0, 0.0, T, bias=bias, spike_dtype=torch.bfloat16)
    s_hm, st_hm = ops.ln_lif_fwd(pre, gamma, None, 1e-5, 0.8, 1.0, 0.0, T, bias=bias, spike_dtype=torch.bfloat16,
                                 heads=(dh, N))
    assert s_hm.shape == (T * B, H, N, dh) and s_hm.is_contiguous()
    assert torch.equal(s_hm, s_rm.view(T * B, N, H, dh).transpose(1, 2))
    assert torch.equal(st_hm, st_rm)
    gs_hm = torch.randn(T * B, H, N, dh, generator=g).to(gs_dtype).to(DEV)
    gs_rm = gs_hm.transpose(1, 2).reshape(T * B * N, D).contiguous()
    a = ops.ln_lif_bwd(gs_rm, pre, st_rm, gamma, None, 0.8, 1.0, 0.0, T, 1.0, "arctan", 2.0, need_beta=False,
                       bias=bias, need_bias=True)
    b = ops.ln_lif_bwd(gs_hm, pre, st_hm, gamma, None, 0.8, 1.0, 0.0, T, 1.0, "arctan", 2.0, need_beta=False,
                       bias=bias, need_bias=True, heads=(dh, N))
    for x, y in zip(a, b):
        assert (x is None and y is None) or torch.equal(x, y)


@pytest.mark.parametrize("D", [384, 1536])
def test_ln_lif_train_bf16_gradient_equals_fp32_path(ops, D):
    """A bf16 spike gradient gives the same results as the same values in fp32
    (the kernels widen every input to fp32 before any arithmetic)."""
    g = gen(D + 5)
    T, R = 4, 700
    pre = (torch.randn(T * R, D, generator=g) * 1.4).to(torch.bfloat16).to(DEV)
    gamma = (1.0 + 0.2 * torch.randn(D, generator=g)).to(DEV)
    beta_ln = (0.3 * torch.randn(D, generator=g)).to(DEV)
    bias = (0.1 * torch.randn(D, generator=g)).to(DEV)
    _, stats = ops.ln_lif_fwd(pre, gamma, beta_ln, 1e-5, 0.8, 1.0, 0.0, T, bias=bias, spike_dtype=torch.bfloat16)
    gs16 = torch.randn(T * R, D, generator=g).to(torch.bfloat16).to(DEV)
    a = ops.ln_lif_bwd(gs16, pre, stats, gamma, beta_ln, 0.8, 1.0, 0.0, T, 1.0, "arctan", 2.0, bias=bias,
                       need_bias=True)
    b = ops.ln_lif_bwd(gs16.float(), pre, stats, gamma, beta_ln, 0.8, 1.0, 0.0, T, 1.0, "arctan", 2.0, bias=bias,
                       need_bias=True)
    for x, y in zip(a, b):
        assert torch.equal(x, y)


@pytest.mark.parametrize("D,pre_dtype", [(384, torch.bfloat16), (1536, torch.bfloat16), (384, torch.float32)])
def test_ln_lif_fwd_residual_equals_spikes_plus_residual(ops, D, pre_dtype):
    """The residual form writes residual + the spikes of ln_lif_fwd, bit for
    bit, with the same row statistics, and its bf16 copy equals the output
    cast to bf16."""
    g = gen(D + 77)
    T, R = 4, 900
    pre = (torch.randn(T * R, D, generator=g) * 1.3).to(pre_dtype).to(DEV)
    gamma = (1.0 + 0.2 * torch.randn(D, generator=g)).to(DEV)
    beta_ln = (0.3 * torch.randn(D, generator=g)).to(DEV)
    bias = (0.1 * torch.randn(D, generator=g)).to(DEV)
    resid = torch.randint(0, 9, (T * R, D), generator=g).float().to(DEV)
    s, st = ops.ln_lif_fwd(pre, gamma, beta_ln, 1e-5, 0.8, 1.0, 0.0, T, in_gain=0.5, bias=bias)
    assert ops.ln_lif_residual_ok(pre, resid)
    out, st2, outb = ops.ln_lif_fwd_residual(pre, gamma, beta_ln, 1e-5, 0.8, 1.0, 0.0, T, resid, in_gain=0.5,
                                             bias=bias, want_bf16=True)
    assert torch.equal(out, resid + s)
    assert torch.equal(st2, st)
    assert torch.equal(outb, out.to(torch.bfloat16))
    out2, _, none = ops.ln_lif_fwd_residual(pre, gamma, beta_ln, 1e-5, 0.8, 1.0, 0.0, T, resid, in_gain=0.5,
                                            bias=bias)
    assert none is None and torch.equal(out2, out)


def test_ln_lif_train_unaligned_inputs(ops):
    """The vectorised one-token-per-block kernels need 16-byte aligned rows:
    an input offset by one element takes the scalar kernels (D <= 512) with the
    same results, or is rejected (D > 512)."""
    g = gen(11)
    T, R, D = 4, 6, 384
    flat = torch.randn(T * R * D + 1, generator=g).to(DEV)
    pre_off = flat[1:].view(T * R, D)            # 4-byte offset
    pre_al = pre_off.clone()
    bias = (0.1 * torch.randn(D, generator=g)).to(DEV)
    s1, st1 = ops.ln_lif_fwd(pre_off, None, None, 1e-5, 0.8, 1.0, 0.0, T, bias=bias)
    s2, st2 = ops.ln_lif_fwd(pre_al, None, None, 1e-5, 0.8, 1.0, 0.0, T, bias=bias)
    assert torch.equal(s1, s2)
    assert torch.allclose(st1, st2, rtol=1e-6, atol=1e-6)
    wide = torch.randn(T * 2 * 1536 + 1, generator=g).to(DEV)[1:].view(T * 2, 1536)
    with pytest.raises(RuntimeError):
        ops.ln_lif_fwd(wide, None, None, 1e-5, 0.8, 1.0, 0.0, T)


def test_ln_lif_train_rejects_unsupported(ops):
    with pytest.raises(RuntimeError):
        ops.ln_lif_fwd(torch.zeros(5 * 4, 96, device=DEV), None, None, 1e-5, 0.5, 1.0, 0.0, 5)  # T > 4
    with pytest.raises(RuntimeError):
        ops.ln_lif_fwd(torch.zeros(4 * 4, 100, device=DEV), None, None, 1e-5, 0.5, 1.0, 0.0, 4)  # D % 32
