"""Module-level parity of the Triton_Layers-compatible surface on the GPU:
against the golden fixtures (made by running the reference) and the CPU
oracle, including the full OCR benchmark architecture at a small batch."""

import math
import os

import pytest
import torch

from oracle import modules as om
from parity import assert_spikes_match, assert_close_rel, membrane_history, spike_mismatch_rate

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def pkg():
    import spikingtransformer_b200 as p
    p.install_as_triton_layers()
    return p


def load(golden_dir, name):
    return torch.load(os.path.join(golden_dir, name), weights_only=False)


def test_lif_module_golden(pkg, golden_dir):
    from spikingtransformer_b200.Lif import LIF
    for c in load(golden_dir, "lif_module.pt"):
        m = LIF(beta=0.8, v_th=0.9, n_steps=3, learn_beta=c["learn_beta"]).to(DEV)
        m.load_state_dict(c["state"])
        with torch.no_grad():
            s, vf = m(c["x"].to(DEV))
        assert torch.equal(s.cpu(), c["spikes"])
        assert torch.equal(vf.cpu(), c["v_final"])


def test_lif_layer_autograd_golden(pkg, golden_dir):
    from spikingtransformer_b200.Lif import LIFLayer
    for c in load(golden_dir, "lif.pt"):
        x = c["x_in"].to(DEV).requires_grad_(True)
        b = torch.tensor(c["beta"], device=DEV, requires_grad=True)
        s, vf = LIFLayer.apply(x, b, torch.tensor(c["v_th"], device=DEV), torch.tensor(c["v_reset"], device=DEV), 4.0)
        (s * c["g_spikes"].to(DEV)).sum().backward()
        assert torch.equal(x.grad.cpu(), c["grad_x"].to(x.dtype))
        assert torch.allclose(b.grad.cpu(), c["grad_beta"], rtol=1e-5, atol=1e-5)


def test_triton_layers_alias(pkg):
    import Triton_Layers.Seq2Seq as S
    import spikingtransformer_b200.Seq2Seq as T
    assert S is T


def _ssa_cls(c):
    from spikingtransformer_b200.SSA import SSAMultiHeadAttention, SSAMultiHeadAttention_
    return SSAMultiHeadAttention if c["variant"] == "xnor" else SSAMultiHeadAttention_


@pytest.mark.parametrize("path", ["fused", "autograd"])
def test_ssa_golden(pkg, golden_dir, path):
    for c in load(golden_dir, "ssa.pt"):
        m = _ssa_cls(c)(d_model=c["D"], n_heads=c["H"], n_steps=c["T"]).to(DEV)
        m.load_state_dict(c["state"])
        q, k = c["query"].to(DEV), c["key"].to(DEV)
        mask = None if c["mask"] is None else c["mask"].to(DEV)
        if path == "fused":
            with torch.no_grad():
                y = m(q, k, k, attention_mask=mask)
        else:
            y = m(q, k, k, attention_mask=mask)
        T = c["T"]
        vh = membrane_history(c["ln_o"].reshape(T, -1), 0.9, 1.0, 0.0)
        assert_spikes_match(y.reshape(T, -1), c["out"].reshape(T, -1), vh, 1.0,
                            what=f"ssa {c['variant']} {c['case']} {path}")


@pytest.mark.parametrize("Nq,Nk,dtype", [(40, 70, torch.float32), (64, 256, torch.bfloat16), (33, 5, torch.float32)])
def test_xnor_score_free_training_core(pkg, Nq, Nk, dtype):
    """The tensor-core autograd core of the unmasked XNOR attention against the
    dense reference formula (``SSA.py:145-165``, ``:235-240``) in float64:
    forward bit for bit, gradients of Q, K, V and the scale within 1e-4 of
    the largest gradient (split-bf16 products)."""
    from spikingtransformer_b200.SSA import SSAMultiHeadAttention, XnorScoreFree
    TB, H, dh = 6, 3, 48
    m = SSAMultiHeadAttention(d_model=H * dh, n_heads=H).to(DEV)
    g = torch.Generator(device=DEV).manual_seed(Nq + Nk)
    leaves = [(torch.rand(TB, n, H, dh, generator=g, device=DEV) < 0.3).to(dtype).requires_grad_()
              for n in (Nq, Nk, Nk)]
    q, k, v = (t.transpose(1, 2) for t in leaves)
    R = m.get_log_pe_bias_cross(Nq, Nk, DEV)
    out = XnorScoreFree.apply(q, k, v, R, m.scale)
    w = torch.randn(out.shape, generator=g, device=DEV)
    (out * w).sum().backward()

    ref_leaves = [t.detach().double().requires_grad_() for t in leaves]
    rq, rk, rv = (t.transpose(1, 2) for t in ref_leaves)
    rs = m.scale.detach().double().requires_grad_()
    S = dh - (rq.sum(-1, keepdim=True) + rk.sum(-1, keepdim=True).transpose(2, 3) - 2 * rq @ rk.transpose(2, 3))
    ref = (((S + R.double()) * rs) @ rv).transpose(1, 2).reshape(TB, Nq, H * dh)  # token-major, as ours
    (ref * w.double()).sum().backward()
    assert out.dtype == torch.float32 and torch.equal(out, ref.float())
    for name, a, b in (("q", leaves[0].grad, ref_leaves[0].grad), ("k", leaves[1].grad, ref_leaves[1].grad),
                       ("v", leaves[2].grad, ref_leaves[2].grad)):
        assert a.dtype == dtype
        err = (a.double() - b).abs().max().item()
        tol = 1e-4 if dtype == torch.float32 else 1e-2  # bf16 gradients carry 8 bits
        assert err <= tol * b.abs().max().item(), (name, err, b.abs().max().item())
    gs_bound = (w.double().abs() * ref.detach().abs()).sum().item() / abs(rs.item())
    assert abs(m.scale.grad.item() - rs.grad.item()) <= 1e-5 * gs_bound


@pytest.mark.parametrize("variant,Nq,Nk,dtype,maskkind", [
    (1, 64, 64, torch.float32, "causal+pad"),   # the decoder's masked self-attention
    (1, 64, 64, torch.bfloat16, "causal"),
    (1, 17, 40, torch.float32, "dense"),
    (0, 64, 64, torch.float32, "causal"),       # plain form (SSAMultiHeadAttention_)
    (0, 33, 20, torch.bfloat16, None),
])
def test_masked_short_attention_training_core(pkg, variant, Nq, Nk, dtype, maskkind):
    """The masked attention core of the training path (one kernel each way,
    score matrix in shared memory) against the reference formula
    (``SSA.py:234-242``; plain ``SSA.py:81-84``) differentiated in float64:
    the forward bit for bit (integer S, P V, one scale multiply), gradients of
    Q, K, V and the scale within 1e-5 of the largest element (1e-2 in bf16)."""
    from spikingtransformer_b200.SSA import MaskedShortAttention
    T, Bp, H, dh = 4, 3, 2, 48
    TB = T * Bp
    g = torch.Generator(device=DEV).manual_seed(Nq * 7 + Nk + variant)
    leaves = [(torch.rand(TB, n, H, dh, generator=g, device=DEV) < 0.3).to(dtype).requires_grad_()
              for n in (Nq, Nk, Nk)]
    q, k, v = (t.transpose(1, 2) for t in leaves)
    mask = None
    if maskkind is not None:
        if maskkind.startswith("causal"):
            m = torch.tril(torch.ones(Nq, Nk, device=DEV)).expand(Bp, 1, Nq, Nk).clone()
            if maskkind.endswith("pad"):
                m[0, :, :, 50:] = 0.0  # padded keys of image 0
        else:
            m = (torch.rand(Bp, 1, Nq, Nk, generator=g, device=DEV) < 0.7).float()
        mask = m.unsqueeze(0).repeat(T, 1, 1, 1, 1).reshape(TB, 1, Nq, Nk)  # the reference's T-fold
    scale = torch.tensor((1.0 / dh) ** 0.5 if variant == 1 else 0.125, device=DEV, requires_grad=variant == 1)
    out = MaskedShortAttention.apply(q, k, v, scale, mask, T, variant)
    w = torch.randn(out.shape, generator=g, device=DEV)
    (out * w).sum().backward()
    rl = [t.detach().double().requires_grad_() for t in leaves]
    rq, rk, rv = (t.transpose(1, 2) for t in rl)
    rs = scale.detach().double().requires_grad_()
    if variant == 1:
        iq = torch.arange(Nq, device=DEV).unsqueeze(1)
        jk = torch.arange(Nk, device=DEV).unsqueeze(0)
        R = torch.ceil(torch.log2((max(Nq, Nk) - 1) / ((iq - jk).abs().double() + 1))).clamp(min=0)
        S = dh - (rq.sum(-1, keepdim=True) + rk.sum(-1, keepdim=True).transpose(2, 3) - 2 * rq @ rk.transpose(2, 3))
        S = S + R
    else:
        S = rq @ rk.transpose(2, 3)
    if mask is not None:
        S = S * mask.double()
    ref = ((S @ rv) * rs).transpose(1, 2).reshape(TB, Nq, H * dh)
    (ref * w.double()).sum().backward()
    assert out.dtype == torch.float32 and torch.equal(out, ref.float())
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    for name, a, b in (("q", leaves[0].grad, rl[0].grad), ("k", leaves[1].grad, rl[1].grad),
                       ("v", leaves[2].grad, rl[2].grad)):
        assert a.dtype == dtype
        assert (a.double() - b).abs().max().item() <= tol * b.abs().max().item(), name
    if variant == 1:
        assert abs(scale.grad.item() - rs.grad.item()) <= 1e-5 * abs(rs.grad.item())


def test_decoder_masked_attention_trains_on_the_fused_core(pkg):
    """A decoder layer's masked self-attention under autograd runs the fused
    core kernels (no eager score matrix)."""
    from spikingtransformer_b200 import _lib
    from spikingtransformer_b200.Decoder import DecoderLayer
    T, B, N, D = 4, 2, 16, 64
    layer = DecoderLayer(D, 2, 128, n_steps=T).to(DEV)
    x = (torch.rand(T * B, N, D, device=DEV) < 0.3).float().requires_grad_()
    enc = (torch.rand(T * B, 24, D, device=DEV) < 0.3).float()
    mask = torch.tril(torch.ones(N, N, device=DEV)).expand(T * B, 1, N, N)
    with _lib.LaunchCounter() as counter:
        y = layer(x, enc, mask=mask)
        y.sum().backward()
    assert counter.counts.get("attn_masked_train_fwd") == 1, counter.counts
    assert counter.counts.get("attn_masked_train_bwd") == 1, counter.counts
    assert x.grad is not None and torch.isfinite(x.grad).all()


@pytest.mark.parametrize("in_dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("spike_dtype", [torch.float32, torch.bfloat16])
def test_xnor_lif_fused_equals_composition(pkg, spike_dtype, in_dtype):
    """The attention core with the output LIF fused into its kernels equals the
    core followed by the lifs LIF module: spikes bit for bit, gradients of Q,
    K, V and the scale to fp32 rounding.  With bf16 operands the forward runs
    the score-free inference kernel on the head-split views in place."""
    from spikingtransformer_b200.SSA import SSAMultiHeadAttention, XnorLIF, XnorScoreFree
    T, Bp, H, Nq, Nk, dh = 4, 3, 2, 24, 40, 48
    TB = T * Bp
    m = SSAMultiHeadAttention(d_model=H * dh, n_heads=H, n_steps=T).to(DEV)
    m.lifs.set_surrogate("arctan", 2.0)
    g = torch.Generator(device=DEV).manual_seed(17)
    base = [(torch.rand(TB, n, H, dh, generator=g, device=DEV) < 0.3).to(in_dtype) for n in (Nq, Nk, Nk)]
    R = m.get_log_pe_bias_cross(Nq, Nk, DEV)
    gsp = torch.randn(TB, Nq, H * dh, generator=g, device=DEV).to(torch.bfloat16).float()
    results = []
    for fused in (False, True):
        leaves = [t.clone().requires_grad_() for t in base]
        q, k, v = (t.transpose(1, 2) for t in leaves)
        m.scale.grad = None
        if fused:
            lifs = m.lifs
            s = XnorLIF.apply(q, k, v, R, m.scale, lifs.effective_beta(), lifs.v_th, lifs.v_reset, lifs.in_gain,
                              lifs.surrogate, lifs._k_host, T, spike_dtype)
            assert s.dtype == spike_dtype
        else:
            s = m.lifs(XnorScoreFree.apply(q, k, v, R, m.scale))[0]
        (s.float() * gsp).sum().backward()
        results.append((s.float(), [t.grad for t in leaves], m.scale.grad.clone()))
    (s0, g0, sc0), (s1, g1, sc1) = results
    assert torch.equal(s0, s1)
    for a, b in zip(g0, g1):
        assert torch.allclose(a.float(), b.float(), rtol=1e-5, atol=1e-6)
    assert torch.allclose(sc0, sc1, rtol=1e-4, atol=1e-6)


def test_fused_qkv_training_path_matches_separate(pkg, monkeypatch):
    """Self-attention under bf16 autocast with Q, K and V from one GEMM and one
    LayerNorm->LIF Function against the three separate projections: the same
    spikes (up to a GEMM rounding flip near threshold) and close gradients for
    every projection, LayerNorm and LIF parameter."""
    import spikingtransformer_b200.SSA as ssa_mod
    T, TB, N, D, H = 4, 8, 16, 256, 4
    g = torch.Generator(device=DEV).manual_seed(23)
    x = (torch.rand(TB, N, D, generator=g, device=DEV) < 0.3).float()
    base = ssa_mod.SSAMultiHeadAttention(d_model=D, n_heads=H, n_steps=T).to(DEV)
    base.lifq.set_surrogate("arctan", 2.0)
    w = torch.randn(TB, N, D, generator=g, device=DEV)
    runs = []
    for fused in (True, False):
        m = ssa_mod.SSAMultiHeadAttention(d_model=D, n_heads=H, n_steps=T).to(DEV)
        m.load_state_dict(base.state_dict())
        if not fused:
            monkeypatch.setattr(ssa_mod, "qkv_ln_lif_train", lambda *a, **k: None)
        xi = x.clone().requires_grad_()
        with torch.autocast("cuda", dtype=torch.bfloat16):
            y = m(xi)
        (y.float() * w).sum().backward()
        runs.append((y.float().detach(), xi.grad.clone(), {n: p.grad.clone() for n, p in m.named_parameters()
                                                           if p.grad is not None}))
    (y1, gx1, g1), (y2, gx2, g2) = runs
    assert (y1 != y2).float().mean().item() < 0.01
    assert set(g1) == set(g2)
    for n in g1:
        ref = g2[n].abs().max().item()
        assert (g1[n] - g2[n]).abs().max().item() <= 0.05 * ref + 1e-6, n
    assert (gx1 - gx2).abs().max().item() <= 0.05 * gx2.abs().max().item() + 1e-6


def test_residual_fusion_matches_composition(pkg, monkeypatch):
    """An encoder and a decoder layer trained under bf16 autocast with the
    residual adds fused into the LayerNorm->LIF kernels (and the next GEMM's
    bf16 copy written by them) against spikes plus separate adds: identical
    outputs (spike counts are exact either way) and the same gradients up to
    the order of fp32 gradient sums."""
    import spikingtransformer_b200._fused as fz
    from spikingtransformer_b200.Encoder import EncoderLayer
    from spikingtransformer_b200.Decoder import DecoderLayer
    T, B, N, M, D, H, F = 4, 3, 16, 8, 384, 8, 1536
    g = torch.Generator(device=DEV).manual_seed(41)
    x = (torch.rand(T * B, N, D, generator=g, device=DEV) < 0.2).float()
    y0 = (torch.rand(T * B, M, D, generator=g, device=DEV) < 0.2).float()
    w = torch.randn(T * B, M, D, generator=g, device=DEV)
    torch.manual_seed(3)
    enc0 = EncoderLayer(d_model=D, n_heads=H, ff_dim=F, n_steps=T).to(DEV)
    dec0 = DecoderLayer(d_model=D, n_heads=H, ff_dim=F, n_steps=T).to(DEV)
    runs = []
    for fused in (True, False):
        monkeypatch.setattr(fz, "RESIDUAL_FUSION", fused)
        enc = EncoderLayer(d_model=D, n_heads=H, ff_dim=F, n_steps=T).to(DEV)
        dec = DecoderLayer(d_model=D, n_heads=H, ff_dim=F, n_steps=T).to(DEV)
        enc.load_state_dict(enc0.state_dict())
        dec.load_state_dict(dec0.state_dict())
        xi, yi = x.clone().requires_grad_(), y0.clone().requires_grad_()
        with torch.autocast("cuda", dtype=torch.bfloat16):
            out = dec(yi, enc(xi))
        (out.float() * w).sum().backward()
        grads = {n: p.grad.clone() for m in (enc, dec) for n, p in m.named_parameters() if p.grad is not None}
        runs.append((out.detach().float(), xi.grad.clone(), yi.grad.clone(), grads))
    (o1, gx1, gy1, g1), (o2, gx2, gy2, g2) = runs
    assert torch.equal(o1, o2)
    assert set(g1) == set(g2)
    for n in g1:
        assert torch.allclose(g1[n], g2[n], rtol=1e-5, atol=1e-6 * (g2[n].abs().max().item() + 1.0)), n
    for a, b in ((gx1, gx2), (gy1, gy2)):
        assert torch.allclose(a, b, rtol=1e-5, atol=1e-6 * (b.abs().max().item() + 1.0))


def test_linear_bf16_training_gemm(pkg):
    """The training path's bias-free bf16 GEMM against torch's autocast Linear:
    the same bf16 output, and fp32 input / weight gradients at least as close
    to the fp64 reference as autocast's (which round them to bf16 first)."""
    from spikingtransformer_b200._fused import LinearBF16, bf16_input
    g = torch.Generator(device=DEV).manual_seed(3)
    lin = torch.nn.Linear(96, 160, bias=False).to(DEV)
    x = torch.randn(4, 50, 96, generator=g, device=DEV, requires_grad=True)
    gy = torch.randn(4, 50, 160, generator=g, device=DEV).to(torch.bfloat16)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        xb = bf16_input(x)
        y = LinearBF16.apply(x, lin.weight, xb, lin.weight.detach().to(torch.bfloat16))
        y_ref = torch.nn.functional.linear(x, lin.weight)
    assert y.dtype == torch.bfloat16 and torch.equal(y, y_ref)
    y.backward(gy)
    dx, dw = x.grad.clone(), lin.weight.grad.clone()
    assert dx.dtype == torch.float32 and dw.dtype == torch.float32
    x64, w64 = x.detach().double(), lin.weight.detach().double()
    xr, wr = x64.to(torch.bfloat16).double(), w64.to(torch.bfloat16).double()
    dx64 = gy.double() @ wr
    dw64 = gy.double().reshape(-1, 160).t() @ xr.reshape(-1, 96)
    assert (dx.double() - dx64).abs().max() <= 1e-5 * dx64.abs().max()
    assert (dw.double() - dw64).abs().max() <= 1e-5 * dw64.abs().max()


def test_mlp_golden(pkg, golden_dir):
    from spikingtransformer_b200.SpikingMLP import SpikingMLP
    c = load(golden_dir, "mlp.pt")
    m = SpikingMLP(c["D"], c["F"], n_steps=c["T"]).to(DEV)
    m.load_state_dict(c["state"])
    with torch.no_grad():
        y = m(c["x"].to(DEV))
    T = c["T"]
    beta = torch.sigmoid(c["state"]["lifcompress.beta_raw"])
    vh = membrane_history(c["ln_compress"].reshape(T, -1), beta, 1.0, 0.0)
    assert_spikes_match(y.reshape(T, -1), c["out"].reshape(T, -1), vh, 1.0, what="mlp")


def test_encoder_decoder_golden(pkg, golden_dir):
    from spikingtransformer_b200.Encoder import Encoder
    from spikingtransformer_b200.Decoder import Decoder
    c = load(golden_dir, "stacks.pt")
    enc = Encoder(2, c["D"], c["H"], c["F"], n_steps=c["T"]).to(DEV)
    enc.load_state_dict(c["enc_state"])
    dec = Decoder(1, c["D"], c["H"], c["F"], n_steps=c["T"]).to(DEV)
    dec.load_state_dict(c["dec_state"])
    with torch.no_grad():
        y = enc(c["x"].to(DEV))
        z = dec(c["tgt"].to(DEV), c["enc_out"].to(DEV), mask=c["mask"].to(DEV))
    assert spike_mismatch_rate(y, c["enc_out"]) < 0.01
    assert spike_mismatch_rate(z, c["dec_out"]) < 0.01


def test_seq2seq_cnn_golden(pkg, golden_dir):
    from spikingtransformer_b200.Seq2Seq import Seq2Seq
    c = load(golden_dir, "seq2seq_cnn.pt")
    m = Seq2Seq(patch_size=4, d_model=32, n_heads=4, ff_dim=64, num_encoder_layers=1, num_decoder_layers=1,
                tgt_vocab_size=40, nb_sps_blocks=1, n_steps=c["T"]).to(DEV)
    m.load_state_dict(c["state"])
    m.eval()
    with torch.no_grad():
        logits, aux = m(c["src"].to(DEV), c["tgt"].to(DEV), look_ahead_mask=c["mask"].to(DEV))
        enc, _ = m.encode(c["src"].to(DEV))
    assert aux is None
    assert logits.shape == c["logits"].shape
    assert spike_mismatch_rate(enc, c["enc"]) < 0.01
    close = torch.isclose(logits.cpu(), c["logits"], rtol=1e-4, atol=1e-4).float().mean().item()
    assert close > 0.95, close


def _cnn_pair(D=64, nb_layers=2, T=4, seed=5):
    """CNNBackbone (ours on the GPU, the oracle's on the CPU) with bf16-rounded
    convolution weights and non-trivial BatchNorm statistics, in eval mode."""
    from spikingtransformer_b200.ImageEncoder import CNNBackbone
    torch.manual_seed(seed)
    ours = CNNBackbone(d_model=D, nb_layers=nb_layers, patch_size=4, n_steps=T)
    with torch.no_grad():
        for m in ours.modules():
            if isinstance(m, (torch.nn.Conv2d, torch.nn.Conv1d)):
                m.weight.copy_((m.weight * 3).to(torch.bfloat16).float())
            if isinstance(m, (torch.nn.BatchNorm2d, torch.nn.BatchNorm1d)):
                m.running_mean.uniform_(-0.2, 0.2)
                m.running_var.uniform_(0.5, 1.5)
                m.weight.uniform_(0.8, 1.2)
                m.bias.uniform_(0.2, 0.6)
    ref = om.CNNBackbone(d_model=D, nb_layers=nb_layers, patch_size=4, n_steps=T)
    ref.load_state_dict(ours.state_dict())
    return ours.to(DEV).eval(), ref.eval()


def test_cnn_backbone_fused_matches_oracle(pkg):
    """The CNN image encoder in eval mode on this package's kernels (patch
    gathers, tcgen05 GEMMs with the BatchNorm affine and LIF epilogue), no
    library convolution: the first convolution's spikes bit-exact outside the
    near-threshold band, the output tokens within the whole-stack bound, and
    the once-per-image path equal to the T-fold path."""
    T, B = 4, 3
    ours, ref = _cnn_pair()
    src = synthetic_lines(B, 21, H=32, W=128)
    x = src.unsqueeze(0).expand(T, *src.shape).reshape(T * B, *src.shape[1:])
    with torch.no_grad():
        y, rec = ours(x.to(DEV))
        y_ref, rec_ref = ref(x)
        pre1 = ref.bn1(ref.conv1(ref.space_to_depth(x)))
        once = ours.encode_images(src.to(DEV), T)
    assert y.shape == y_ref.shape and y.dtype == torch.float32
    vh = membrane_history(pre1.reshape(T, -1), 0.5, 1.0, 0.0)
    assert_spikes_match(rec["conv1"].float().reshape(T, -1), rec_ref["conv1"].reshape(T, -1), vh, 1.0,
                        what="conv1 spikes")
    rate = spike_mismatch_rate(y, y_ref)
    assert rate < 0.01, rate
    assert torch.equal(once.float(), y)


def test_cnn_backbone_runs_no_library_convolution(pkg):
    ours, _ = _cnn_pair(nb_layers=1)
    x = synthetic_lines(4, 22, H=32, W=128).to(DEV)
    with torch.no_grad():
        ours(x)
        torch.cuda.synchronize()
        with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA]) as prof:
            ours(x)
            torch.cuda.synchronize()
    names = [e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]
    assert any("gemm_ln_lif_kernel" in n for n in names), names[:20]
    library_conv = [n for n in names if ("cudnn" in n.lower() or "conv" in n.lower()) and "spk::" not in n]
    assert not library_conv, library_conv


def _bench_models(seed=0, enc_layers=8, dec_layers=4, T=4):
    """The OCR benchmark architecture (D=384, H=8, F=1536, patch 16, vocab 256),
    bf16-rounded random weights, ours on the GPU and the oracle on the CPU."""
    from spikingtransformer_b200.Seq2Seq import Seq2Seq
    torch.manual_seed(seed)
    ours = Seq2Seq(patch_size=16, d_model=384, n_heads=8, ff_dim=1536, num_encoder_layers=enc_layers,
                   num_decoder_layers=dec_layers, tgt_vocab_size=256, n_steps=T, image_encoder="patch")
    with torch.no_grad():
        for mod in ours.modules():
            if isinstance(mod, (torch.nn.Linear, torch.nn.Conv2d)):
                mod.weight.copy_(mod.weight.to(torch.bfloat16).float())
    ref = om.Seq2Seq(patch_size=16, d_model=384, n_heads=8, ff_dim=1536, num_encoder_layers=enc_layers,
                     num_decoder_layers=dec_layers, tgt_vocab_size=256, n_steps=T, image_encoder="patch")
    ref.load_state_dict(ours.state_dict())
    return ours.to(DEV).eval(), ref.eval()


def synthetic_lines(B, seed, H=64, W=1024):
    """Text-line stand-ins: U(0, 0.2) background plus 5-40 black rectangles of
    side 8-20 px per image, from a seed."""
    g = torch.Generator().manual_seed(seed)
    img = torch.rand(B, 1, H, W, generator=g) * 0.2
    for b in range(B):
        n = int(torch.randint(5, 41, (1,), generator=g))
        for _ in range(n):
            h, w = (int(v) for v in torch.randint(8, 21, (2,), generator=g))
            y = int(torch.randint(0, H - h + 1, (1,), generator=g))
            x = int(torch.randint(0, W - w + 1, (1,), generator=g))
            img[b, 0, y:y + h, x:x + w] = 0.0
    return img


def test_seq2seq_ocr_benchmark_architecture(pkg):
    ours, ref = _bench_models()
    B, N = 2, 64
    src = synthetic_lines(B, 1)
    tgt = torch.randint(0, 256, (B, N), generator=torch.Generator().manual_seed(2))
    mask = torch.tril(torch.ones(N, N)).expand(B, 1, N, N)
    with torch.no_grad():
        enc_ref, _ = ref.encode(src)
        logits_ref, _ = ref(src, tgt, look_ahead_mask=mask)
        enc, _ = ours.encode(src.to(DEV))
        logits, _ = ours(src.to(DEV), tgt.to(DEV), look_ahead_mask=mask.to(DEV))
    # the first layer's patch-embedding spikes must match outside the near-threshold band
    with torch.no_grad():
        pe_ours, _ = ours.image_encoder(src.to(DEV).unsqueeze(0).expand(4, *src.shape).reshape(4 * B,
                                                                                              *src.shape[1:]))
        y = ref.image_encoder.norm(ref.image_encoder.proj(
            src.unsqueeze(0).expand(4, *src.shape).reshape(4 * B, *src.shape[1:])).flatten(2).transpose(1, 2))
        pe_ref = ref.image_encoder.lif(y)[0]
    vh = membrane_history(y.reshape(4, -1), 0.9, 1.0, 0.0)
    assert_spikes_match(pe_ours.reshape(4, -1), pe_ref.reshape(4, -1), vh, 1.0, what="patch embedding")
    rate_enc = spike_mismatch_rate(enc, enc_ref)
    assert rate_enc < 0.02, rate_enc
    close = torch.isclose(logits.cpu(), logits_ref, rtol=1e-3, atol=1e-3).float().mean().item()
    assert close > 0.9, close


def test_seq2seq_training_path_runs(pkg):
    """Autograd path (reference composition over the LIF kernels) with the
    arctan surrogate: finite loss and gradients on every parameter."""
    ours, _ = _bench_models(enc_layers=1, dec_layers=1)
    ours.train()
    ours.set_surrogate("arctan", 2.0)
    B, N = 2, 16
    src = synthetic_lines(B, 3).to(DEV)
    tgt = torch.randint(0, 256, (B, N + 1), device=DEV)
    mask = torch.tril(torch.ones(N, N, device=DEV)).expand(B, 1, N, N)
    logits, _ = ours(src, tgt[:, :-1], look_ahead_mask=mask)
    loss = sum(torch.nn.functional.cross_entropy(logits[t].reshape(-1, 256), tgt[:, 1:].reshape(-1))
               for t in range(logits.shape[0])) / logits.shape[0]
    loss.backward()
    assert math.isfinite(loss.item())
    missing = [n for n, p in ours.named_parameters() if p.grad is None]
    assert not [n for n in missing if "image_encoder" not in n], missing


def test_seq2seq_train_steps_bf16_autocast(pkg):
    """Three optimizer steps as the training workload runs them (bf16
    autocast, mean over T of the per-step cross-entropy, AdamW): finite losses
    and every trained weight updated."""
    ours, _ = _bench_models(enc_layers=1, dec_layers=1)
    ours.train()
    ours.set_surrogate("arctan", 2.0)
    opt = torch.optim.AdamW(ours.parameters(), lr=1e-3)
    B, N = 2, 16
    src = synthetic_lines(B, 5).to(DEV)
    tgt = torch.randint(0, 256, (B, N + 1), device=DEV, generator=torch.Generator(device=DEV).manual_seed(5))
    mask = torch.tril(torch.ones(N, N, device=DEV)).expand(B, 1, N, N)
    before = {n: p.detach().clone() for n, p in ours.named_parameters()}
    losses = []
    for _ in range(3):
        opt.zero_grad(set_to_none=True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            logits, _ = ours(src, tgt[:, :-1], look_ahead_mask=mask)
            loss = sum(torch.nn.functional.cross_entropy(logits[t].reshape(-1, 256).float(), tgt[:, 1:].reshape(-1))
                       for t in range(logits.shape[0])) / logits.shape[0]
        loss.backward()
        assert all(torch.isfinite(p.grad).all() for p in ours.parameters() if p.grad is not None)
        opt.step()
        losses.append(loss.item())
    assert all(math.isfinite(x) for x in losses)
    changed = [n for n, p in ours.named_parameters() if not torch.equal(p.detach(), before[n])]
    assert any("out_proj" in n for n in changed) and any("output_layer" in n for n in changed)


def test_train_step_cuda_graph_matches_eager(pkg):
    """A training step (bf16 autocast, fused loss, capturable AdamW) captured in
    a CUDA graph and replayed gives the losses of the same steps run eagerly
    from the same start: the training path makes no host synchronisation and
    keeps no stale cached tensor that a graph would freeze."""
    from spikingtransformer_b200 import ops
    B, N = 2, 16
    data = []
    for i in range(4):
        src = synthetic_lines(B, 30 + i).to(DEV)
        tgt = torch.randint(1, 256, (B, N + 1), device=DEV, generator=torch.Generator(device=DEV).manual_seed(i))
        data.append((src, tgt))
    mask = torch.tril(torch.ones(N, N, device=DEV)).expand(B, 1, N, N)

    def make():
        m, _ = _bench_models(enc_layers=1, dec_layers=1)
        m.train()
        m.set_surrogate("arctan", 2.0)
        return m, torch.optim.AdamW(m.parameters(), lr=1e-3, fused=True, capturable=True)

    def step(m, opt, src, tgt, cache):
        with torch.autocast("cuda", dtype=torch.bfloat16, cache_enabled=cache):
            logits, _ = m(src, tgt[:, :-1], look_ahead_mask=mask)
        loss, acc, _ = ops.ce_over_t(logits, tgt[:, 1:], ignore_index=0, label_smoothing=0.1)
        loss.backward()
        opt.step()
        return loss

    m1, o1 = make()
    eager = []
    for src, tgt in data:
        o1.zero_grad(set_to_none=True)
        eager.append(step(m1, o1, src, tgt, False).item())

    m2, o2 = make()
    s_src, s_tgt = data[0][0].clone(), data[0][1].clone()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for src, tgt in data[:2]:
            s_src.copy_(src)
            s_tgt.copy_(tgt)
            o2.zero_grad(set_to_none=True)
            step(m2, o2, s_src, s_tgt, False)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    o2.zero_grad(set_to_none=True)
    with torch.cuda.graph(graph):
        g_loss = step(m2, o2, s_src, s_tgt, False)
    replayed = []
    for src, tgt in data[2:]:
        s_src.copy_(src)
        s_tgt.copy_(tgt)
        graph.replay()
        replayed.append(g_loss.item())
    assert all(math.isfinite(x) for x in eager + replayed)
    assert replayed == pytest.approx(eager[2:], rel=1e-4), (eager, replayed)
    del graph


def test_greedy_decode(pkg):
    ours, _ = _bench_models(enc_layers=1, dec_layers=1)
    src = synthetic_lines(1, 4)[0]
    ys, rec, out = ours.greedy_decode(src, max_len=5, start_symbol=1, eos_idx=2, pad_idx=0, device=DEV)
    assert ys.shape[0] == 1 and 2 <= ys.shape[1] <= 5
    assert rec is None
    assert out.shape[0] == 4


def test_cached_cross_kv_decode_is_exact(pkg):
    """The decoder with the cross-attention K/V spikes computed once gives the
    logits of the decoder that projects the encoder output every call."""
    ours, _ = _bench_models(enc_layers=1, dec_layers=2)
    with torch.no_grad():
        src = synthetic_lines(2, 11).to(DEV)
        enc = ours._encode_fast(src)
        cross_kv = ours.decoder.cross_key_values(enc)
        tgt = torch.randint(0, 256, (2, 9), device=DEV, generator=torch.Generator(device=DEV).manual_seed(3))
        mask = ours.create_decoder_mask(tgt, 0, DEV)
        a = ours._decode_fast(tgt, enc, mask)
        b = ours._decode_fast(tgt, enc, mask, cross_kv)
    assert torch.equal(a, b)


def test_greedy_decode_batch_matches_single_image(pkg):
    """Row b of the batched greedy decode is what greedy_decode returns for
    image b alone, with an eos that stops one row early."""
    ours, _ = _bench_models(enc_layers=1, dec_layers=1)
    B, L = 3, 7
    src = synthetic_lines(B, 12)
    singles = [ours.greedy_decode(src[b], max_len=L, start_symbol=1, eos_idx=-1, pad_idx=0, device=DEV)[0]
               for b in range(B)]
    eos = int(singles[0][0, 2])  # the token image 0 emits second: it stops there
    singles = [ours.greedy_decode(src[b], max_len=L, start_symbol=1, eos_idx=eos, pad_idx=0, device=DEV)[0]
               for b in range(B)]
    ys, lengths = ours.greedy_decode_batch(src, max_len=L, start_symbol=1, eos_idx=eos, pad_idx=0, device=DEV)
    assert ys.shape[0] == B
    for b in range(B):
        n = singles[b].shape[1]
        assert int(lengths[b]) == n
        assert torch.equal(ys[b, :n], singles[b][0])
        assert bool((ys[b, n:] == 0).all())
    assert int(lengths[0]) == 3


def test_greedy_decode_matches_oracle(pkg):
    """Token sequence of the fused greedy decode against the CPU oracle's on a
    small model."""
    ours, ref = _bench_models(enc_layers=1, dec_layers=1)
    src = synthetic_lines(1, 13)[0]
    ys, _, out = ours.greedy_decode(src, max_len=5, start_symbol=1, eos_idx=-1, pad_idx=0, device=DEV)
    ys_ref, _, out_ref = ref.greedy_decode(src, max_len=5, start_symbol=1, eos_idx=-1, pad_idx=0, device="cpu")
    assert torch.equal(ys.cpu(), ys_ref)
    close = torch.isclose(out.cpu(), out_ref, rtol=1e-3, atol=1e-3).float().mean().item()
    assert close > 0.9, close


def test_stream_forward_matches_direct_forward(pkg):
    """Host batches streamed with overlapped copies give the logits of a
    direct forward of each batch, bit for bit, including a host buffer reused
    by several batches."""
    from spikingtransformer_b200.streaming import stream_forward
    ours, _ = _bench_models(enc_layers=1, dec_layers=1)
    B, N = 2, 16
    batches = []
    for i in range(5):
        src = synthetic_lines(B, 20 + i)
        tgt = torch.randint(0, 256, (B, N), generator=torch.Generator().manual_seed(30 + i))
        mask = torch.tril(torch.ones(N, N)).expand(B, 1, N, N).contiguous()
        batches.append((src.pin_memory(), tgt.pin_memory(), mask.pin_memory()))
    with torch.no_grad():
        want = [ours(s.to(DEV), t.to(DEV), look_ahead_mask=m.to(DEV))[0].cpu() for s, t, m in batches]
        outs = [torch.empty_like(want[0]).pin_memory() for _ in range(5)]
        stream_forward(lambda s, t, m: ours(s, t, look_ahead_mask=m)[0], batches, outs)
        torch.cuda.current_stream().synchronize()
        for i in range(5):
            assert torch.equal(outs[i], want[i]), i
        shared = torch.empty_like(want[0]).pin_memory()
        stream_forward(lambda s, t, m: ours(s, t, look_ahead_mask=m)[0], batches, [shared] * 5)
        torch.cuda.current_stream().synchronize()
        assert torch.equal(shared, want[4])


def test_public_stack_forwards_do_not_synchronise(pkg):
    """Seq2Seq.encode / decode and the Encoder / Decoder / LIF module forwards
    on the inference path enqueue work without a device-to-host read (the
    stream's exactness in bf16 is known from where it came from, not read
    back)."""
    from spikingtransformer_b200.Lif import LIF
    ours, _ = _bench_models(enc_layers=1, dec_layers=1)
    B, N = 2, 16
    src = synthetic_lines(B, 6).to(DEV)
    tgt = torch.randint(0, 256, (B, N), device=DEV, generator=torch.Generator(device=DEV).manual_seed(6))
    mask = torch.tril(torch.ones(N, N, device=DEV)).expand(B, 1, N, N)
    lif = LIF(n_steps=4).to(DEV)
    x_in = torch.rand(4 * B, 10, device=DEV)
    with torch.no_grad():
        ours(src, tgt, look_ahead_mask=mask)  # warm caches (weights, LIF parameters)
        torch.cuda.synchronize()
        torch.cuda.set_sync_debug_mode("error")
        try:
            enc, _ = ours.encode(src)
            logits, _ = ours.decode(tgt, enc, mask)
            enc2 = ours.encoder(ours.image_encoder.encode_images(src).float())
            s, _ = lif(x_in)
        finally:
            torch.cuda.set_sync_debug_mode(0)
        want, _ = ours(src, tgt, look_ahead_mask=mask)
    assert torch.equal(logits, want)
    assert enc2.dtype == torch.float32 and s.shape == x_in.shape


def test_stack_forward_leaves_bf16_input_unchanged(pkg):
    """A bf16 residual stream handed to Encoder.forward is copied, not
    updated in place."""
    ours, _ = _bench_models(enc_layers=1, dec_layers=1)
    src = synthetic_lines(2, 8).to(DEV)
    with torch.no_grad():
        x = ours.image_encoder.encode_images(src)
        keep = x.clone()
        y = ours.encoder(x)
    assert torch.equal(x, keep)
    assert not torch.equal(y, keep)


def test_no_device_timeouts(pkg):
    from spikingtransformer_b200 import ops
    ops.device_error_check()


def test_forward_cuda_graph_matches_eager(pkg):
    """The inference forward captured once in a CUDA graph (as the forward
    benchmark times it) and replayed on new inputs copied into its buffers
    gives the eager forward's logits bit for bit."""
    ours, _ = _bench_models(enc_layers=2, dec_layers=1)
    B, N = 4, 64
    sets = []
    for i in range(3):
        src = synthetic_lines(B, 40 + i).to(DEV)
        tgt = torch.randint(0, 256, (B, N), device=DEV, generator=torch.Generator(device=DEV).manual_seed(40 + i))
        sets.append((src, tgt))
    mask = torch.tril(torch.ones(N, N, device=DEV)).expand(B, 1, N, N).contiguous()
    with torch.no_grad():
        static = [t.clone() for t in sets[0]]
        ours(static[0], static[1], look_ahead_mask=mask)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            out = ours(static[0], static[1], look_ahead_mask=mask)[0]
        for i in (1, 2, 0):
            for a, b in zip(static, sets[i]):
                a.copy_(b)
            graph.replay()
            want = ours(sets[i][0], sets[i][1], look_ahead_mask=mask)[0]
            assert torch.equal(out, want), i
