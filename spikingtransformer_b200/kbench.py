"""Kernel micro-benchmarks at the benchmark shapes (CUDA events, device time).

    python -m spikingtransformer_b200.kbench [--only lif|gemm|ssa|ssa_model|data|shapes|lnlif] [--iters N]

  lif   LIF forward on [T=4, 64*256, 1536] fp32 input -> bf16 and packed-bit
        spikes (the MLP expansion LIF of a 64-image batch), and the backward
        from packed bits; bound: HBM bytes.
  gemm  fused Linear(384->1536) -> LayerNorm -> LIF on A [4*32*256, 384]
        Bernoulli(0.15) spikes (bf16), tau=2 neuron; bound: bf16 tensor FLOPs.
  ssa   spiking attention on Q, K, V [T=4, B=32, H=8, N=256, d=48]
        Bernoulli(0.15), plain (QK^T)V*0.125 and XNOR variants, plus the
        causal N=64 case; FLOPs counted dense (QK^T and PV); and the n-major
        copy of V [2048, 256, 48] bf16 that the training path's R V reads,
        beside torch's permute copy.
  attn_train  the decoder's masked self-attention core in training (forward
        and backward), fused kernels beside the reference composition.
  cnn   the reference's CNN image encoder (eval) on 64 text lines of 32 x 512,
        fused path beside the library convolutions.
  train_gemm  the training step's Linear gradient GEMMs (dgrad, wgrad) at 64
        images, this package's kernels beside torch's.
  ssa_model  the forward's three attention calls at the bench batch (256
        images): encoder self 256 x 256, decoder cross 64 x 256, decoder
        self 64 x 64 with the dense look-ahead mask; bound: HBM bytes.
Inputs are regenerated per configuration; each timed iteration rotates over
input copies whose total exceeds the 126 MB L2.  Prints one JSON line.
"""

import argparse
import json
import os

import torch

from . import ops


def _peaks():
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    try:
        with open(os.path.join(root, "MEASURED_PEAKS.json")) as f:
            return json.load(f), "measured"
    except (OSError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def _time(fn, iters, warmup=3):
    """Device time per call: the calls are captured once into a CUDA graph and
    replayed, so host launch overhead does not enter the measurement."""
    for i in range(warmup):
        fn(i)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(iters):
            fn(i)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    g.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters


def bench_lif(iters, N=64 * 256 * 1536):
    """Forward to bf16 and to packed-bit spikes, and the backward from packed
    bits, on [4, N] fp32 N(0.5, 1) currents (tau = 2 neuron)."""
    T = 4
    copies = 2
    xs = [torch.randn(T, N, device="cuda") + 0.5 for _ in range(copies)]
    res = []
    for fmt, sbytes in ((torch.bfloat16, 2 * T * N), ("bits", T * ((N + 7) // 8))):
        ms = _time(lambda i: ops.lif_fwd(xs[i % copies], 0.5, 1.0, 0.0, in_gain=0.5, spike_dtype=fmt), iters)
        nbytes = T * N * 4 + sbytes + 4 * N
        res.append({"kernel": "lif_fwd", "spikes": str(fmt), "shape": [T, N], "ms": ms, "GB/s": nbytes / ms / 1e6,
                    "bytes": nbytes})
    sb = [ops.lif_fwd(x, 0.5, 1.0, 0.0, in_gain=0.5, spike_dtype="bits", want_v_final=False)[0] for x in xs]
    gs = torch.randn(T, N, device="cuda")
    ms = _time(lambda i: ops.lif_bwd(gs, None, xs[i % copies], sb[i % copies], 0.5, 1.0, 0.0, in_gain=0.5,
                                     spikes_packed=True), iters)
    nbytes = T * N * 12 + T * ((N + 7) // 8)
    res.append({"kernel": "lif_bwd", "spikes": "bits", "shape": [T, N], "ms": ms, "GB/s": nbytes / ms / 1e6,
                "bytes": nbytes})
    return res


def bench_gemm(iters, N=1536, K=384, T=4, R=32 * 256):
    g = torch.Generator(device="cuda").manual_seed(0)
    copies = 3
    As = [(torch.rand(T * R, K, device="cuda", generator=g) < 0.15).to(torch.bfloat16) for _ in range(copies)]
    bound = 1.0 / K ** 0.5
    W = ((torch.rand(N, K, device="cuda", generator=g) * 2 - 1) * bound).to(torch.bfloat16)
    b = (torch.rand(N, device="cuda", generator=g) * 2 - 1) * 0.01
    gamma, beta = torch.ones(N, device="cuda"), torch.zeros(N, device="cuda")
    ms = _time(lambda i: ops.linear_ln_lif(As[i % copies], W, b, gamma, beta, 1e-5, 0.5, 1.0, 0.0, T,
                                           in_gain=0.5), iters)
    flops = 2.0 * T * R * K * N
    return {"kernel": "linear_ln_lif", "shape": [T * R, K, N], "ms": ms, "TFLOP/s": flops / ms / 1e9,
            "flops": flops}


def bench_ssa(iters, variant, N=256, causal=False, T=4, B=32, H=8, d=48, Nk=None, dense_mask=False):
    """``dense_mask``: the decoder's call, a [B, 1, N, N] look-ahead mask
    passed as uint8 and broadcast over T and heads (strides 0)."""
    Nk = N if Nk is None else Nk
    g = torch.Generator(device="cuda").manual_seed(1)
    copies = 2
    mk = lambda n: (torch.rand(T * B, n, H * d, device="cuda", generator=g) < 0.15).to(torch.bfloat16)  # noqa
    qkv = [(mk(N), mk(Nk), mk(Nk)) for _ in range(copies)]
    scale = 0.125 if variant == 0 else (1.0 / d) ** 0.5
    mask = ops.mask_to_u8(torch.tril(torch.ones(N, Nk, device="cuda")).expand(B, 1, N, Nk), T, B, H, N, Nk) \
        if dense_mask else None

    def run(i):
        q, k, v = qkv[i % copies]
        ops.ssa(q, k, v, T, B, H, variant, scale, 0.5, 0.5, 0.0, in_gain=0.5, causal=causal, mask=mask)
    ms = _time(run, iters)
    flops = 4.0 * T * B * H * N * Nk * d
    nbytes = 2.0 * T * B * H * d * (2 * N + 2 * Nk)
    return {"kernel": "ssa", "variant": "plain" if variant == 0 else "xnor", "causal": causal,
            "dense_mask": dense_mask, "shape": [T, B, H, N, Nk, d], "ms": ms,
            "TFLOP/s_dense_equiv": flops / ms / 1e9, "flops_dense": flops, "GB/s": nbytes / ms / 1e6}


def bench_train_gemm(iters, M=65536):
    """The training step's Linear gradient GEMMs at 64 images (M = 4 x 64 x 256
    rows): this package's tcgen05 kernels beside torch's (cuBLAS), bf16
    operands, fp32 output; FLOPs 2 M N K."""
    g = torch.Generator(device="cuda").manual_seed(5)
    out = []
    for N, K, what in ((1152, 384, "q/k/v stacked"), (384, 384, "out_proj"), (1536, 384, "expand"),
                       (384, 1536, "compress")):
        Gs = [torch.randn(M, N, device="cuda", generator=g).to(torch.bfloat16) for _ in range(2)]
        Xs = [(torch.rand(M, K, device="cuda", generator=g) < 0.2).to(torch.bfloat16) for _ in range(2)]
        W = (torch.randn(N, K, device="cuda", generator=g) * 0.05).to(torch.bfloat16)
        flops = 2.0 * M * N * K
        for name, fn in (("dgrad ours", lambda i: ops.linear_dgrad(Gs[i % 2], W)),
                         ("dgrad torch", lambda i: torch.mm(Gs[i % 2], W, out_dtype=torch.float32)),
                         ("wgrad ours", lambda i: ops.linear_wgrad(Gs[i % 2], Xs[i % 2])),
                         ("wgrad torch", lambda i: torch.mm(Gs[i % 2].t(), Xs[i % 2], out_dtype=torch.float32))):
            ms = _time(fn, iters)
            out.append({"kernel": name, "layer": what, "M": M, "N": N, "K": K, "ms": ms,
                        "TFLOP/s": flops / ms / 1e9})
    return out


def bench_cnn(iters, B=64, T=4, D=384, layers=4, H=32, W=512):
    """The reference's CNN image encoder (``CNNBackbone``, patch 4, 32 x 512
    text lines, eval mode) on B images repeated over T: this package's fused
    path (patch gathers + GEMMs with the BatchNorm-affine and LIF epilogue,
    first convolution once per image) beside the reference composition on
    the same module (library convolutions and BatchNorm, the LIF kernel) on
    the T-fold."""
    from .ImageEncoder import CNNBackbone
    torch.manual_seed(0)
    m = CNNBackbone(d_model=D, nb_layers=layers, patch_size=4, n_steps=T).cuda().eval()
    g = torch.Generator(device="cuda").manual_seed(3)
    srcs = [torch.rand(B, 1, H, W, device="cuda", generator=g) * 0.2 for _ in range(2)]
    folds = [x.unsqueeze(0).expand(T, *x.shape).reshape(T * B, 1, H, W).contiguous() for x in srcs]
    out = []
    with torch.no_grad():
        ms = _time(lambda i: m.encode_images(srcs[i % 2], T), iters)
        out.append({"kernel": "cnn_backbone fused", "images": B, "T": T, "layers": layers, "ms": ms,
                    "images/s": B / ms * 1e3})

        def library(i):
            x = m.space_to_depth(folds[i % 2])
            x = m.lif_1(m.bn1(m.conv1(x)))[0]
            x = m.lif_2(m.bn2(m.conv2(x)))[0]
            for layer in m.layers:
                x = layer(x)
            x = m.reduce(x)
            return x + m.rpe(x)
        ms = _time(library, iters)
        out.append({"kernel": "cnn_backbone library conv + BatchNorm + LIF kernel", "images": B, "T": T,
                    "layers": layers, "ms": ms, "images/s": B / ms * 1e3})
    return out


def bench_attn_train(iters, B=64, T=4, H=8, N=64, d=48):
    """The decoder's masked self-attention core in training at 64 images
    (``[T*B, H, 64, 48]`` head-major bf16 spikes, causal mask, XNOR with the
    log-distance bias): the fused forward and backward kernels, and the
    reference composition (score matrix, bias, mask, scale, @ V and their
    autograd) beside them."""
    from .SSA import MaskedShortAttention, SSAMultiHeadAttention
    g = torch.Generator(device="cuda").manual_seed(7)
    TB = T * B
    q, k, v = ((torch.rand(TB, H, N, d, device="cuda", generator=g) < 0.3).to(torch.bfloat16) for _ in range(3))
    mask = torch.tril(torch.ones(N, N, device="cuda")).expand(TB, 1, N, N)
    scale = torch.tensor((1.0 / d) ** 0.5, device="cuda", requires_grad=True)
    gout = torch.randn(TB, N, H * d, device="cuda", generator=g)
    m = SSAMultiHeadAttention(H * d, H, n_steps=T).cuda()
    out = []

    def fused(i):
        qq, kk, vv = (t.detach().requires_grad_() for t in (q, k, v))
        MaskedShortAttention.apply(qq, kk, vv, scale, mask, T, 1).backward(gout)

    def composition(i):
        qq, kk, vv = (t.detach().float().requires_grad_() for t in (q, k, v))
        a = m.xnor_attention(qq, kk) + m.get_log_pe_bias_cross(N, N, qq.device)
        ((a * mask * scale) @ vv).transpose(1, 2).reshape(TB, N, H * d).backward(gout)
    for name, fn in (("masked attention fwd+bwd, fused kernels", fused),
                     ("masked attention fwd+bwd, reference composition", composition)):
        for i in range(3):
            fn(i)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(iters):
            fn(i)
        e1.record()
        torch.cuda.synchronize()
        out.append({"kernel": name, "shape": [TB, H, N, d], "ms": e0.elapsed_time(e1) / iters})
    return out


def bench_n_major(iters, B=2048, N=256, d=48):
    """The n-major copy of V for the training attention's R V product
    ([B, N, d] bf16 -> [N, B*d], B = T*images*H at 64 images), against
    torch's strided permute copy of the same tensor; bound: HBM bytes."""
    g = torch.Generator(device="cuda").manual_seed(2)
    xs = [(torch.rand(B, N, d, device="cuda", generator=g) < 0.15).to(torch.bfloat16) for _ in range(3)]
    nbytes = 2 * xs[0].numel() * 2
    out = []
    for name, fn in (("xnor_train_n_major", ops.xnor_train_n_major),
                     ("torch permute copy", lambda x: x.permute(1, 0, 2).reshape(N, B * d))):
        ms = _time(lambda i: fn(xs[i % 3]), iters)
        out.append({"kernel": name, "shape": [B, N, d], "ms": ms, "GB/s": nbytes / ms / 1e6, "bytes": nbytes})
    return out


def bench_data(iters):
    """The on-device batch generator (256 images [1, 64, 1024] + 64 targets
    each) and the fused loss at the training shape (T=4, 64 images x 64
    positions, vocab 256; forward and gradient); bound: HBM bytes."""
    out = []
    ms = _time(lambda i: ops.synth_text_lines(256, 1000 + i, H=64, W=1024, L=64, V=256), iters)
    nbytes = 256 * 64 * 1024 * 4 + 256 * 64 * 8
    out.append({"kernel": "synth_text_lines", "shape": [256, 1, 64, 1024], "ms": ms, "GB/s": nbytes / ms / 1e6,
                "images/s": 256 / ms * 1e3, "bytes": nbytes})
    g = torch.Generator(device="cuda").manual_seed(5)
    logits = [torch.randn(4, 64, 64, 256, device="cuda", generator=g).requires_grad_(True) for _ in range(2)]
    tgt = torch.randint(0, 256, (64, 64), device="cuda", generator=g)

    def run(i):
        loss, _, _ = ops.ce_over_t(logits[i % 2], tgt, ignore_index=0, label_smoothing=0.1)
        loss.backward()
    ms = _time(run, iters)
    nbytes = 2 * logits[0].numel() * 4 * 2  # logits read, gradient written, gradient accumulated
    out.append({"kernel": "ce_over_t (+backward)", "shape": [4, 64, 64, 256], "ms": ms, "GB/s": nbytes / ms / 1e6,
                "bytes": nbytes})
    return out


def bench_shapes_once():
    """Each fused launch shape of the 256-image forward, twice, untimed (a
    short program for per-launch DRAM captures with ncu).  Order: q/k/v,
    out_proj + residual, expand, compress + residual (encoder rows 4 x 256 x
    256), patch embedding (t-broadcast), encoder self-attention, decoder
    cross-attention, decoder causal self-attention."""
    g = torch.Generator(device="cuda").manual_seed(0)
    T, R, D = 4, 256 * 256, 384
    spk = lambda *shape: (torch.rand(*shape, device="cuda", generator=g) < 0.15).to(torch.bfloat16)  # noqa: E731
    w = lambda n, k: ((torch.rand(n, k, device="cuda", generator=g) * 2 - 1) / k ** 0.5).to(torch.bfloat16)  # noqa
    ones = lambda n: torch.ones(n, device="cuda")  # noqa: E731
    zeros = lambda n: torch.zeros(n, device="cuda")  # noqa: E731
    A384, A1536 = spk(T * R, D), spk(T * R, 4 * D)
    W = {(384, 384): w(384, 384), (1536, 384): w(1536, 384), (384, 1536): w(384, 1536), (384, 512): w(384, 512)}
    res = torch.zeros(T * R, D, dtype=torch.bfloat16, device="cuda")
    patches = (torch.rand(R, 512, device="cuda", generator=g) * 0.2).to(torch.bfloat16)
    lif = (0.5, 1.0, 0.0)
    for _ in range(2):
        ops.linear_ln_lif(A384, W[(384, 384)], zeros(384), ones(384), zeros(384), 1e-5, *lif, T, in_gain=0.5)
    for _ in range(2):
        ops.linear_ln_lif(A384, W[(384, 384)], zeros(384), ones(384), zeros(384), 1e-5, *lif, T, in_gain=0.5,
                          residual=res, want_spikes=False)
    for _ in range(2):
        ops.linear_ln_lif(A384, W[(1536, 384)], zeros(1536), ones(1536), zeros(1536), 1e-5, *lif, T, in_gain=0.5)
    for _ in range(2):
        ops.linear_ln_lif(A1536, W[(384, 1536)], zeros(384), ones(384), zeros(384), 1e-5, *lif, T, in_gain=0.5,
                          residual=res, want_spikes=False)
    for _ in range(2):
        ops.linear_ln_lif(patches, W[(384, 512)], zeros(384), ones(384), zeros(384), 1e-5, *lif, T,
                          t_broadcast=True)
    del A1536
    B, H = 256, 8
    q, k, v = spk(T * B, 256, D), spk(T * B, 256, D), spk(T * B, 256, D)
    for _ in range(2):
        ops.ssa(q, k, v, T, B, H, 1, 0.125, 0.5, 0.5, 0.0, in_gain=0.5)
    qd = spk(T * B, 64, D)
    for _ in range(2):
        ops.ssa(qd, k, v, T, B, H, 1, 0.125, 0.5, 0.5, 0.0, in_gain=0.5)
    kd, vd = spk(T * B, 64, D), spk(T * B, 64, D)
    for _ in range(2):
        ops.ssa(qd, kd, vd, T, B, H, 1, 0.125, 0.5, 0.5, 0.0, in_gain=0.5, causal=True)
    torch.cuda.synchronize()


def bench_lnlif(iters, R=16384, T=4):
    """LayerNorm->LIF training kernels (``ops.ln_lif_fwd`` / ``ops.ln_lif_bwd``)
    at the encoder shapes of 64 images per GPU: R tokens x T rows, bf16
    pre-activation with the folded bias. Cases: D = 384 and 1536 with bf16
    spikes and gradient (the MLP hidden layer and the plain row-major form),
    D = 384 with head-major spikes and gradient [T*B, 8, 256, 48] (Q, K, V),
    and D = 384 with fp32 spikes and gradient (spikes that join the residual
    stream). Algorithmic bytes: forward pre + spikes + the row statistics,
    backward pre + gradient + g_pre + the statistics; every input rotates
    over three copies, 150 MB or more per set."""
    res = []
    g = torch.Generator(device="cuda").manual_seed(0)
    cases = ((384, torch.bfloat16, None), (1536, torch.bfloat16, None), (384, torch.bfloat16, (48, 256)),
             (384, torch.float32, None))
    for D, sdt, heads in cases:
        copies = 3
        pres = [torch.randn(T * R, D, device="cuda", generator=g).to(torch.bfloat16) for _ in range(copies)]
        gshape = (T * R // heads[1], D // heads[0], heads[1], heads[0]) if heads else (T * R, D)
        gss = [torch.randn(gshape, device="cuda", generator=g).to(sdt) for _ in range(copies)]
        gamma, beta = torch.ones(D, device="cuda"), torch.zeros(D, device="cuda")
        bias = torch.zeros(D, device="cuda")
        lif = torch.tensor([0.5, 1.0, 0.0], device="cuda")
        stats = ops.ln_lif_fwd(pres[0], gamma, beta, 1e-5, lif[0:1], lif[1:2], lif[2:3], T, in_gain=0.5,
                               spike_dtype=sdt, bias=bias, heads=heads)[1]
        fms = _time(lambda i: ops.ln_lif_fwd(pres[i % copies], gamma, beta, 1e-5, lif[0:1], lif[1:2], lif[2:3], T,
                                             in_gain=0.5, spike_dtype=sdt, bias=bias, heads=heads), iters)
        bms = _time(lambda i: ops.ln_lif_bwd(gss[i % copies], pres[i % copies], stats, gamma, beta, lif[0:1],
                                             lif[1:2], lif[2:3], T, 0.5, "arctan", 2.0, bias=bias, need_bias=True,
                                             heads=heads), iters)
        el, rows, es = T * R * D, T * R, torch.finfo(sdt).bits // 8
        fbytes = el * (2 + es) + rows * 8
        bbytes = el * (2 + es + 2) + rows * 8
        tag = "D=%d %s%s" % (D, str(sdt).replace("torch.", ""), " head-major" if heads else "")
        res.append({"kernel": "ln_lif_fwd", "case": tag, "rows": rows, "D": D, "us": fms * 1e3,
                    "GB/s": fbytes / fms / 1e6})
        res.append({"kernel": "ln_lif_bwd", "case": tag, "rows": rows, "D": D, "us": bms * 1e3,
                    "GB/s": bbytes / bms / 1e6})
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default=None,
                    choices=["lif", "gemm", "ssa", "ssa_model", "train_gemm", "cnn", "attn_train", "data", "shapes",
                             "lnlif"])
    ap.add_argument("--ssa-batch", type=int, default=256, help="images for --only ssa_model")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--tokens", type=int, default=32 * 256, help="tokens per step for the gemm shapes")
    ap.add_argument("--lif-neurons", type=int, default=64 * 256 * 1536, help="neurons per step for the LIF scan")
    a = ap.parse_args()
    if a.only == "shapes":
        bench_shapes_once()
        ops.device_error_check()
        print(json.dumps({"shapes": "done"}))
        return
    peaks, src = _peaks()
    out = {"peaks": {"hbm_gbs": peaks.get("hbm_gbs"), "bf16_tflops_sustained": peaks.get("bf16_tflops_sustained"),
                     "source": src}, "results": []}
    if a.only in (None, "lif"):
        for r in bench_lif(a.iters, N=a.lif_neurons):
            r["frac_hbm"] = r["GB/s"] / peaks["hbm_gbs"]
            out["results"].append(r)
    if a.only in (None, "gemm"):
        for n, k in ((1536, 384), (384, 384), (384, 1536)):
            r = bench_gemm(a.iters, N=n, K=k, R=a.tokens)
            r["frac_tensor"] = r["TFLOP/s"] / peaks["bf16_tflops_sustained"]
            out["results"].append(r)
    if a.only == "attn_train":
        for r in bench_attn_train(a.iters):
            out["results"].append(r)
    if a.only == "cnn":
        for r in bench_cnn(a.iters):
            out["results"].append(r)
    if a.only == "train_gemm":
        for r in bench_train_gemm(a.iters):
            out["results"].append(r)
    if a.only == "ssa_model":
        # the three attention calls of the forward at the bench batch: encoder
        # self (256 x 256), decoder cross (64 x 256), decoder self (64 x 64,
        # dense look-ahead mask), XNOR form
        for N, Nk, dm in ((256, 256, False), (64, 256, False), (64, 64, True)):
            r = bench_ssa(a.iters, 1, N=N, Nk=Nk, B=a.ssa_batch, dense_mask=dm)
            r["frac_hbm"] = r["GB/s"] / peaks["hbm_gbs"]
            out["results"].append(r)
    if a.only in (None, "ssa"):
        for variant in (0, 1):
            out["results"].append(bench_ssa(a.iters, variant))
        out["results"].append(bench_ssa(a.iters, 0, N=64, causal=True))
        for r in bench_n_major(a.iters):
            r["frac_hbm"] = r["GB/s"] / peaks["hbm_gbs"]
            out["results"].append(r)
    if a.only in (None, "lnlif"):
        for r in bench_lnlif(a.iters):
            r["frac_hbm"] = r["GB/s"] / peaks["hbm_gbs"]
            out["results"].append(r)
    if a.only in (None, "data"):
        for r in bench_data(a.iters):
            r["frac_hbm"] = r["GB/s"] / peaks["hbm_gbs"]
            out["results"].append(r)
    ops.device_error_check()
    print(json.dumps(out))


if __name__ == "__main__":
    main()
