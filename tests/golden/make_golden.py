"""Generate the golden fixtures in this folder from the reference implementation.

Runs the reference ``Triton_Layers`` modules of flofiz/SpikingTransformer
(imported from a local checkout given by ``--ref`` or the
``SPK_REFERENCE`` environment variable) on seeded inputs
and stores inputs, state dicts, intermediate tensors and outputs as small
``.pt`` files.  The reference LIF kernels (``Lif.py:108-276``) are Triton
kernels behind an autotuner that needs a GPU; here they run under the Triton
interpreter (``TRITON_INTERPRET=1``) with the autotuner bypassed at its
smallest configuration (``BLOCK_SIZE_N=128``, ``Lif.py:110``).  Everything
else in the reference is stock torch and runs as-is on the CPU in fp32.

Linear weights are rounded to bf16 before the reference runs (the benchmark
model uses bf16 weights, and the CUDA kernels consume bf16 weights), so the
fixtures pin the reference's fp32 arithmetic on bf16-representable weights.

Usage:  python tests/golden/make_golden.py --ref <reference checkout>
"""

import argparse
import os
import sys

os.environ.setdefault("TRITON_INTERPRET", "1")

import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))


class _DirectLaunch:
    """Replaces an autotuned kernel object: ``k[grid](*args)`` launches the
    underlying jitted function with BLOCK_SIZE_N=128 (autotuning needs a GPU)."""

    def __init__(self, autotuned):
        self.fn = autotuned.fn

    def __getitem__(self, grid):
        return lambda *a: self.fn[grid](*a, BLOCK_SIZE_N=128)


def load_reference(path):
    sys.path.insert(0, path)
    import Triton_Layers.Lif as L
    import Triton_Layers.SSA as S
    import Triton_Layers.SpikingMLP as M
    import Triton_Layers.Encoder as E
    import Triton_Layers.Decoder as D
    import Triton_Layers.Seq2Seq as Q
    L.lif_forward_kernel = _DirectLaunch(L.lif_forward_kernel)
    L.lif_backward_kernel = _DirectLaunch(L.lif_backward_kernel)
    return dict(L=L, S=S, M=M, E=E, D=D, Q=Q)


def round_linear_weights_bf16(module):
    for m in module.modules():
        if isinstance(m, torch.nn.Linear):
            m.weight.data = m.weight.data.to(torch.bfloat16).to(torch.float32)


def perturb_layernorms(module, gen):
    for m in module.modules():
        if isinstance(m, torch.nn.LayerNorm):
            m.weight.data = 1.0 + 0.1 * torch.randn(m.weight.shape, generator=gen)
            m.bias.data = 0.1 * torch.randn(m.bias.shape, generator=gen)


def capture_inputs(module, names):
    """Forward pre-hooks recording the first positional input of submodules."""
    store = {}
    handles = []
    for name in names:
        sub = module.get_submodule(name)

        def hook(mod, args, _name=name):
            store.setdefault(_name, []).append(args[0].detach().clone())
        handles.append(sub.register_forward_pre_hook(hook))
    return store, handles


def spikes_input(gen, shape, p=0.3, max_count=1):
    x = torch.zeros(shape)
    for _ in range(max_count):
        x += (torch.rand(shape, generator=gen) < p).float()
    return x


def make_lif(ref):
    L = ref["L"]
    cases = []
    specs = [
        # (T, B, F, beta, v_th, v_reset, dtype, input scale)
        (4, 8, 300, 0.9, 1.0, 0.0, torch.float32, 1.0),
        (4, 2, 4096, 0.5, 1.0, 0.0, torch.float32, 0.5),  # tau=2 neuron (beta .5, gain .5)
        (1, 3, 17, 0.9, 1.0, 0.0, torch.float32, 1.0),
        (7, 3, 129, 0.8, 0.7, -0.2, torch.float32, 1.0),
        (4, 5, 260, 0.9, 0.5, 0.0, torch.float16, 1.0),
    ]
    for i, (T, B, F, beta, vth, vr, dt, scale) in enumerate(specs):
        g = torch.Generator().manual_seed(100 + i)
        x = torch.randn(T, B, F, generator=g) + 0.5
        x_in = (x * scale).to(dt).requires_grad_(True)
        gs = torch.randn(T, B, F, generator=g)
        gvf = torch.randn(B, F, generator=g)
        b = torch.tensor(beta)
        s, vf = L.LIFLayer.apply(x_in, b, torch.tensor(vth), torch.tensor(vr), 4.0)
        # grad through spikes and v_final (Lif.py:46-102)
        b.requires_grad_(True)
        x_in2 = x_in.detach().clone().requires_grad_(True)
        s2, vf2 = L.LIFLayer.apply(x_in2, b, torch.tensor(vth), torch.tensor(vr), 4.0)
        (s2 * gs).sum().backward(retain_graph=True)
        cases.append(dict(T=T, B=B, F=F, beta=beta, v_th=vth, v_reset=vr, dtype=str(dt),
                          x=x, scale=scale, x_in=x_in.detach(), g_spikes=gs, g_vfinal=gvf,
                          spikes=s.detach(), v_final=vf.detach(),
                          grad_x=x_in2.grad.detach(), grad_beta=b.grad.detach()))
        # second backward: including a v_final gradient
        b2 = torch.tensor(beta, requires_grad=True)
        x_in3 = x_in.detach().clone().requires_grad_(True)
        s3, vf3 = L.LIFLayer.apply(x_in3, b2, torch.tensor(vth), torch.tensor(vr), 4.0)
        ((s3 * gs).sum() + (vf3 * gvf).sum()).backward()
        cases[-1]["grad_x_vf"] = x_in3.grad.detach()
        cases[-1]["grad_beta_vf"] = b2.grad.detach()
    torch.save(cases, os.path.join(HERE, "lif.pt"))


def make_lif_module(ref):
    L = ref["L"]
    g = torch.Generator().manual_seed(7)
    out = []
    for learn_beta in (False, True):
        torch.manual_seed(11)
        m = L.LIF(beta=0.8, v_th=0.9, n_steps=3, learn_beta=learn_beta)
        x = torch.randn(6, 5, 7, generator=g) + 0.4
        s, vf = m(x)
        out.append(dict(learn_beta=learn_beta, state=m.state_dict(), x=x,
                        spikes=s.detach(), v_final=vf.detach()))
    torch.save(out, os.path.join(HERE, "lif_module.pt"))


def make_logpe(ref):
    m = ref["S"].SSAMultiHeadAttention(8, 2, n_steps=1)
    pairs = [(256, 256), (64, 64), (64, 256), (1, 1), (1, 5), (300, 7), (2, 2), (65, 33)]
    out = {}
    for nq, nk in pairs:
        out[(nq, nk)] = m.get_log_pe_bias_cross(nq, nk, "cpu").clone()
    torch.save(out, os.path.join(HERE, "logpe.pt"))


def make_ssa(ref):
    S = ref["S"]
    T, B, D, H = 2, 2, 32, 4
    out = []
    cases = [(v, c) for v in ("xnor", "plain") for c in ("self", "self_causal", "cross")]
    for idx, (variant, case) in enumerate(cases):
        g = torch.Generator().manual_seed(200 + idx)
        torch.manual_seed(3)
        cls = S.SSAMultiHeadAttention if variant == "xnor" else S.SSAMultiHeadAttention_
        m = cls(d_model=D, n_heads=H, n_steps=T)
        round_linear_weights_bf16(m)
        perturb_layernorms(m, g)
        Nq = 12 if case != "cross" else 8
        Nk = 12
        q = spikes_input(g, (T * B, Nq, D), 0.3, 3)
        kv = q if case != "cross" else spikes_input(g, (T * B, Nk, D), 0.3, 3)
        mask = None
        if case == "self_causal":
            tri = torch.tril(torch.ones(Nq, Nq))
            pad = torch.ones(B, 1, 1, Nq)
            pad[1, :, :, -2:] = 0.0
            mask = torch.minimum(pad, tri).unsqueeze(0).repeat(T, 1, 1, 1, 1).reshape(T * B, 1, Nq, Nq)
        store, hs = capture_inputs(m, ["lifq", "lifk", "lifv", "lifs", "lifo"])
        with torch.no_grad():
            y = m(q, kv, kv, attention_mask=mask)
        for h in hs:
            h.remove()
        out.append(dict(variant=variant, case=case, T=T, B=B, D=D, H=H, Nq=Nq, Nk=Nk,
                        state=m.state_dict(), query=q, key=kv, mask=mask, out=y,
                        ln_q=store["lifq"][0], ln_k=store["lifk"][0], ln_v=store["lifv"][0],
                        attn=store["lifs"][0], ln_o=store["lifo"][0]))
    torch.save(out, os.path.join(HERE, "ssa.pt"))


def make_mlp(ref):
    M = ref["M"]
    T, B, N, D, F = 2, 2, 6, 32, 128
    g = torch.Generator().manual_seed(21)
    torch.manual_seed(5)
    m = M.SpikingMLP(D, F, n_steps=T)
    round_linear_weights_bf16(m)
    perturb_layernorms(m, g)
    x = spikes_input(g, (T * B, N, D), 0.3, 4)
    store, hs = capture_inputs(m, ["lifexpand", "lifcompress"])
    with torch.no_grad():
        y = m(x)
    for h in hs:
        h.remove()
    torch.save(dict(T=T, B=B, N=N, D=D, F=F, state=m.state_dict(), x=x, out=y,
                    ln_expand=store["lifexpand"][0], ln_compress=store["lifcompress"][0]),
               os.path.join(HERE, "mlp.pt"))


def make_stacks(ref):
    E, D = ref["E"], ref["D"]
    T, B, N, Dm, H, F = 2, 2, 8, 32, 4, 64
    g = torch.Generator().manual_seed(31)
    torch.manual_seed(9)
    enc = E.Encoder(2, Dm, H, F, n_steps=T)
    round_linear_weights_bf16(enc)
    perturb_layernorms(enc, g)
    x = spikes_input(g, (T * B, N, Dm), 0.3, 1)
    with torch.no_grad():
        y = enc(x)
    torch.manual_seed(10)
    dec = D.Decoder(1, Dm, H, F, n_steps=T)
    round_linear_weights_bf16(dec)
    perturb_layernorms(dec, g)
    Nt = 5
    yt = spikes_input(g, (T * B, Nt, Dm), 0.3, 1)
    mask = torch.tril(torch.ones(Nt, Nt)).expand(T * B, 1, Nt, Nt).contiguous()
    with torch.no_grad():
        z = dec(yt, y, mask=mask)
    torch.save(dict(T=T, B=B, N=N, D=Dm, H=H, F=F, enc_state=enc.state_dict(), x=x, enc_out=y,
                    dec_state=dec.state_dict(), tgt=yt, mask=mask, dec_out=z),
               os.path.join(HERE, "stacks.pt"))


def make_seq2seq(ref):
    Q = ref["Q"]
    T = 2
    g = torch.Generator().manual_seed(41)
    torch.manual_seed(13)
    m = Q.Seq2Seq(patch_size=4, d_model=32, n_heads=4, ff_dim=64, num_encoder_layers=1,
                  num_decoder_layers=1, tgt_vocab_size=40, nb_sps_blocks=1, n_steps=T)
    round_linear_weights_bf16(m)
    m.eval()
    src = torch.rand(2, 1, 32, 64, generator=g)
    tgt = torch.randint(0, 40, (2, 6), generator=g)
    mask = torch.minimum(torch.ones(2, 1, 1, 6), torch.tril(torch.ones(6, 6)))
    with torch.no_grad():
        logits, _ = m(src, tgt, look_ahead_mask=mask)
        enc, _ = m.encode(src)
    torch.save(dict(T=T, state=m.state_dict(), src=src, tgt=tgt, mask=mask, logits=logits, enc=enc),
               os.path.join(HERE, "seq2seq_cnn.pt"))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("SPK_REFERENCE"),
                    help="checkout of flofiz/SpikingTransformer (default: $SPK_REFERENCE)")
    args = ap.parse_args()
    if not args.ref:
        ap.error("give the reference checkout with --ref or SPK_REFERENCE")
    torch.set_num_threads(1)
    ref = load_reference(args.ref)
    make_lif(ref)
    make_lif_module(ref)
    make_logpe(ref)
    make_ssa(ref)
    make_mlp(ref)
    make_stacks(ref)
    make_seq2seq(ref)
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".pt"):
            print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()
