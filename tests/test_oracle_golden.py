"""The CPU oracle against the golden fixtures made from the reference itself.

These pin the oracle: every fixture in ``tests/golden`` was produced by the
reference modules (``tests/golden/make_golden.py``), with the reference's
Triton LIF kernels executed by the Triton interpreter.
"""

import os

import pytest
import torch

import oracle
from oracle import modules as om
from parity import assert_spikes_match, assert_close_rel, membrane_history


def load(golden_dir, name):
    return torch.load(os.path.join(golden_dir, name), weights_only=False)


def test_lif_forward_bit_exact(golden_dir):
    for c in load(golden_dir, "lif.pt"):
        s, vf = oracle.lif_forward(c["x_in"], c["beta"], c["v_th"], c["v_reset"])
        assert torch.equal(s, c["spikes"]), c["dtype"]
        assert torch.equal(vf, c["v_final"]), c["dtype"]


def test_lif_forward_gain_equals_prescaled_input(golden_dir):
    # tau=2 neuron: beta .5 with in_gain .5 on x equals the reference fed 0.5*x
    for c in load(golden_dir, "lif.pt"):
        if c["scale"] != 0.5:
            continue
        s, vf = oracle.lif_forward(c["x"], c["beta"], c["v_th"], c["v_reset"], in_gain=0.5)
        assert torch.equal(s, c["spikes"])
        assert torch.equal(vf, c["v_final"])


def test_lif_backward(golden_dir):
    for c in load(golden_dir, "lif.pt"):
        dt = c["x_in"].dtype
        gx, gb = oracle.lif_backward(c["g_spikes"], None, c["x_in"], c["spikes"], c["beta"],
                                     c["v_th"], c["v_reset"], 4.0)
        assert torch.equal(gx.to(dt), c["grad_x"].to(dt))
        assert torch.allclose(gb, c["grad_beta"], rtol=1e-5, atol=1e-5)
        gx, gb = oracle.lif_backward(c["g_spikes"], c["g_vfinal"], c["x_in"], c["spikes"],
                                     c["beta"], c["v_th"], c["v_reset"], 4.0)
        assert torch.equal(gx.to(dt), c["grad_x_vf"].to(dt))
        assert torch.allclose(gb, c["grad_beta_vf"], rtol=1e-5, atol=1e-5)


def test_lif_module(golden_dir):
    for c in load(golden_dir, "lif_module.pt"):
        m = om.LIF(beta=0.8, v_th=0.9, n_steps=3, learn_beta=c["learn_beta"])
        m.load_state_dict(c["state"])
        s, vf = m(c["x"])
        assert torch.equal(s, c["spikes"])
        assert torch.equal(vf, c["v_final"])


def test_lif_module_bad_reshape():
    m = om.LIF(n_steps=3)
    with pytest.raises(RuntimeError):
        m(torch.zeros(4, 5))


def test_log_pe_bias(golden_dir):
    for (nq, nk), ref in load(golden_dir, "logpe.pt").items():
        assert torch.equal(om.log_pe_bias(nq, nk), ref), (nq, nk)


def _ssa_module(c):
    cls = om.SSAMultiHeadAttention if c["variant"] == "xnor" else om.SSAMultiHeadAttention_
    m = cls(d_model=c["D"], n_heads=c["H"], n_steps=c["T"])
    m.load_state_dict(c["state"])
    return m


def test_ssa(golden_dir):
    for c in load(golden_dir, "ssa.pt"):
        m = _ssa_module(c)
        with torch.no_grad():
            y = m(c["query"], c["key"], c["key"], attention_mask=c["mask"])
        T = c["T"]
        ln_o = c["ln_o"].reshape(T, -1)
        vh = membrane_history(ln_o, 0.9, 1.0, 0.0)
        assert_spikes_match(y.reshape(T, -1), c["out"].reshape(T, -1), vh, 1.0,
                            what=f"ssa {c['variant']} {c['case']}")


def test_mlp(golden_dir):
    c = load(golden_dir, "mlp.pt")
    m = om.SpikingMLP(c["D"], c["F"], n_steps=c["T"])
    m.load_state_dict(c["state"])
    with torch.no_grad():
        y = m(c["x"])
        h = m.bn_expand(m.expand(c["x"]))
    assert_close_rel(h, c["ln_expand"], what="ln_expand")
    T = c["T"]
    vh = membrane_history(c["ln_compress"].reshape(T, -1), torch.sigmoid(m.lifcompress.beta_raw), 1.0, 0.0)
    assert_spikes_match(y.reshape(T, -1), c["out"].reshape(T, -1), vh, 1.0, what="mlp")


def test_encoder_decoder(golden_dir):
    c = load(golden_dir, "stacks.pt")
    enc = om.Encoder(2, c["D"], c["H"], c["F"], n_steps=c["T"])
    enc.load_state_dict(c["enc_state"])
    dec = om.Decoder(1, c["D"], c["H"], c["F"], n_steps=c["T"])
    dec.load_state_dict(c["dec_state"])
    with torch.no_grad():
        y = enc(c["x"])
        z = dec(c["tgt"], c["enc_out"], mask=c["mask"])
    assert torch.equal(y, c["enc_out"])
    assert torch.equal(z, c["dec_out"])


def test_seq2seq_cnn(golden_dir):
    c = load(golden_dir, "seq2seq_cnn.pt")
    m = om.Seq2Seq(patch_size=4, d_model=32, n_heads=4, ff_dim=64, num_encoder_layers=1,
                   num_decoder_layers=1, tgt_vocab_size=40, nb_sps_blocks=1, n_steps=c["T"])
    m.load_state_dict(c["state"])
    m.eval()
    with torch.no_grad():
        logits, aux = m(c["src"], c["tgt"], look_ahead_mask=c["mask"])
        enc, _ = m.encode(c["src"])
    assert aux is None
    assert torch.equal(enc, c["enc"])
    assert_close_rel(logits, c["logits"], tol=1e-5, what="logits")
