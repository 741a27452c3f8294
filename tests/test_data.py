"""On-device data generator and training loss against the CPU oracle
(``oracle/data.py``): the generated batch bit for bit, the fused loss and
token accuracy against the reference's ``step_loss`` / ``compute_token_accuracy``
composition, and its gradient against autograd through that composition."""

import pytest
import torch

from oracle import data as od

DEV = "cuda"


def test_oracle_generator_properties():
    img, tok = od.synth_text_lines(3, seed=7, H=64, W=256, L=10, V=256)
    assert img.shape == (3, 1, 64, 256) and img.dtype == torch.float32
    assert float(img.min()) == 0.0 and float(img.max()) < 0.2
    assert tok.shape == (3, 10) and int(tok.min()) >= 0 and int(tok.max()) < 256
    for b in range(3):
        n = 5 + int(od.draw(7, b, od.S_COUNT, 0) % 36)
        assert 5 <= n <= 40
        assert float((img[b] == 0).float().sum()) >= 64  # at least one 8x8 rectangle
    again, tok2 = od.synth_text_lines(3, seed=7, H=64, W=256, L=10, V=256)
    assert torch.equal(img, again) and torch.equal(tok, tok2)
    other, _ = od.synth_text_lines(3, seed=8, H=64, W=256)
    assert not torch.equal(img, other)


@pytest.mark.gpu
@pytest.mark.parametrize("B,H,W,seed", [(3, 64, 256, 1), (2, 64, 1024, 123456789), (4, 32, 96, 2 ** 63 + 5),
                                         (2, 21, 23, 9)])  # H*W not a multiple of 4: scalar stores
def test_synth_text_lines_bit_exact(B, H, W, seed):
    from spikingtransformer_b200 import ops
    img, tok = ops.synth_text_lines(B, seed, H=H, W=W, L=17, V=256)
    ref_img, ref_tok = od.synth_text_lines(B, seed, H=H, W=W, L=17, V=256)
    assert torch.equal(img.cpu(), ref_img)
    assert torch.equal(tok.cpu(), ref_tok)


@pytest.mark.gpu
@pytest.mark.parametrize("T,B,N,V,dtype,ignore,eps", [
    (4, 8, 64, 256, torch.float32, 0, 0.1),     # the training configuration
    (4, 8, 64, 256, torch.bfloat16, 0, 0.1),
    (3, 5, 7, 100, torch.float32, -100, 0.0),   # V not a multiple of 32, no smoothing
    (1, 2, 33, 40, torch.float32, 3, 0.2),
])
def test_ce_over_t_matches_reference_loss(T, B, N, V, dtype, ignore, eps):
    from spikingtransformer_b200 import ops
    g = torch.Generator().manual_seed(T * 100 + V)
    logits = (torch.randn(T, B, N, V, generator=g) * 3).to(dtype)
    tgt = torch.randint(0, V, (B, N), generator=g)
    if ignore >= 0:
        tgt[0, : N // 2] = ignore  # some ignored positions
    x = logits.float().clone().requires_grad_(True)
    ref_loss = od.step_loss(x, tgt, ignore, eps)
    ref_loss.backward()
    ref_acc = od.token_accuracy(x.detach().mean(dim=0), tgt, ignore)
    xd = logits.to(DEV).requires_grad_(True)
    loss, acc, bad = ops.ce_over_t(xd, tgt.to(DEV), ignore_index=ignore, label_smoothing=eps)
    loss.backward()
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    assert abs(float(loss) - float(ref_loss)) <= tol * max(1.0, abs(float(ref_loss)))
    assert abs(float(acc) - float(ref_acc)) < 1e-6
    assert int(bad) == 0
    gref = x.grad
    gk = xd.grad.float().cpu()
    assert (gk - gref).abs().max().item() <= tol * gref.abs().max().item()


@pytest.mark.gpu
def test_ce_over_t_flags_bad_target():
    from spikingtransformer_b200 import ops
    logits = torch.randn(2, 4, 10, device=DEV)
    tgt = torch.tensor([1, 2, 10, 3], device=DEV)  # 10 is outside [0, 10)
    _, _, bad = ops.ce_over_t(logits, tgt, ignore_index=-100)
    assert int(bad) == 1
