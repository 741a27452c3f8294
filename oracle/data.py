"""CPU oracle of the on-device data generator and the training loss (test
infrastructure only).

``synth_text_lines`` restates, with numpy uint64 arithmetic, the counter-based
generator of the synthetic text-line batch: every value is a function of
(seed, image, stream, draw index) through the SplitMix64 finaliser (Steele,
Lea and Flood, 2014), so it reproduces the CUDA generator bit for bit.  The
batch itself stands in for the reference's rendered Wikipedia lines
(``wiki_text_images3.py:173-236``): a U(0, 0.2) background with 5-40 black
rectangles of side 8-20 px per image.

``step_loss`` and ``token_accuracy`` restate the reference's training loss and
metric: ``train_spikeformer.py:309-323`` (the mean over the T steps of
``nn.CrossEntropyLoss(ignore_index=PAD_IDX, label_smoothing=0.1)`` of each
step's logits, the criterion of ``:269``) and ``:84-93`` (the argmax of the
logits averaged over T, ``:556-559``, against the non-pad targets).
"""

import numpy as np
import torch
import torch.nn as nn

_M64 = np.uint64(0xFFFFFFFFFFFFFFFF)
S_BG, S_COUNT, S_RECT, S_TOKEN = 0, 1, 2, 3


def mix64(z):
    """SplitMix64 finaliser on numpy uint64 (wrapping arithmetic)."""
    with np.errstate(over="ignore"):
        z = np.asarray(z, dtype=np.uint64) + np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def draw(seed, b, s, i):
    """Draw(s) ``i`` of stream ``s`` for image ``b``."""
    with np.errstate(over="ignore"):
        key = mix64(np.uint64(seed & 0xFFFFFFFFFFFFFFFF)) ^ (np.uint64(b) * np.uint64(0xD1342543DE82EF95))
        key = key ^ (np.uint64(s) << np.uint64(56))
        return mix64(key ^ np.asarray(i, dtype=np.uint64))


def synth_text_lines(B, seed, H=64, W=1024, L=None, V=256):
    """``([B, 1, H, W] float32 images, [B, L] int64 targets or None)``."""
    img = np.empty((B, 1, H, W), dtype=np.float32)
    idx = np.arange(H * W, dtype=np.uint64)
    for b in range(B):
        u = draw(seed, b, S_BG, idx)
        unit = (u >> np.uint64(40)).astype(np.float32) * np.float32(1.0 / 16777216.0)
        img[b, 0] = (np.float32(0.2) * unit).reshape(H, W)
        n = 5 + int(draw(seed, b, S_COUNT, 0) % np.uint64(36))
        for r in range(n):
            h = 8 + int(draw(seed, b, S_RECT, 4 * r) % np.uint64(13))
            w = 8 + int(draw(seed, b, S_RECT, 4 * r + 1) % np.uint64(13))
            y = int(draw(seed, b, S_RECT, 4 * r + 2) % np.uint64(H - h + 1))
            x = int(draw(seed, b, S_RECT, 4 * r + 3) % np.uint64(W - w + 1))
            img[b, 0, y:y + h, x:x + w] = 0.0
    tok = None
    if L:
        tok = np.empty((B, L), dtype=np.int64)
        for b in range(B):
            tok[b] = (draw(seed, b, S_TOKEN, np.arange(L, dtype=np.uint64)) % np.uint64(V)).astype(np.int64)
    return torch.from_numpy(img), None if tok is None else torch.from_numpy(tok)


def step_loss(logits_steps, tgt_out, ignore_index, label_smoothing):
    """``train_spikeformer.py:309-323`` with the criterion of ``:269``."""
    criterion = nn.CrossEntropyLoss(ignore_index=ignore_index, label_smoothing=label_smoothing)
    loss = 0.0
    for s in range(logits_steps.shape[0]):
        logits = logits_steps[s]
        loss = loss + criterion(logits.reshape(-1, logits.size(-1)), tgt_out.reshape(-1))
    return loss / logits_steps.shape[0]


def token_accuracy(logits, targets, pad_idx):
    """``train_spikeformer.py:84-93`` on the T-averaged logits (``:556-559``)."""
    preds = torch.argmax(logits, dim=-1)
    mask = targets != pad_idx
    correct = (preds == targets) & mask
    return correct.sum().float() / max(1.0, mask.sum().float())
