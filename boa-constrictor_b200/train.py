"""Training-side evaluation (train.py:9-22): bits per byte of a model over a
loader of byte sequences, through the model's forward pass.

BoaBytePredictor.forward runs the fused sm_100a kernel in logits mode with
time blocks of 4 positions (the same kernel and weight tiles as compression),
so evaluation costs one launch per batch instead of one per byte.  Training
itself (train.py:24 onwards) is out of scope for this build and raises.
"""
from __future__ import annotations

import math

import torch


@torch.inference_mode()
def evaluate_bpp(model, loader, criterion, device="cuda", vocab_size=256) -> float:
    """Mean next-byte negative log-likelihood over every position of every
    batch, in bits: each batch [B, L] predicts bytes 1..L-1 from 0..L-2."""
    model.eval()
    nll_sum = 0.0
    count = 0
    for batch in loader:
        inputs = batch[:, :-1].to(device)
        targets = batch[:, 1:].to(device)
        logits = model(inputs)                             # [B, L-1, vocab]
        loss = criterion(logits.reshape(-1, vocab_size), targets.reshape(-1).long())
        nll_sum += float(loss.item()) * targets.numel()
        count += targets.numel()
    return nll_sum / max(count, 1) / math.log(2.0)


def train(*args, **kwargs):
    raise NotImplementedError("training (train.py:24-) is not part of the compress/decompress hot path; "
                              "train with the reference code and load the state_dict here")
