"""Fused LM cross-entropy (screen_cross_entropy_fwd / _bwd) against
F.cross_entropy on the same bf16 logits upcast to fp32 (what autocast does
for the reference's loss, multiscreen/model.py:103-107): the mean loss
within 1e-4 relative, the logits gradient within 2e-2 (bf16 output)."""
import importlib

import pytest
import torch
import torch.nn.functional as F

from tests.conftest import rel_err

pytestmark = pytest.mark.gpu
FN = importlib.import_module("pytorch-implementation-of-screening-attention_b200.functional")


@pytest.mark.parametrize("N,V,pad", [(64, 104, 0), (300, 50257, 47), (1, 8, 0), (257, 4096, 64)])
def test_cross_entropy_matches_torch(cuda, N, V, pad):
    g = torch.Generator(device=cuda).manual_seed(N + V)
    logits = (3.0 * torch.randn(N, V + pad, device=cuda, generator=g)).to(torch.bfloat16)
    if pad:
        logits[:, V:] = float("-inf")
    labels = torch.randint(0, V, (N,), device=cuda, generator=g)
    labels[1::7] = -100
    a = logits.clone().requires_grad_(True)
    loss = FN.cross_entropy(a, labels)
    dmean = torch.tensor(1.7, device=cuda)
    (loss * dmean).backward()
    b = logits.float().clone().requires_grad_(True)
    ref = F.cross_entropy(b, labels, ignore_index=-100)
    (ref * dmean).backward()
    assert rel_err(loss.float().view(1), ref.view(1)) <= 1e-4
    assert rel_err(a.grad.float(), b.grad) <= 2e-2
    assert torch.isfinite(a.grad.float()).all()


def test_cross_entropy_all_ignored_is_nan_like_torch(cuda):
    logits = torch.randn(4, 16, device=cuda).to(torch.bfloat16)
    labels = torch.full((4,), -100, device=cuda)
    assert torch.isnan(FN.cross_entropy(logits, labels))
    assert torch.isnan(F.cross_entropy(logits.float(), labels, ignore_index=-100))


def test_cross_entropy_flags_out_of_range_labels(cuda, ms):
    """A label outside [0, V) that is not ignore_index: F.cross_entropy stops
    with a device assert; the fused kernel gives the row loss 0, leaves it out
    of the mean and raises the device status word instead."""
    ms._lib.device_status(clear=True)
    g = torch.Generator(device=cuda).manual_seed(5)
    logits = torch.randn(6, 32, device=cuda, generator=g).to(torch.bfloat16)
    labels = torch.tensor([3, 40, 7, -5, -100, 0], device=cuda)
    loss = FN.cross_entropy(logits, labels)
    keep = torch.tensor([0, 2, 5], device=cuda)
    ref = F.cross_entropy(logits.float()[keep], labels[keep])
    assert rel_err(loss.float().view(1), ref.view(1)) <= 1e-4
    assert ms._lib.device_status(clear=True) == -1
    # in-range labels leave the status clear
    FN.cross_entropy(logits, labels.clamp(0, 31))
    assert ms._lib.device_status(clear=True) == 0
