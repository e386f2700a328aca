"""The reference's own test suite (tests/test_attention.py of the reference
project, 13 tests) re-run against this package on the GPU: same shapes,
same assertions, tensors on cuda:0."""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


class TestTanhNorm:
    def test_zero_input(self, ms):
        out = ms.TanhNorm()(torch.zeros(2, 4, device=DEV))
        assert out.shape == (2, 4)
        assert torch.allclose(out, torch.zeros_like(out))

    def test_magnitude_bounded(self, ms):
        out = ms.TanhNorm()(torch.randn(8, 16, device=DEV) * 100)
        assert (out.norm(dim=-1) <= 1.0 + 1e-5).all()

    def test_direction_preserved(self, ms):
        x = torch.randn(4, 8, device=DEV)
        out = ms.TanhNorm()(x)
        assert torch.allclose(torch.nn.functional.normalize(x, dim=-1),
                              torch.nn.functional.normalize(out, dim=-1), atol=1e-5)


class TestScreeningAttention:
    B, T, d = 2, 16, 64

    def attn(self, ms, **kw):
        return ms.ScreeningAttention(d_model=self.d, num_heads=4, **kw).to(DEV)

    def test_output_shape(self, ms):
        x = torch.randn(self.B, self.T, self.d, device=DEV)
        assert self.attn(ms)(x, x, x).shape == (self.B, self.T, self.d)

    def test_causal_masking(self, ms):
        attn = self.attn(ms, causal=True)
        x = torch.randn(1, self.T, self.d, device=DEV)
        x2 = x.clone()
        x2[0, -1] = torch.randn(self.d, device=DEV)
        assert torch.allclose(attn(x, x, x)[0, 0], attn(x2, x2, x2)[0, 0], atol=1e-5)

    def test_key_padding_mask(self, ms):
        x = torch.randn(self.B, self.T, self.d, device=DEV)
        mask = torch.zeros(self.B, self.T, dtype=torch.bool, device=DEV)
        mask[:, -4:] = True
        assert self.attn(ms)(x, x, x, key_padding_mask=mask).shape == (self.B, self.T, self.d)

    def test_non_causal(self, ms):
        x = torch.randn(self.B, self.T, self.d, device=DEV)
        assert self.attn(ms, causal=False)(x, x, x).shape == (self.B, self.T, self.d)

    def test_different_q_k_lengths(self, ms):
        q = torch.randn(self.B, 8, self.d, device=DEV)
        kv = torch.randn(self.B, 20, self.d, device=DEV)
        assert self.attn(ms, causal=False)(q, kv, kv).shape == (self.B, 8, self.d)


class TestMultiscreenBlock:
    def test_output_shape(self, ms):
        x = torch.randn(2, 16, 64, device=DEV)
        assert ms.MultiscreenBlock(d_model=64, num_heads=4).to(DEV)(x).shape == x.shape

    def test_residual_gradient_flow(self, ms):
        block = ms.MultiscreenBlock(d_model=64, num_heads=4).to(DEV)
        x = torch.randn(2, 16, 64, device=DEV, requires_grad=True)
        block(x).sum().backward()
        assert x.grad is not None


class TestMultiscreenLM:
    def model(self, ms):
        return ms.MultiscreenLM(vocab_size=100, d_model=64, num_heads=4, num_layers=2,
                                max_seq_len=64).to(DEV)

    def test_forward_logits_shape(self, ms):
        ids = torch.randint(0, 100, (2, 16), device=DEV)
        assert self.model(ms)(ids)["logits"].shape == (2, 16, 100)

    def test_loss_computation(self, ms):
        ids = torch.randint(0, 100, (2, 16), device=DEV)
        labels = ids.clone()
        labels[:, :4] = -100
        out = self.model(ms)(ids, labels=labels)
        assert "loss" in out and out["loss"].ndim == 0

    def test_generate(self, ms):
        prompt = torch.randint(0, 100, (1, 4), device=DEV)
        assert self.model(ms).generate(prompt, max_new_tokens=8).shape == (1, 12)
