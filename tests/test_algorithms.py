"""Scheduler, sampler, GRPO and HiF8 math vs the reference's formulas (CPU)."""
import math

import numpy as np
import pytest
import torch

from osp_next_b200.ops import reference as ref
from osp_next_b200.rl import grpo
from osp_next_b200.schedulers.flow_matching import FlowMatchingScheduler


def test_sigma_schedules_match_reference(reference):
    _, fm = reference
    for kw in (dict(num_inference_steps=50, shift=5.0), dict(num_inference_steps=8, shift=1.0)):
        a = fm.FlowMatchingScheduler(**kw)._set_sigmas(training=False)
        b = FlowMatchingScheduler(**kw)._set_sigmas(training=False)
        assert torch.allclose(a, b)
    kw = dict(use_dynamic_shifting=True, use_logitnorm_time_sampling=True)
    torch.manual_seed(0)
    a = fm.FlowMatchingScheduler(**kw)._set_sigmas(batch_size=4, image_seq_len=4000)
    torch.manual_seed(0)
    b = FlowMatchingScheduler(**kw)._set_sigmas(batch_size=4, image_seq_len=4000)
    assert torch.allclose(a, b)


def test_sampling_loop_matches_reference(reference):
    _, fm = reference

    class Toy(torch.nn.Module):
        def forward(self, x, t, text, **k):
            return torch.sin(x) * (t.view(-1, 1, 1, 1, 1) / 1000) + text.mean(dim=(1, 2)).view(-1, 1, 1, 1, 1)

    lat = torch.randn(1, 4, 2, 4, 4)
    pe, ne = torch.randn(1, 3, 8), torch.randn(1, 3, 8)
    a = fm.FlowMatchingScheduler(num_inference_steps=6, guidance_scale=5.0, shift=3.0).sample(
        Toy(), lat.clone(), prompt_embeds=pe, negative_prompt_embeds=ne)
    b = FlowMatchingScheduler(num_inference_steps=6, guidance_scale=5.0, shift=3.0).sample(
        Toy(), lat.clone(), prompt_embeds=pe, negative_prompt_embeds=ne)
    assert torch.allclose(a, b, atol=1e-5)


def test_sde_logprob_formula():
    torch.manual_seed(0)
    sig = grpo.shifted_sigmas(10, 1.0)
    x, v = torch.randn(2, 4, 2, 4, 4), torch.randn(2, 4, 2, 4, 4)
    noise = torch.randn_like(x)
    prev, lp, mean, sd = grpo.sde_step_with_logprob(sig, v, 3, x, 10, noise=noise)
    s, dt = sig[3], sig[4] - sig[3]
    std = sig[-1] + (sig[0] - sig[-1]) * s
    m = x * (1 + std ** 2 / (2 * s) * dt) + v * (1 + std ** 2 * (1 - s) / (2 * s)) * dt
    assert torch.allclose(mean, m, atol=1e-6)
    assert torch.allclose(prev, m + std * torch.sqrt(-dt) * noise, atol=1e-6)
    want = (-((prev - m) ** 2) / (2 * (std * torch.sqrt(-dt)) ** 2) - torch.log(std * torch.sqrt(-dt))
            - math.log(math.sqrt(2 * math.pi))).mean(dim=(1, 2, 3, 4))
    assert torch.allclose(lp, want, atol=1e-5)


def test_stat_tracker_and_loss():
    tr = grpo.PerPromptStatTracker()
    adv = tr.update(["a", "a", "b", "b"], [1.0, 3.0, 0.0, 0.0])
    assert np.allclose(adv[:2], [-1 / (1 + 1e-4), 1 / (1 + 1e-4)], atol=1e-3) and np.allclose(adv[2:], 0)
    lp = torch.tensor([0.1, -0.2], requires_grad=True)
    loss, info = grpo.grpo_loss(lp, torch.zeros(2), torch.tensor([1.0, -1.0]), clip_range=0.05, adv_clip_max=5)
    loss.backward()
    assert lp.grad is not None and float(info["clipfrac"]) == 1.0
    assert grpo.calculate_zero_std_ratio(["a", "a", "b"], np.array([1.0, 1.0, 2.0])) == 1.0


def test_hif8_kernel_semantics_vs_torch_oracle():
    """Kernel-semantics restatement vs the reference's torch formula: they differ only
    where the reference's log2 rounds up just below a power of two, below 2^-23, or ≥ 40960."""
    x = torch.randn(1 << 16) * torch.exp(torch.randn(1 << 16) * 3)
    a = ref.hif8_round(x)
    b = ref.hif8_round_torch_oracle(x)
    diff = ~torch.isclose(a, b, rtol=0, atol=0)
    ax = x.abs()
    explained = (ax < 2 ** -23) | (ax >= 40960)
    l2 = torch.log2(ax)
    explained |= (torch.floor(l2) != torch.floor(torch.log2(ax.double())).float())
    assert bool((~diff | explained).all())
    assert diff.float().mean() < 1e-3
    # grid check: three mantissa bits near 1
    assert ref.hif8_round(torch.tensor([1.0625, 1.19, 3.3]))[:2].tolist() == [1.125, 1.25]


def test_hif8_linear_ste_grads():
    from osp_next_b200.quant.hif8 import HIF8Linear
    torch.manual_seed(0)
    lin = HIF8Linear(16, 8)
    x = torch.randn(4, 16, requires_grad=True)
    y = lin(x)
    y.sum().backward()
    assert x.grad is not None and lin.weight.grad is not None
    assert torch.allclose(y, torch.nn.functional.linear(x, lin.weight, lin.bias), atol=0.3)
