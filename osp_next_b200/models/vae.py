"""Wan-2.1 3-D causal VAE (frozen; reference: ospnext/modules/vae.py:18-664).

Same architecture and parameter names as the Wan checkpoint (``encoder.conv1``,
``encoder.downsamples.{i}``, ``encoder.middle``, ``encoder.head``, ``conv1``,
``conv2``, ``decoder.*``), 8× spatial / 4× temporal compression to 16 latent
channels, latents normalised with the per-channel statistics below.

Streaming: video is encoded in chunks of 1, 4, 4, … frames and decoded one
latent frame at a time.  Here every causal convolution keeps its own state (the
last two input frames of the previous chunk) and every temporal resampler keeps
its own first-chunk state, instead of threading cache lists through the call
tree; the chunk schedule and the per-layer caching rules are the reference's, so
chunked and whole-video semantics agree with it.
"""
from __future__ import annotations

import logging
import os
from contextlib import nullcontext
from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

CACHE_T = 2

# latent normalisation constants of the Wan-2.1 VAE (data constants of the checkpoint)
LATENT_MEAN = [-0.7571, -0.7089, -0.9113, 0.1075, -0.1745, 0.9653, -0.1517, 1.5508,
               0.4134, -0.0715, 0.5517, -0.3632, -0.1922, -0.9497, 0.2503, -0.2921]
LATENT_STD = [2.8184, 1.4541, 2.3275, 2.6558, 1.2196, 1.7708, 2.6052, 2.0743,
              3.2687, 2.1526, 2.8652, 1.5579, 1.6382, 1.1253, 2.8251, 1.9160]


class CausalConv3d(nn.Conv3d):
    """Conv3d padded only on the past side in time; streams with a 2-frame state."""

    def __init__(self, *args, **kwargs):
        super().__init__(*args, **kwargs)
        pt, ph, pw = self.padding
        self._pad = (pw, pw, ph, ph, 2 * pt, 0)
        self.padding = (0, 0, 0)
        self.streaming = False
        self._state: Optional[torch.Tensor] = None

    def forward(self, x):
        pad = list(self._pad)
        prev = self._state if self.streaming else None
        if self.streaming:
            keep = x[:, :, -CACHE_T:].clone()
            if keep.shape[2] < CACHE_T and prev is not None:
                keep = torch.cat([prev[:, :, -1:], keep], dim=2)
            self._state = keep
        if prev is not None and pad[4] > 0:
            x = torch.cat([prev.to(x.dtype), x], dim=2)
            pad[4] -= prev.shape[2]
        return super().forward(F.pad(x, pad))


class RMS_norm(nn.Module):
    def __init__(self, dim, channel_first=True, images=True, bias=False):
        super().__init__()
        shape = (dim, *((1, 1) if images else (1, 1, 1))) if channel_first else (dim,)
        self.channel_first = channel_first
        self.scale = dim ** 0.5
        self.gamma = nn.Parameter(torch.ones(shape))
        self.bias = nn.Parameter(torch.zeros(shape)) if bias else 0.0

    def forward(self, x):
        return F.normalize(x, dim=1 if self.channel_first else -1) * self.scale * self.gamma + self.bias


class Upsample(nn.Upsample):
    def forward(self, x):
        return super().forward(x.float()).type_as(x)


def _per_frame(fn, x):
    b, c, t, h, w = x.shape
    y = fn(x.permute(0, 2, 1, 3, 4).reshape(b * t, c, h, w))
    return y.reshape(b, t, *y.shape[1:]).permute(0, 2, 1, 3, 4)


class Resample(nn.Module):
    def __init__(self, dim, mode):
        super().__init__()
        self.dim, self.mode = dim, mode
        if mode == "upsample2d":
            self.resample = nn.Sequential(Upsample(scale_factor=(2.0, 2.0), mode="nearest-exact"),
                                          nn.Conv2d(dim, dim // 2, 3, padding=1))
        elif mode == "upsample3d":
            self.resample = nn.Sequential(Upsample(scale_factor=(2.0, 2.0), mode="nearest-exact"),
                                          nn.Conv2d(dim, dim // 2, 3, padding=1))
            self.time_conv = CausalConv3d(dim, dim * 2, (3, 1, 1), padding=(1, 0, 0))
        elif mode == "downsample2d":
            self.resample = nn.Sequential(nn.ZeroPad2d((0, 1, 0, 1)), nn.Conv2d(dim, dim, 3, stride=(2, 2)))
        elif mode == "downsample3d":
            self.resample = nn.Sequential(nn.ZeroPad2d((0, 1, 0, 1)), nn.Conv2d(dim, dim, 3, stride=(2, 2)))
            self.time_conv = CausalConv3d(dim, dim, (3, 1, 1), stride=(2, 1, 1), padding=(0, 0, 0))
        else:
            self.resample = nn.Identity()
        self.streaming = False
        self._first = True
        self._state: Optional[torch.Tensor] = None

    def reset(self):
        self._first, self._state = True, None
        if hasattr(self, "time_conv"):
            self.time_conv._state = None

    def forward(self, x):
        b, c, t, h, w = x.shape
        if self.mode == "upsample3d" and self.streaming:
            if self._first:                       # first latent frame: no temporal upsampling
                self._first = False
            else:
                keep = x[:, :, -CACHE_T:].clone()
                if keep.shape[2] < CACHE_T:
                    prev = self._state[:, :, -1:] if self._state is not None else torch.zeros_like(keep)
                    keep = torch.cat([prev, keep], dim=2)
                tc = self.time_conv
                tc.streaming, tc._state = True, self._state
                x = tc(x)
                tc.streaming = False
                self._state = keep
                x = x.reshape(b, 2, c, t, h, w)
                x = torch.stack((x[:, 0], x[:, 1]), 3).reshape(b, c, t * 2, h, w)
        x = _per_frame(self.resample, x)
        if self.mode == "downsample3d" and self.streaming:
            if self._first:                       # first chunk (one frame): keep it, no temporal conv
                self._first = False
                self._state = x.clone()
            else:
                keep = x[:, :, -1:].clone()
                x = self.time_conv(torch.cat([self._state[:, :, -1:], x], dim=2))
                self._state = keep
        return x


class ResidualBlock(nn.Module):
    def __init__(self, in_dim, out_dim, dropout=0.0):
        super().__init__()
        self.in_dim, self.out_dim = in_dim, out_dim
        self.residual = nn.Sequential(
            RMS_norm(in_dim, images=False), nn.SiLU(), CausalConv3d(in_dim, out_dim, 3, padding=1),
            RMS_norm(out_dim, images=False), nn.SiLU(), nn.Dropout(dropout), CausalConv3d(out_dim, out_dim, 3, padding=1))
        self.shortcut = CausalConv3d(in_dim, out_dim, 1) if in_dim != out_dim else nn.Identity()

    def forward(self, x):
        return self.residual(x) + self.shortcut(x)


class AttentionBlock(nn.Module):
    """Single-head self-attention over the pixels of each frame."""

    def __init__(self, dim):
        super().__init__()
        self.dim = dim
        self.norm = RMS_norm(dim)
        self.to_qkv = nn.Conv2d(dim, dim * 3, 1)
        self.proj = nn.Conv2d(dim, dim, 1)
        nn.init.zeros_(self.proj.weight)

    def forward(self, x):
        def f(z):
            bt, c, h, w = z.shape
            q, k, v = self.to_qkv(self.norm(z)).reshape(bt, 1, c * 3, h * w).permute(0, 1, 3, 2).chunk(3, dim=-1)
            o = F.scaled_dot_product_attention(q.contiguous(), k.contiguous(), v.contiguous())
            return self.proj(o.squeeze(1).permute(0, 2, 1).reshape(bt, c, h, w))
        return x + _per_frame(f, x)


class Encoder3d(nn.Module):
    def __init__(self, dim=128, z_dim=4, dim_mult=(1, 2, 4, 4), num_res_blocks=2, attn_scales=(),
                 temperal_downsample=(True, True, False), dropout=0.0):
        super().__init__()
        dims = [dim * u for u in [1] + list(dim_mult)]
        scale = 1.0
        self.conv1 = CausalConv3d(3, dims[0], 3, padding=1)
        layers = []
        for i, (din, dout) in enumerate(zip(dims[:-1], dims[1:])):
            for _ in range(num_res_blocks):
                layers.append(ResidualBlock(din, dout, dropout))
                if scale in attn_scales:
                    layers.append(AttentionBlock(dout))
                din = dout
            if i != len(dim_mult) - 1:
                layers.append(Resample(dout, "downsample3d" if temperal_downsample[i] else "downsample2d"))
                scale /= 2.0
        self.downsamples = nn.Sequential(*layers)
        self.middle = nn.Sequential(ResidualBlock(dout, dout, dropout), AttentionBlock(dout),
                                    ResidualBlock(dout, dout, dropout))
        self.head = nn.Sequential(RMS_norm(dout, images=False), nn.SiLU(), CausalConv3d(dout, z_dim, 3, padding=1))

    def forward(self, x):
        return self.head(self.middle(self.downsamples(self.conv1(x))))


class Decoder3d(nn.Module):
    def __init__(self, dim=128, z_dim=4, dim_mult=(1, 2, 4, 4), num_res_blocks=2, attn_scales=(),
                 temperal_upsample=(False, True, True), dropout=0.0):
        super().__init__()
        dims = [dim * u for u in [dim_mult[-1]] + list(dim_mult)[::-1]]
        scale = 1.0 / 2 ** (len(dim_mult) - 2)
        self.conv1 = CausalConv3d(z_dim, dims[0], 3, padding=1)
        self.middle = nn.Sequential(ResidualBlock(dims[0], dims[0], dropout), AttentionBlock(dims[0]),
                                    ResidualBlock(dims[0], dims[0], dropout))
        layers = []
        for i, (din, dout) in enumerate(zip(dims[:-1], dims[1:])):
            if i in (1, 2, 3):
                din = din // 2
            for _ in range(num_res_blocks + 1):
                layers.append(ResidualBlock(din, dout, dropout))
                if scale in attn_scales:
                    layers.append(AttentionBlock(dout))
                din = dout
            if i != len(dim_mult) - 1:
                layers.append(Resample(dout, "upsample3d" if temperal_upsample[i] else "upsample2d"))
                scale *= 2.0
        self.upsamples = nn.Sequential(*layers)
        self.head = nn.Sequential(RMS_norm(dout, images=False), nn.SiLU(), CausalConv3d(dout, 3, 3, padding=1))

    def forward(self, x):
        return self.head(self.upsamples(self.middle(self.conv1(x))))


def _set_streaming(module: nn.Module, on: bool):
    for m in module.modules():
        if isinstance(m, (CausalConv3d, Resample)):
            m.streaming = on
            if isinstance(m, Resample):
                m.reset()
            else:
                m._state = None


class WanVAE_(nn.Module):
    def __init__(self, dim=128, z_dim=4, dim_mult=(1, 2, 4, 4), num_res_blocks=2, attn_scales=(),
                 temperal_downsample=(True, True, False), dropout=0.0):
        super().__init__()
        self.z_dim = z_dim
        self.encoder = Encoder3d(dim, z_dim * 2, dim_mult, num_res_blocks, attn_scales, temperal_downsample, dropout)
        self.conv1 = CausalConv3d(z_dim * 2, z_dim * 2, 1)
        self.conv2 = CausalConv3d(z_dim, z_dim, 1)
        self.decoder = Decoder3d(dim, z_dim, dim_mult, num_res_blocks, attn_scales,
                                 list(temperal_downsample)[::-1], dropout)

    def encode(self, x, scale):
        """x [B,3,1+4k,H,W] in [-1,1] → normalised latent mean [B,z,1+k,H/8,W/8]."""
        _set_streaming(self.encoder, True)
        t = x.shape[2]
        outs = [self.encoder(x[:, :, :1])]
        for i in range(1, 1 + (t - 1) // 4):
            outs.append(self.encoder(x[:, :, 1 + 4 * (i - 1): 1 + 4 * i]))
        _set_streaming(self.encoder, False)
        mu, _ = self.conv1(torch.cat(outs, dim=2)).chunk(2, dim=1)
        mean, inv_std = scale
        return (mu - mean.view(1, -1, 1, 1, 1)) * inv_std.view(1, -1, 1, 1, 1)

    def decode(self, z, scale):
        mean, inv_std = scale
        z = z / inv_std.view(1, -1, 1, 1, 1) + mean.view(1, -1, 1, 1, 1)
        x = self.conv2(z)
        _set_streaming(self.decoder, True)
        outs = [self.decoder(x[:, :, i:i + 1]) for i in range(z.shape[2])]
        _set_streaming(self.decoder, False)
        return torch.cat(outs, dim=2)


def video_vae(pretrained_path=None, z_dim=16, device="cuda", dtype=torch.float32, **kw):
    cfg = dict(dim=96, z_dim=z_dim, dim_mult=[1, 2, 4, 4], num_res_blocks=2, attn_scales=[],
               temperal_downsample=[False, True, True], dropout=0.0)
    cfg.update(kw)
    model = WanVAE_(**cfg)
    if pretrained_path is not None and os.path.exists(pretrained_path):
        logging.info(f"loading {pretrained_path}")
        model.load_state_dict(torch.load(pretrained_path, map_location="cpu", weights_only=True))
    return model.to(device=device, dtype=dtype)


class WanVAE:
    def __init__(self, z_dim=16, vae_pth=None, dtype=torch.float32, device="cuda", **kw):
        self.dtype, self.device = dtype, device
        self.mean = torch.tensor(LATENT_MEAN, dtype=dtype, device=device)
        self.std = torch.tensor(LATENT_STD, dtype=dtype, device=device)
        self.scale = [self.mean, 1.0 / self.std]
        self.model = video_vae(vae_pth, z_dim, device, dtype, **kw).eval().requires_grad_(False)

    def _ctx(self):
        dev = torch.device(self.device)
        if self.dtype != torch.float32 and dev.type == "cuda":
            return torch.autocast("cuda", dtype=self.dtype)
        return nullcontext()

    @torch.no_grad()
    def encode(self, videos):
        with self._ctx():
            return self.model.encode(videos.to(self.device, self.dtype), self.scale).float()

    @torch.no_grad()
    def decode(self, zs):
        with self._ctx():
            return self.model.decode(zs.to(self.device, self.dtype), self.scale).float().clamp_(-1, 1)
