"""Per-kernel benchmarks at the 14B production shapes (and small cases for profiling).

``python -m benchmarks.kernels [--case NAME ...] [--size full|small] [--iters N]``

Each case is timed with CUDA events on the launching stream after warm-up
(median of ``iters``); inputs exceed the 126 MB L2 at ``--size full``.  Output:
one JSON line per case with milliseconds, achieved TFLOP/s or GB/s, and the
fraction of the measured B200 peak (``MEASURED_PEAKS.json`` at the repository
root; fallback 1.59 PFLOP/s bf16 burst, 6.65 TB/s copy).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics

import torch

from osp_next_b200.ops import (adamw_, attention, attention_bwd, bias_grad, cfg_euler_step, gemm_t,
                               hif8_quant_dequant, linear, linear_gated_residual, ln_modulate, qk_norm_rope,
                               sde_step)
from osp_next_b200.ops.reference import rope_freqs

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d["bf16_tflops"], d.get("bf16_tflops_sustained", d["bf16_tflops"]), d["hbm_gbs"], "measured"
    return 1590.0, 1400.0, 6650.0, "fallback"


def _segs(lengths, dev):
    s = [0]
    for L in lengths:
        s.append(s[-1] + L)
    return torch.tensor(s, dtype=torch.int32)


def _time(fn, iters):
    fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(iters):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b))
    return statistics.median(ts)


def cases(size: str):
    """name → (setup() → (fn, flops, bytes))"""
    full = size == "full"
    B = 2 if full else 1
    N = 80640 if full else 20160       # tokens per sample (81f 768×1280 = 80 640)
    C, F, H, D = 5120, 13824, 40, 128
    dev = "cuda"
    bf = torch.bfloat16

    def gemm(M, Nn, K, mode):
        def setup():
            x = torch.randn(M, K, device=dev, dtype=bf)
            w = torch.randn(Nn, K, device=dev, dtype=bf) * K ** -0.5
            b = torch.randn(Nn, device=dev)
            if mode == "resid":
                r = torch.randn(1, M, Nn, device=dev)
                g = torch.randn(1, Nn, device=dev)
                fn = lambda: linear_gated_residual(x.view(1, M, K), w, b, r, g, out=r)
                byts = M * K * 2 + Nn * K * 2 + 2 * M * Nn * 4
            else:
                fn = lambda: linear(x, w, b, "gelu_tanh" if mode == "gelu" else None)
                byts = M * K * 2 + Nn * K * 2 + M * Nn * 2
            return fn, 2.0 * M * Nn * K, byts
        return setup

    def attn(lengths, nk=None):
        def setup():
            n = sum(lengths)
            q = torch.randn(B, n, H, D, device=dev, dtype=bf)
            if nk is None:
                k, v = torch.randn_like(q), torch.randn_like(q)
                sq = sk = _segs(lengths, dev)
                fl = 4.0 * B * H * sum(L * L for L in lengths) * D
            else:
                k = torch.randn(B, nk, H, D, device=dev, dtype=bf)
                v = torch.randn_like(k)
                sq, sk = _segs([n], dev), _segs([nk], dev)
                fl = 4.0 * B * H * n * nk * D
            return (lambda: attention(q, k, v, sq, sk)), fl, (q.numel() * 4 + k.numel() * 4) * 2
        return setup

    def gemm_bwd(kind, n_out, k_in):
        # backward GEMMs of a Linear with M tokens: dX = dY·W (W read MN-major),
        # dW = dYᵀ·X (dY and X read MN-major), fp32 dW
        def setup():
            dy = torch.randn(M, n_out, device=dev, dtype=bf)
            if kind == "dx":
                w = torch.randn(n_out, k_in, device=dev, dtype=bf)
                fn = lambda: gemm_t(dy, w, False, True, out_dtype=bf)
                byts = (M * n_out + n_out * k_in + M * k_in) * 2
            else:
                x = torch.randn(M, k_in, device=dev, dtype=bf)
                fn = lambda: gemm_t(dy, x, True, True)
                byts = (M * n_out + M * k_in) * 2 + n_out * k_in * 4
            return fn, 2.0 * M * n_out * k_in, byts
        return setup

    def attn_bwd(lengths):
        # algorithmic FLOPs of the backward: 5 matmuls of 2·L²·D per head (S, dP, dV, dK, dQ)
        def setup():
            n = sum(lengths)
            q = torch.randn(B, n, H, D, device=dev, dtype=bf)
            k, v = torch.randn_like(q), torch.randn_like(q)
            sq = _segs(lengths, dev)
            o, lse = attention(q, k, v, sq, sq, return_lse=True)
            g = torch.randn_like(q)
            fl = 10.0 * B * H * sum(L * L for L in lengths) * D
            return (lambda: attention_bwd(q, k, v, o, g, lse, sq, sq)), fl, q.numel() * 2 * 8
        return setup

    def lnmod():
        x = torch.randn(B, N, C, device=dev)
        sh, sc = torch.randn(B, C, device=dev), torch.randn(B, C, device=dev)
        return (lambda: ln_modulate(x, sh, sc)), 0.0, x.numel() * 6

    def qkrope():
        qkv = torch.randn(B, N, 3 * C, device=dev, dtype=bf)
        wq, wk = torch.rand(C, device=dev), torch.rand(C, device=dev)
        pos = torch.zeros(N, 3, dtype=torch.int32, device=dev)
        fr = rope_freqs(D).to(dev)
        return (lambda: qk_norm_rope(qkv, wq, wk, pos, fr, H)), 0.0, B * N * C * 2 * 4

    def hif8():
        # per-tensor HiF8 quant-dequant of an FFN-input activation: amax pass + rounding pass
        x = torch.randn(B * N, C, device=dev, dtype=bf)
        return (lambda: hif8_quant_dequant(x, 15.0)), 0.0, x.numel() * 2 * 3

    def biasg():
        g = torch.randn(B * N, F, device=dev, dtype=bf)
        return (lambda: bias_grad(g)), 0.0, g.numel() * 2

    def cfg():
        shape = (1, 16, 21, 96, 160)
        lat, c, u = (torch.randn(shape, device=dev) for _ in range(3))
        return (lambda: cfg_euler_step(lat, c, u, 5.0, -0.02)), 0.0, lat.numel() * 4 * 4

    def sde():
        shape = (12, 16, 9, 60, 104)             # Mix-GRPO rollout batch at 33f 480×832
        x, v, nz = (torch.randn(shape, device=dev) for _ in range(3))
        return (lambda: sde_step(x, v, 0.5, -0.02, 0.0, 1.0, noise=nz)), 0.0, x.numel() * 4 * 5

    def adamw():
        n = 351_000_000 // 8                      # one 14B block's shard at FSDP-8
        p_, g_, m_, v_ = (torch.randn(n, device=dev) for _ in range(4))
        v_.abs_()
        return (lambda: adamw_(p_, g_, m_, v_, 1e-5, 0.9, 0.999, 1e-8, 0.01, 3, 0.5)), 0.0, n * 4 * 7

    M = B * N
    G = N // 4
    return {
        "gemm_qkv": gemm(M, 3 * C, C, "plain"),
        "gemm_attn_out_resid": gemm(M, C, C, "resid"),
        "gemm_ffn_up_gelu": gemm(M, F, C, "gelu"),
        "gemm_ffn_down_resid": gemm(M, C, F, "resid"),
        "attn_sparse": attn([G, G, G, G]),
        "attn_dense": attn([N]),
        "attn_cross": attn([N], nk=512),
        "gemm_ffn_down_bwd_dx": gemm_bwd("dx", C, F),
        "gemm_ffn_down_bwd_dw": gemm_bwd("dw", C, F),
        "attn_sparse_bwd": attn_bwd([G, G, G, G]),
        "attn_dense_bwd": attn_bwd([N]),
        "ln_modulate": lnmod,
        "qk_norm_rope": qkrope,
        "hif8_qdq": hif8,
        "bias_grad": biasg,
        "cfg_euler": cfg,
        "sde_step": sde,
        "adamw": adamw,
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", nargs="*", default=None)
    ap.add_argument("--size", choices=["full", "small"], default="full")
    ap.add_argument("--iters", type=int, default=5)
    a = ap.parse_args()
    burst, sustained, hbm, src = peaks()
    allc = cases(a.size)
    for name in (a.case or list(allc)):
        fn, flops, byts = allc[name]()
        ms = _time(fn, a.iters)
        rec = {"case": name, "size": a.size, "ms": round(ms, 3)}
        if flops:
            tf = flops / ms / 1e9
            rec.update(tflops=round(tf, 1), frac_bf16_burst=round(tf / burst, 3), peak_source=src)
        if byts:
            gbs = byts / ms / 1e6
            rec.update(gbs=round(gbs, 1), frac_hbm=round(gbs / hbm, 3))
        print(json.dumps(rec), flush=True)
        del fn
        torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
