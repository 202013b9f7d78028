"""umT5 text encoder (frozen; reference: ospnext/modules/t5.py:53-522).

Architecture of umT5-XXL as used by Wan-2.1: 24 pre-norm encoder layers, width
4096, 64 heads of 64, gated-GELU(tanh) FFN 10240, RMS-style T5 LayerNorm, no
attention scaling, a relative-position bias per layer (bidirectional, 32
buckets, max distance 128).  Parameter names follow the Wan checkpoint layout
(``token_embedding``, ``blocks.{i}.{norm1,attn.{q,k,v,o},norm2,ffn.{gate.0,fc1,fc2},
pos_embedding.embedding}``, ``norm``).  ``T5EncoderModel`` tokenises, encodes and
zero-pads every sequence beyond its length to ``text_len`` tokens, which is the
text embedding the DiT consumes.

The relative-position bucket function is the standard T5 one (exact buckets for
small offsets, logarithmic buckets up to ``max_dist``), restated here.
"""
from __future__ import annotations

import math
from typing import List, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F


class T5LayerNorm(nn.Module):
    def __init__(self, dim, eps=1e-6):
        super().__init__()
        self.dim, self.eps = dim, eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x):
        x = x * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + self.eps)
        if self.weight.dtype in (torch.float16, torch.bfloat16):
            x = x.type_as(self.weight)
        return self.weight * x


def relative_position_bucket(rel: torch.Tensor, num_buckets: int, bidirectional: bool, max_dist: int) -> torch.Tensor:
    if bidirectional:
        num_buckets //= 2
        base = (rel > 0).long() * num_buckets
        rel = rel.abs()
    else:
        base = torch.zeros_like(rel)
        rel = -torch.clamp(rel, max=0)
    exact = num_buckets // 2
    large = exact + (torch.log(rel.float().clamp(min=1) / exact) / math.log(max_dist / exact)
                     * (num_buckets - exact)).long()
    large = torch.clamp(large, max=num_buckets - 1)
    return base + torch.where(rel < exact, rel, large)


class T5RelativeEmbedding(nn.Module):
    def __init__(self, num_buckets, num_heads, bidirectional, max_dist=128):
        super().__init__()
        self.num_buckets, self.num_heads = num_buckets, num_heads
        self.bidirectional, self.max_dist = bidirectional, max_dist
        self.embedding = nn.Embedding(num_buckets, num_heads)

    def forward(self, lq, lk):
        dev = self.embedding.weight.device
        rel = torch.arange(lk, device=dev)[None, :] - torch.arange(lq, device=dev)[:, None]
        b = relative_position_bucket(rel, self.num_buckets, self.bidirectional, self.max_dist)
        return self.embedding(b).permute(2, 0, 1).unsqueeze(0).contiguous()     # [1, H, Lq, Lk]


class T5Attention(nn.Module):
    def __init__(self, dim, dim_attn, num_heads, dropout=0.1):
        super().__init__()
        self.num_heads, self.head_dim = num_heads, dim_attn // num_heads
        self.q = nn.Linear(dim, dim_attn, bias=False)
        self.k = nn.Linear(dim, dim_attn, bias=False)
        self.v = nn.Linear(dim, dim_attn, bias=False)
        self.o = nn.Linear(dim_attn, dim, bias=False)
        self.dropout = nn.Dropout(dropout)

    def forward(self, x, context=None, mask=None, pos_bias=None):
        ctx = x if context is None else context
        b, n, c = x.size(0), self.num_heads, self.head_dim
        q = self.q(x).view(b, -1, n, c).transpose(1, 2)
        k = self.k(ctx).view(b, -1, n, c).transpose(1, 2)
        v = self.v(ctx).view(b, -1, n, c).transpose(1, 2)
        bias = torch.zeros(b, n, q.size(2), k.size(2), dtype=torch.float32, device=x.device)
        if pos_bias is not None:
            bias = bias + pos_bias.float()
        if mask is not None:
            m = mask.view(b, 1, 1, -1) if mask.ndim == 2 else mask.unsqueeze(1)
            bias = bias.masked_fill(m == 0, torch.finfo(torch.float32).min)
        # T5 uses no 1/sqrt(d) scaling
        attn = torch.softmax(torch.matmul(q.float(), k.float().transpose(-1, -2)) + bias, dim=-1).type_as(v)
        out = torch.matmul(attn, v).transpose(1, 2).reshape(b, -1, n * c)
        return self.dropout(self.o(out))


class T5FeedForward(nn.Module):
    def __init__(self, dim, dim_ffn, dropout=0.1):
        super().__init__()
        self.gate = nn.Sequential(nn.Linear(dim, dim_ffn, bias=False), nn.GELU(approximate="tanh"))
        self.fc1 = nn.Linear(dim, dim_ffn, bias=False)
        self.fc2 = nn.Linear(dim_ffn, dim, bias=False)
        self.dropout = nn.Dropout(dropout)

    def forward(self, x):
        return self.dropout(self.fc2(self.dropout(self.fc1(x) * self.gate(x))))


def _fp16_clamp(x):
    if x.dtype == torch.float16 and torch.isinf(x).any():
        c = torch.finfo(x.dtype).max - 1000
        x = torch.clamp(x, -c, c)
    return x


class T5SelfAttention(nn.Module):
    def __init__(self, dim, dim_attn, dim_ffn, num_heads, num_buckets, shared_pos=True, dropout=0.1):
        super().__init__()
        self.shared_pos = shared_pos
        self.norm1 = T5LayerNorm(dim)
        self.attn = T5Attention(dim, dim_attn, num_heads, dropout)
        self.norm2 = T5LayerNorm(dim)
        self.ffn = T5FeedForward(dim, dim_ffn, dropout)
        self.pos_embedding = None if shared_pos else T5RelativeEmbedding(num_buckets, num_heads, True)

    def forward(self, x, mask=None, pos_bias=None):
        e = pos_bias if self.shared_pos else self.pos_embedding(x.size(1), x.size(1))
        x = _fp16_clamp(x + self.attn(self.norm1(x), mask=mask, pos_bias=e))
        return _fp16_clamp(x + self.ffn(self.norm2(x)))


class T5Encoder(nn.Module):
    def __init__(self, vocab, dim, dim_attn, dim_ffn, num_heads, num_layers, num_buckets, shared_pos=True,
                 dropout=0.1):
        super().__init__()
        self.dim = dim
        self.shared_pos = shared_pos
        self.token_embedding = vocab if isinstance(vocab, nn.Embedding) else nn.Embedding(vocab, dim)
        self.pos_embedding = T5RelativeEmbedding(num_buckets, num_heads, True) if shared_pos else None
        self.dropout = nn.Dropout(dropout)
        self.blocks = nn.ModuleList([T5SelfAttention(dim, dim_attn, dim_ffn, num_heads, num_buckets, shared_pos,
                                                     dropout) for _ in range(num_layers)])
        self.norm = T5LayerNorm(dim)
        self.apply(_init)

    def forward(self, ids, mask=None):
        x = self.dropout(self.token_embedding(ids))
        e = self.pos_embedding(x.size(1), x.size(1)) if self.shared_pos else None
        for blk in self.blocks:
            x = blk(x, mask, pos_bias=e)
        return self.dropout(self.norm(x))


T5Model = T5Encoder
T5Decoder = None          # the T2V pipeline only uses the encoder


def _init(m):
    if isinstance(m, T5LayerNorm):
        nn.init.ones_(m.weight)
    elif isinstance(m, nn.Linear):
        nn.init.normal_(m.weight, std=m.in_features ** -0.5)
    elif isinstance(m, nn.Embedding):
        nn.init.normal_(m.weight, std=1.0)


UMT5_XXL = dict(vocab=256384, dim=4096, dim_attn=4096, dim_ffn=10240, num_heads=64, num_layers=24,
                num_buckets=32, shared_pos=False, dropout=0.0)


def umt5_xxl(**overrides) -> T5Encoder:
    cfg = dict(UMT5_XXL)
    cfg.update(overrides)
    return T5Encoder(**cfg)


def shard_t5(model: nn.Module, mesh=None) -> nn.Module:
    """FSDP2-shard the frozen encoder: every T5SelfAttention layer, then the root
    (reference: ospnext/modules/t5.py:500-506).  ``mesh`` is a (replicate, shard) mesh
    (8-way shards by default, see :func:`t5_mesh`) or None for the default world mesh."""
    from torch.distributed.fsdp import fully_shard
    for m in model.modules():
        if isinstance(m, T5SelfAttention):
            fully_shard(m, mesh=mesh)
    fully_shard(model, mesh=mesh)
    return model


def t5_mesh(world_size: int, shard: int = 8, device_type: str = "cuda"):
    """(replicate, shard) mesh for the text encoder: shards of ``shard`` ranks (fewer when
    the world is smaller), replicated over the rest (reference: train_osp.py:189-193)."""
    from torch.distributed.device_mesh import init_device_mesh
    n_rep = max(world_size // shard, 1)
    return init_device_mesh(device_type, (n_rep, world_size // n_rep), mesh_dim_names=("replicate", "shard"))


class T5EncoderModel:
    """Tokenise + encode prompts → ``[B, text_len, 4096]`` with zeros past each length."""

    def __init__(self, text_len=512, dtype=torch.bfloat16, device="cuda", checkpoint_path=None, tokenizer_path=None,
                 shard_fn=None, encoder: Optional[T5Encoder] = None, tokenizer=None, use_fsdp: bool = False,
                 device_mesh=None):
        self.text_len = text_len
        self.dtype = dtype
        self.device = device
        model = encoder if encoder is not None else umt5_xxl()
        model = model.eval().requires_grad_(False)
        if checkpoint_path:
            sd = torch.load(checkpoint_path, map_location="cpu", weights_only=True)
            model.load_state_dict(sd)
        if use_fsdp and shard_fn is None:
            shard_fn = lambda m: shard_t5(m.to(device=device, dtype=dtype), device_mesh)  # noqa: E731
        self.model = shard_fn(model) if shard_fn is not None else model.to(device=device, dtype=dtype)
        if tokenizer is None and tokenizer_path:
            from .tokenizers import HuggingfaceTokenizer
            tokenizer = HuggingfaceTokenizer(tokenizer_path, seq_len=text_len, clean="whitespace")
        self.tokenizer = tokenizer

    @torch.no_grad()
    def __call__(self, ids_or_texts, mask=None):
        if isinstance(ids_or_texts, (list, str)):
            ids, mask = self.tokenizer(ids_or_texts, return_mask=True, add_special_tokens=True)
        else:
            ids = ids_or_texts
        ids, mask = ids.to(self.device), mask.to(self.device)
        seq_lens = mask.gt(0).sum(dim=1).long()
        ctx = self.model(ids, mask)
        out = torch.zeros(ids.shape[0], self.text_len, ctx.shape[-1], dtype=ctx.dtype, device=ctx.device)
        for i, L in enumerate(seq_lens.tolist()):
            out[i, :L] = ctx[i, :L]
        return out
