"""Prompt tokenizer for the umT5 text encoder (reference: ospnext/modules/tokenizers.py:37-82).

What the framework needs from a tokenizer is narrow: the T5 encoder turns a batch
of prompts into fixed-length ids plus an attention mask, and the dataset turns one
caption into ids.  This module therefore has two parts:

* ``CLEANERS`` — a table from a cleaning mode to an ordered list of text passes
  (``None``, ``"whitespace"``, ``"lower"``, ``"canonicalize"``).  Each pass is a
  plain ``str -> str`` function; a mode is their composition.
* ``PromptTokenizer`` — a Hugging Face tokenizer (a directory such as
  google/umt5-xxl, or an already constructed object) plus a cleaning mode and a
  fixed length.  ``encode`` returns a ``TokenBatch``; calling the object keeps the
  reference's call convention (``tok(texts, return_mask=True)`` → ``(ids, mask)``).

``HuggingfaceTokenizer`` is the reference's public name for the same object.
"""
from __future__ import annotations

import html
import re
import string
from dataclasses import dataclass
from typing import Callable, Dict, List, Optional, Sequence, Union

import torch

_WS = re.compile(r"\s+")


def _repair(text: str) -> str:
    """Undo mojibake when ftfy is installed, then resolve (doubly) escaped HTML entities."""
    try:
        import ftfy
    except ImportError:
        ftfy = None
    if ftfy is not None:
        text = ftfy.fix_text(text)
    for _ in range(2):
        text = html.unescape(text)
    return text.strip()


def _collapse(text: str) -> str:
    return _WS.sub(" ", text).strip()


def _lower(text: str) -> str:
    return text.lower()


def _strip_punct(text: str, keep: Optional[str] = None) -> str:
    """Underscores become spaces and ASCII punctuation is dropped, except inside `keep` runs."""
    table = str.maketrans("", "", string.punctuation)
    text = text.replace("_", " ")
    pieces = text.split(keep) if keep else [text]
    return (keep or "").join(p.translate(table) for p in pieces)


CLEANERS: Dict[Optional[str], List[Callable[[str], str]]] = {
    None: [],
    "whitespace": [_repair, _collapse],
    "lower": [_repair, _collapse, _lower],
    "canonicalize": [_repair, _strip_punct, _lower, _collapse],
}


def clean_text(text: str, mode: Optional[str]) -> str:
    if mode not in CLEANERS:
        raise ValueError(f"unknown cleaning mode {mode!r}; expected one of {sorted(map(str, CLEANERS))}")
    for step in CLEANERS[mode]:
        text = step(text)
    return text


def load_tokenizer(path):
    """A Hugging Face tokenizer from a local directory (no network on the training boxes)."""
    from transformers import AutoTokenizer
    return AutoTokenizer.from_pretrained(path)


@dataclass
class TokenBatch:
    ids: torch.Tensor       # [B, L] int64
    mask: torch.Tensor      # [B, L] int64, 1 on real tokens

    @property
    def lengths(self) -> torch.Tensor:
        return self.mask.gt(0).sum(dim=1)


class PromptTokenizer:
    def __init__(self, name_or_tokenizer, seq_len: Optional[int] = None, clean: Optional[str] = None, **_unused):
        if clean not in CLEANERS:
            raise ValueError(f"unknown cleaning mode {clean!r}")
        self.name = name_or_tokenizer if isinstance(name_or_tokenizer, str) else type(name_or_tokenizer).__name__
        self.tokenizer = load_tokenizer(name_or_tokenizer) if isinstance(name_or_tokenizer, str) else name_or_tokenizer
        self.seq_len = seq_len
        self.clean = clean
        self.vocab_size = self.tokenizer.vocab_size

    def _hf_kwargs(self, extra: dict) -> dict:
        kw = {"return_tensors": "pt"}
        if self.seq_len is not None:     # fixed length: pad to and cut at seq_len
            kw.update(padding="max_length", truncation=True, max_length=self.seq_len)
        kw.update(extra)
        return kw

    def encode(self, texts: Union[str, Sequence[str]], **hf_kwargs) -> TokenBatch:
        batch = [texts] if isinstance(texts, str) else list(texts)
        batch = [clean_text(t, self.clean) for t in batch]
        enc = self.tokenizer(batch, **self._hf_kwargs(hf_kwargs))
        return TokenBatch(enc.input_ids, enc.attention_mask)

    def __call__(self, texts, return_mask: bool = False, **hf_kwargs):
        tb = self.encode(texts, **hf_kwargs)
        return (tb.ids, tb.mask) if return_mask else tb.ids


HuggingfaceTokenizer = PromptTokenizer
