"""Tokenizer wrapper (reference: ospnext/modules/tokenizers.py:37-82).

Wraps a Hugging Face tokenizer directory (umT5 / google/umt5-xxl for Wan):
optional cleaning ("whitespace", "lower", "canonicalize"), fixed-length
padding/truncation to ``seq_len``, and ids (+ attention mask) as tensors.
"""
from __future__ import annotations

import html
import re
import string

import torch


def _basic_clean(text):
    try:
        import ftfy
        text = ftfy.fix_text(text)
    except ImportError:
        pass
    return html.unescape(html.unescape(text)).strip()


def _whitespace_clean(text):
    return re.sub(r"\s+", " ", text).strip()


def _canonicalize(text, keep_punctuation_exact_string=None):
    text = text.replace("_", " ")
    if keep_punctuation_exact_string:
        text = keep_punctuation_exact_string.join(
            part.translate(str.maketrans("", "", string.punctuation))
            for part in text.split(keep_punctuation_exact_string))
    else:
        text = text.translate(str.maketrans("", "", string.punctuation))
    return re.sub(r"\s+", " ", text.lower()).strip()


def load_tokenizer(path):
    from transformers import AutoTokenizer
    return AutoTokenizer.from_pretrained(path)


class HuggingfaceTokenizer:
    def __init__(self, name, seq_len=None, clean=None, **kwargs):
        assert clean in (None, "whitespace", "lower", "canonicalize")
        self.name, self.seq_len, self.clean = name, seq_len, clean
        self.tokenizer = load_tokenizer(name) if isinstance(name, str) else name
        self.vocab_size = self.tokenizer.vocab_size

    def __call__(self, sequence, **kwargs):
        return_mask = kwargs.pop("return_mask", False)
        _kw = {"return_tensors": "pt"}
        if self.seq_len is not None:
            _kw.update(padding="max_length", truncation=True, max_length=self.seq_len)
        _kw.update(**kwargs)
        if isinstance(sequence, str):
            sequence = [sequence]
        if self.clean:
            sequence = [self._clean(u) for u in sequence]
        ids = self.tokenizer(sequence, **_kw)
        return (ids.input_ids, ids.attention_mask) if return_mask else ids.input_ids

    def _clean(self, text):
        if self.clean == "whitespace":
            return _whitespace_clean(_basic_clean(text))
        if self.clean == "lower":
            return _whitespace_clean(_basic_clean(text)).lower()
        return _canonicalize(_basic_clean(text))
