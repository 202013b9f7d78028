"""Metadata stores for video datasets (reference: ospnext/data/utils/utils.py:78-170, 273-611).

One record per sample: ``{"path", "cap", "num_frames", "fps", "resolution": {"height","width"},
"motion"?, "cut"?, "crop"?}``.  Two interchangeable backends:

* **LMDB** (the reference's format; key ``str(index)``, value zstd/pickle) when
  the ``lmdb`` package is installed;
* **JSONL** (one JSON record per line, with a byte-offset index built on open)
  that needs no extra dependency.

``open_meta_reader(path)`` picks the backend from the path; writers support
building one shard per rank and merging (the reference's multi-rank writer).
"""
from __future__ import annotations

import json
import os
import pickle
from typing import Dict, Iterable, List


def _zstd():
    try:
        import zstandard
        return zstandard
    except ImportError:
        return None


class JSONLMetaReader:
    def __init__(self, path: str):
        self.path = path
        self.offsets: List[int] = []
        with open(path, "rb") as f:
            pos = 0
            for line in f:
                if line.strip():
                    self.offsets.append(pos)
                pos += len(line)
        self._f = None

    def __len__(self):
        return len(self.offsets)

    def getitem(self, index: int) -> Dict:
        if self._f is None:
            self._f = open(self.path, "rb")
        self._f.seek(self.offsets[index])
        return json.loads(self._f.readline())


class JSONLMetaWriter:
    def __init__(self, path: str):
        self.path = path
        self._f = open(path, "w", encoding="utf-8")

    def write(self, records: Iterable[Dict]):
        for r in records:
            self._f.write(json.dumps(r, ensure_ascii=False) + "\n")

    def close(self):
        self._f.close()


class LMDBReader:
    def __init__(self, path: str):
        try:
            import lmdb
        except ImportError as e:
            raise ImportError("LMDB metadata needs the `lmdb` package; convert to JSONL "
                              "(osp_next_b200.data.utils.meta_store.JSONLMetaWriter) or install lmdb") from e
        self.env = lmdb.open(path, readonly=True, lock=False, readahead=False, meminit=False)
        with self.env.begin() as txn:
            self.length = int(txn.get(b"__len__").decode())

    def __len__(self):
        return self.length

    def getitem(self, index):
        with self.env.begin() as txn:
            raw = txn.get(str(index).encode())
        z = _zstd()
        if z is not None and raw[:4] == b"\x28\xb5\x2f\xfd":
            raw = z.ZstdDecompressor().decompress(raw)
        return pickle.loads(raw)


class LMDBWriter:
    def __init__(self, path: str, map_size: int = 1 << 40, compress: bool = True):
        import lmdb
        self.env = lmdb.open(path, map_size=map_size)
        self.n = 0
        self.compress = compress and _zstd() is not None

    def write(self, records: Iterable[Dict]):
        z = _zstd()
        with self.env.begin(write=True) as txn:
            for r in records:
                raw = pickle.dumps(r)
                if self.compress:
                    raw = z.ZstdCompressor().compress(raw)
                txn.put(str(self.n).encode(), raw)
                self.n += 1
            txn.put(b"__len__", str(self.n).encode())

    def close(self):
        self.env.close()


def open_meta_reader(path: str):
    if path.endswith(".jsonl") or path.endswith(".json"):
        return JSONLMetaReader(path)
    return LMDBReader(path)


def merge_jsonl_shards(shards: List[str], out: str):
    """Concatenate per-rank shards written in parallel into one store."""
    w = JSONLMetaWriter(out)
    for s in shards:
        r = JSONLMetaReader(s)
        w.write(r.getitem(i) for i in range(len(r)))
    w.close()
