"""Video / image reading and writing (reference: ospnext/data/utils/video_reader.py:41-353,
image_reader.py:14-70, utils/infer_utils.py).

``VideoReader(backend)(path, layout=..., array_type=...)`` opens a video with one of four
decoders behind one interface — ``get_batch(frame_indices)``, ``get_video_fps()``,
``get_num_frames()``, ``close()`` and use as a context manager:

* ``decord`` and ``av`` (PyAV) when those packages are importable (the reference's
  default is decord);
* ``torchvision`` (``torchvision.io.read_video``, whole clip decoded once);
* ``opencv`` (``cv2.VideoCapture``, sequential decode of only the requested frames).

``backend="auto"`` picks the first available of decord, av, opencv.  Frames are RGB uint8,
``TCHW`` (default) or ``THWC``, as torch tensors or numpy arrays.  ``ImageReader`` does the
same for still images (PIL or OpenCV).
"""
from __future__ import annotations

import gc
import importlib.util
import os
from contextlib import contextmanager
from typing import Optional, Sequence

import numpy as np
import torch

VIDEO_EXTENSIONS = {".mp4", ".avi", ".mov", ".mkv", ".flv", ".wmv", ".webm", ".mpeg", ".mpg", ".3gp"}
IMAGE_EXTENSIONS = {".jpg", ".jpeg", ".png", ".bmp", ".webp", ".tif", ".tiff"}
MAX_FRAMES = 1024


def is_video_file(path: str) -> bool:
    return os.path.splitext(path)[1].lower() in VIDEO_EXTENSIONS


def is_image_file(path: str) -> bool:
    return os.path.splitext(path)[1].lower() in IMAGE_EXTENSIONS


def _has(mod: str) -> bool:
    return importlib.util.find_spec(mod) is not None


class Video:
    """Common interface; subclasses implement ``_open``, ``_frames(indices) → [N,H,W,C] uint8``,
    ``_fps`` and ``_count``."""

    def __init__(self, video_path: str, layout: str = "TCHW", array_type: str = "torch", **kwargs):
        if layout not in ("TCHW", "THWC"):
            raise ValueError(f"layout must be TCHW or THWC, got {layout}")
        if array_type not in ("torch", "numpy"):
            raise ValueError(f"array_type must be torch or numpy, got {array_type}")
        if not os.path.exists(video_path):
            raise FileNotFoundError(video_path)
        self.video_path, self.layout, self.array_type = video_path, layout, array_type
        self._open(**kwargs)

    def get_batch(self, frame_indices):
        idx = [int(i) for i in (frame_indices.tolist() if hasattr(frame_indices, "tolist") else frame_indices)]
        n = self.get_num_frames()
        if idx and (min(idx) < 0 or max(idx) >= n):
            raise IndexError(f"frame indices outside [0, {n}) for {self.video_path}")
        frames = self._frames(idx)                          # [N, H, W, C] uint8 numpy
        out = torch.from_numpy(np.ascontiguousarray(frames))
        if self.layout == "TCHW":
            out = out.permute(0, 3, 1, 2)
        return out if self.array_type == "torch" else out.numpy()

    def get_video_fps(self) -> float:
        return float(self._fps())

    def get_num_frames(self) -> int:
        return int(self._count())

    def close(self):
        pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


class DecordVideo(Video):
    def _open(self, **kw):
        import decord
        self.vr = decord.VideoReader(self.video_path, ctx=decord.cpu(0), num_threads=kw.get("num_threads", 1))

    def _frames(self, idx):
        return self.vr.get_batch(idx).asnumpy()

    def _fps(self):
        return self.vr.get_avg_fps()

    def _count(self):
        return len(self.vr)

    def close(self):
        self.vr = None
        gc.collect()


class AvVideo(Video):
    """PyAV: the whole stream is decoded once into RGB frames."""

    def _open(self, **kw):
        import av
        with av.open(self.video_path, metadata_errors="ignore") as c:
            st = c.streams.video[0]
            self.rate = float(st.average_rate) if st.average_rate is not None else 0.0
            self.all = np.stack([f.to_rgb().to_ndarray() for f in c.decode(st)])

    def _frames(self, idx):
        return self.all[idx]

    def _fps(self):
        return self.rate

    def _count(self):
        return len(self.all)

    def close(self):
        self.all = None
        gc.collect()


class TorchvisionVideo(Video):
    def _open(self, **kw):
        from torchvision.io import read_video
        v, _, info = read_video(self.video_path, pts_unit="sec", output_format="THWC")
        self.all = v.numpy()
        self.rate = float(info.get("video_fps", 0.0))

    def _frames(self, idx):
        return self.all[idx]

    def _fps(self):
        return self.rate

    def _count(self):
        return len(self.all)


class OpenCVVideo(Video):
    """Sequential decoding of only the requested frames (sorted, one seek)."""

    def _open(self, **kw):
        import cv2
        self.cv2 = cv2
        self.cap = cv2.VideoCapture(self.video_path)
        if not self.cap.isOpened():
            raise IOError(f"cannot open video {self.video_path}")

    def _frames(self, idx):
        want = sorted(set(idx))
        got = {}
        if want:
            self.cap.set(self.cv2.CAP_PROP_POS_FRAMES, want[0])
            cur = want[0]
            for tgt in want:
                while cur <= tgt:
                    ok, fr = self.cap.read()
                    if not ok:
                        raise IOError(f"frame {cur} of {self.video_path} unreadable")
                    if cur == tgt:
                        got[tgt] = self.cv2.cvtColor(fr, self.cv2.COLOR_BGR2RGB)
                    cur += 1
        return np.stack([got[i] for i in idx]) if idx else np.zeros((0, 1, 1, 3), np.uint8)

    def _fps(self):
        return self.cap.get(self.cv2.CAP_PROP_FPS)

    def _count(self):
        return self.cap.get(self.cv2.CAP_PROP_FRAME_COUNT)

    def close(self):
        if getattr(self, "cap", None) is not None:
            self.cap.release()
            self.cap = None


_BACKENDS = {"decord": (DecordVideo, "decord"), "av": (AvVideo, "av"), "torchvision": (TorchvisionVideo, None),
             "opencv": (OpenCVVideo, "cv2")}


def available_backends():
    return [b for b, (_, mod) in _BACKENDS.items() if mod is None or _has(mod)]


class VideoReader:
    """``VideoReader(backend)(path, layout="TCHW", array_type="torch")`` → a :class:`Video`."""

    def __init__(self, backend: str = "auto"):
        backend = backend.lower()
        if backend == "auto":
            backend = next(b for b in ("decord", "av", "opencv", "torchvision") if b in available_backends())
        if backend not in _BACKENDS:
            raise ValueError(f"unsupported video reader backend {backend!r}; available: {available_backends()}")
        cls, mod = _BACKENDS[backend]
        if mod is not None and not _has(mod):
            raise ImportError(f"video backend {backend!r} needs the {mod} package, which is not installed")
        self.backend, self.reader_cls = backend, cls

    def __call__(self, *args, **kwargs) -> Video:
        return self.reader_cls(*args, **kwargs)


@contextmanager
def video_reader_contextmanager(path: str, backend: str = "auto", **kwargs):
    r = VideoReader(backend)(path, **kwargs)
    try:
        yield r
    finally:
        r.close()


class ImageReader:
    """Still images as uint8 ``CHW`` (or ``HWC``) RGB tensors / arrays (PIL, else OpenCV)."""

    def __init__(self, backend: str = "auto"):
        self.backend = ("pil" if _has("PIL") else "opencv") if backend == "auto" else backend.lower()

    def __call__(self, path: str, layout: str = "CHW", array_type: str = "torch"):
        if self.backend == "pil":
            from PIL import Image
            with Image.open(path) as im:
                arr = np.asarray(im.convert("RGB"))
        else:
            import cv2
            im = cv2.imread(path, cv2.IMREAD_COLOR)
            if im is None:
                raise IOError(f"cannot read image {path}")
            arr = cv2.cvtColor(im, cv2.COLOR_BGR2RGB)
        t = torch.from_numpy(np.ascontiguousarray(arr))
        if layout == "CHW":
            t = t.permute(2, 0, 1)
        return t if array_type == "torch" else t.numpy()


def read_image(path: str) -> torch.Tensor:
    return ImageReader()(path)


def save_video(video: torch.Tensor, path: str, fps: int = 16):
    """uint8 [T, H, W, C] → mp4 (OpenCV, mp4v)."""
    import cv2
    v = video.cpu().numpy() if torch.is_tensor(video) else np.asarray(video)
    T, H, W, _ = v.shape
    w = cv2.VideoWriter(path, cv2.VideoWriter_fourcc(*"mp4v"), fps, (W, H))
    for t in range(T):
        w.write(cv2.cvtColor(v[t], cv2.COLOR_RGB2BGR))
    w.release()


def video_grid(videos: Sequence[torch.Tensor], nrow: int = 0) -> torch.Tensor:
    """Tile uint8 [T,H,W,C] videos of equal size into one grid video."""
    n = len(videos)
    nrow = nrow or int(np.ceil(np.sqrt(n)))
    ncol = int(np.ceil(n / nrow))
    T, H, W, C = videos[0].shape
    grid = torch.zeros(T, ncol * H, nrow * W, C, dtype=torch.uint8)
    for i, v in enumerate(videos):
        r, c = divmod(i, nrow)
        grid[:, r * H:(r + 1) * H, c * W:(c + 1) * W] = v
    return grid
