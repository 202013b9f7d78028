"""Video / image reading and writing (reference: ospnext/data/utils/video_reader.py,
image_reader.py, utils/infer_utils.py).  Decoding uses OpenCV (decord / PyAV are
not available on this image); frames come out as uint8 ``[T, C, H, W]`` RGB."""
from __future__ import annotations

from contextlib import contextmanager
from typing import Sequence

import numpy as np
import torch


class CV2VideoReader:
    def __init__(self, path: str):
        import cv2
        self.cv2 = cv2
        self.cap = cv2.VideoCapture(path)
        if not self.cap.isOpened():
            raise IOError(f"cannot open video {path}")

    def get_video_fps(self) -> float:
        return float(self.cap.get(self.cv2.CAP_PROP_FPS))

    def get_num_frames(self) -> int:
        return int(self.cap.get(self.cv2.CAP_PROP_FRAME_COUNT))

    def get_batch(self, indices: Sequence[int]) -> torch.Tensor:
        out = []
        want = sorted(set(int(i) for i in indices))
        frames = {}
        self.cap.set(self.cv2.CAP_PROP_POS_FRAMES, want[0])
        cur = want[0]
        for tgt in want:
            while cur <= tgt:
                ok, fr = self.cap.read()
                if not ok:
                    raise IOError(f"frame {cur} unreadable")
                if cur == tgt:
                    frames[tgt] = self.cv2.cvtColor(fr, self.cv2.COLOR_BGR2RGB)
                cur += 1
        for i in indices:
            out.append(torch.from_numpy(frames[int(i)]).permute(2, 0, 1))
        return torch.stack(out)

    def close(self):
        self.cap.release()


@contextmanager
def video_reader_contextmanager(path: str):
    r = CV2VideoReader(path)
    try:
        yield r
    finally:
        r.close()


def read_image(path: str) -> torch.Tensor:
    import cv2
    im = cv2.imread(path, cv2.IMREAD_COLOR)
    if im is None:
        raise IOError(f"cannot read image {path}")
    return torch.from_numpy(cv2.cvtColor(im, cv2.COLOR_BGR2RGB)).permute(2, 0, 1)


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
