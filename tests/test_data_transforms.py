"""Video transforms vs the reference's transforms module (CPU, same random draws), and the
video / image readers on a file written here."""
import importlib
import importlib.util
import os
import random
import sys

import numpy as np
import pytest
import torch

from osp_next_b200.data.utils import transforms as T
from osp_next_b200.data.utils import video_io as vio

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


_REF = []


def _ref():
    """The reference's transforms.py loaded on its own (its package __init__ needs decoders
    that are not installed here)."""
    if _REF:
        return _REF[0]
    path = os.path.join(ROOT, "baseline", "_ref", "ospnext", "data", "utils", "transforms.py")
    if not os.path.exists(path):
        pytest.skip("reference not installed in baseline/_ref")
    spec = importlib.util.spec_from_file_location("ref_transforms", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    _REF.append(mod)
    return mod


@pytest.mark.parametrize("hw", [(720, 1280), (480, 832), (1080, 1080), (333, 517)])
def test_size_rules_match_reference(hw):
    R = _ref()
    h, w = hw
    for size in ((320, 640), (480, 640), (720, 1280), (256, 256)):
        for skip in (False, True):
            assert T.fit_long_side(h, w, size, skip) == R.longsideresize(h, w, size, skip)
            assert T.fit_short_side(h, w, size, skip) == R.shortsideresize(h, w, size, skip)
    for m in (100000, 480 * 832, 10 ** 7):
        assert T.fit_max_area(h, w, m) == R.maxhwresize(h, w, m)
    for s in (8, 16, 32):
        assert T.stride_crop_box(h, w, s) == R.get_params(h, w, s)
    assert T.filter_resolution(h, w) == R.filter_resolution(h, w)


def test_clip_transforms_match_reference():
    R = _ref()
    g = torch.Generator().manual_seed(0)
    clip_u8 = torch.randint(0, 256, (3, 3, 90, 160), generator=g, dtype=torch.uint8)
    clip = clip_u8.float()
    pairs = [
        (T.CenterCropResizeVideo((48, 80), "bicubic", False, True), R.CenterCropResizeVideo((48, 80), "bicubic", False, True)),
        (T.CenterCropResizeVideo((64, 64)), R.CenterCropResizeVideo((64, 64))),
        (T.LongSideResizeVideo((40, 60)), R.LongSideResizeVideo((40, 60))),
        (T.MaxHWResizeVideo({"max_hxw": 3000}), R.MaxHWResizeVideo({"max_hxw": 3000})),
        (T.ResizeVideo({"max_height": 30, "max_width": 50}, mode="shortside"),
         R.ResizeVideo({"max_height": 30, "max_width": 50}, mode="shortside")),
        (T.ResizeVideo(2000, mode="hxw"), R.ResizeVideo(2000, mode="hxw")),
        (T.ResizeVideo((33, 47)), R.ResizeVideo((33, 47))),
        (T.UCFCenterCropVideo(40), R.UCFCenterCropVideo(40)),
        (T.SpatialStrideCropVideo(32), R.SpatialStrideCropVideo(32)),
        (T.ResizeCrop((50, 70)), R.ResizeCrop((50, 70))),
        (T.AENorm(), R.AENorm()), (T.ToTensorAfterResize(), R.ToTensorAfterResize()),
    ]
    for ours, theirs in pairs:
        a, b = ours(clip.clone()), theirs(clip.clone())
        assert a.shape == b.shape and torch.allclose(a, b, atol=1e-4), type(ours).__name__
    assert torch.equal(T.ToTensorVideo()(clip_u8), R.ToTensorVideo()(clip_u8))
    assert torch.equal(T.center_crop_using_short_edge(clip), R.center_crop_using_short_edge(clip))
    for top in (True, False):
        assert torch.equal(T.center_crop_th_tw(clip, 48, 80, top), R.center_crop_th_tw(clip, 48, 80, top))
    for seed in range(5):
        random.seed(seed)
        a = T.RandomSizedCrop((32, 64))(clip)
        random.seed(seed)
        b = R.RandomSizedCrop((32, 64))(clip)
        assert torch.equal(a, b)
        random.seed(seed)
        a = T.RandomHorizontalFlipVideo()(clip)
        random.seed(seed)
        assert torch.equal(a, R.RandomHorizontalFlipVideo()(clip))
        for total in (49, 81, 200):
            random.seed(seed)
            a = T.TemporalRandomCrop(49)(total)
            random.seed(seed)
            assert a == R.TemporalRandomCrop(49)(total)


def test_expand2square_matches_reference():
    R = _ref()
    from PIL import Image
    for size in ((40, 30), (30, 40), (20, 20)):
        im = Image.fromarray(np.random.RandomState(0).randint(0, 255, (size[1], size[0], 3), dtype=np.uint8))
        a, b = T.Expand2Square((0.5, 0.4, 0.3))(im), R.Expand2Square((0.5, 0.4, 0.3))(im)
        assert np.array_equal(np.asarray(a), np.asarray(b))


def test_video_and_image_readers_round_trip(tmp_path):
    frames = np.zeros((12, 32, 48, 3), np.uint8)
    for t in range(12):
        frames[t, :, :, 0] = t * 20           # frame index encoded in the red channel
    p = str(tmp_path / "clip.avi")
    import cv2
    w = cv2.VideoWriter(p, cv2.VideoWriter_fourcc(*"MJPG"), 8, (48, 32))
    for f in frames:
        w.write(cv2.cvtColor(f, cv2.COLOR_RGB2BGR))
    w.release()
    assert vio.is_video_file(p) and "opencv" in vio.available_backends()
    with vio.video_reader_contextmanager(p, backend="opencv") as r:
        assert r.get_num_frames() == 12 and abs(r.get_video_fps() - 8) < 1e-3
        b = r.get_batch([7, 2, 2, 11])
        assert b.shape == (4, 3, 32, 48) and b.dtype == torch.uint8
        red = b[:, 0].float().mean((1, 2))
        assert torch.allclose(red, torch.tensor([140.0, 40.0, 40.0, 220.0]), atol=6)
    r = vio.VideoReader("opencv")(p, layout="THWC", array_type="numpy")
    assert r.get_batch(np.array([0, 1])).shape == (2, 32, 48, 3)
    r.close()
    with pytest.raises(IndexError):
        vio.VideoReader("opencv")(p).get_batch([12])
    ip = str(tmp_path / "im.png")
    cv2.imwrite(ip, cv2.cvtColor(frames[5], cv2.COLOR_RGB2BGR))
    im = vio.ImageReader()(ip)
    assert im.shape == (3, 32, 48) and int(im[0, 0, 0]) == 100
