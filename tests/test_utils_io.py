"""Padding helpers, inference IO, the compile-decorator stand-in and CUDA-graph sampling."""
import os

import pytest
import torch

from osp_next_b200.utils.graphs import maybe_compile
from osp_next_b200.utils.infer_utils import load_prompts, make_video_grid, save_video_grid, save_videos
from osp_next_b200.utils.padding import pad_input, unpad_input


def test_unpad_pad_roundtrip_and_grad():
    torch.manual_seed(0)
    x = torch.randn(3, 7, 4, 5, requires_grad=True)
    mask = torch.tensor([[1, 1, 1, 0, 0, 0, 0], [1] * 7, [1, 0, 1, 0, 1, 0, 0]], dtype=torch.bool)
    packed, idx, cu, max_s = unpad_input(x, mask)
    assert packed.shape == (int(mask.sum()), 4, 5)
    assert cu.tolist() == [0, 3, 10, 13] and cu.dtype == torch.int32
    assert max_s == 7
    torch.testing.assert_close(packed, x[mask])
    back = pad_input(packed, idx, 3, 7)
    torch.testing.assert_close(back, x * mask[..., None, None])
    g = torch.randn_like(back)
    (back * g).sum().backward()
    torch.testing.assert_close(x.grad, g * mask[..., None, None])


def test_video_grid_layout_and_files(tmp_path):
    v = torch.stack([torch.full((2, 4, 6, 3), 10 * (i + 1), dtype=torch.uint8) for i in range(3)])
    grid = make_video_grid(v)                     # nrow = 2, ncol = 2, cells every (1 + size) pixels
    assert grid.shape == (2, 2 * 5 + 1, 2 * 7 + 1, 3)
    assert int(grid[0, 0, 0, 0]) == 10 and int(grid[0, 0, 7, 0]) == 20 and int(grid[0, 5, 0, 0]) == 30
    assert int(grid[0, 4, 0, 0]) == 0 and int(grid[0, 0, 6, 0]) == 0    # separator row / column
    assert int(grid[0, 5, 7, 0]) == 0             # the empty fourth cell
    save_videos(v, 5, str(tmp_path), fps=8)
    save_video_grid(v, str(tmp_path), fps=8)
    names = sorted(os.listdir(tmp_path))
    assert names == ["video_5.mp4", "video_6.mp4", "video_7.mp4", "video_grid.mp4"]
    assert all(os.path.getsize(tmp_path / n) > 0 for n in names)


def test_load_prompts(tmp_path):
    p = tmp_path / "p.txt"
    p.write_text("a cat\n  a dog  \n")
    assert load_prompts(str(p)) == ["a cat", "a dog"]
    assert load_prompts("a literal prompt") == ["a literal prompt"]


def test_maybe_compile_is_identity():
    def f(x):
        return x + 1
    assert maybe_compile()(f) is f and maybe_compile(disable=True)(f) is f


@pytest.mark.gpu
def test_cuda_graph_sampling_matches_eager():
    from osp_next_b200.models.osp_next import OSPNextModel
    from osp_next_b200.schedulers.flow_matching import FlowMatchingScheduler
    torch.manual_seed(0)
    with torch.device("cuda"):
        m = OSPNextModel(dim=256, ffn_dim=512, num_heads=2, num_layers=8, text_len=16,
                         skiparse_model_type="dual_end", sparse_ratio=2, num_full_blocks=4)
    m = m.to(torch.bfloat16).eval()
    x = torch.randn(1, 16, 3, 16, 16, device="cuda")
    c = torch.randn(1, 16, 4096, device="cuda", dtype=torch.bfloat16)
    u = torch.randn(1, 16, 4096, device="cuda", dtype=torch.bfloat16)
    outs = []
    for graph in (False, True):
        for batch_cfg in (True, False):
            sch = FlowMatchingScheduler(num_inference_steps=6, guidance_scale=5.0)
            sch.batch_cfg = batch_cfg
            with torch.no_grad():
                outs.append(sch.sample(m, x.clone(), c, u, cuda_graph=graph).float())
    for o in outs[1:]:
        rel = (o - outs[0]).norm() / outs[0].norm()
        assert rel < 1e-3, rel
