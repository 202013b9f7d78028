"""VideoAlign reward model: prompt templates and frame sampling / resize rules against the
reference's functions, and checkpoint loading (training-time key names, LoRA merge, reward
head) plus special-token pooling on a tiny random Qwen2-VL (CPU)."""
import importlib
import json
import os
import sys

import pytest
import torch

from osp_next_b200.rewards import videoalign as va

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _ref_module(name):
    ref_root = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_root, "ospnext")):
        pytest.skip("reference not installed in baseline/_ref")
    sys.path.insert(0, ref_root)
    try:
        return importlib.import_module(f"ospnext.rewards.{name}")
    except ImportError as e:
        pytest.skip(f"reference module not importable here: {e}")


def test_prompts_match_reference():
    ref = _ref_module("videoalign_prompt_template")
    for t in ("none", "simple", "video_score", "detailed", "detailed_special"):
        for dim in ("VQ", "MQ", "TA", "Overall", ["VQ", "MQ", "TA"]):
            assert va.build_prompt("a cat surfing", dim, t) == ref.build_prompt("a cat surfing", dim, t), (t, dim)


def test_resize_and_frame_counts_match_reference():
    ref = _ref_module("videoalign_vision_process")
    for h, w in ((480, 832), (768, 1280), (33, 900), (1080, 1920), (50, 60)):
        for mx in (240 * 320, 448 * 448, ref.VIDEO_MAX_PIXELS):
            assert va.vl_resize(h, w, max_pixels=mx) == ref.smart_resize(
                h, w, factor=28, min_pixels=ref.VIDEO_MIN_PIXELS, max_pixels=mx), (h, w, mx)
    for total, vfps in ((33, 8.0), (81, 16.0), (200, 24.0)):
        for ele in ({"nframes": 8}, {"nframes": 15}, {"fps": 2.0}, {"fps": 4.0}):
            n = ref.smart_nframes(dict(ele), total_frames=total, video_fps=vfps)
            idx = va.frame_indices(total, vfps, nframes=ele.get("nframes"), fps=ele.get("fps"))
            assert len(idx) == n
            assert idx == torch.linspace(0, total - 1, n).round().long().tolist()


def _tiny_vl():
    from transformers import Qwen2VLConfig, Qwen2VLForConditionalGeneration
    cfg = Qwen2VLConfig(
        text_config=dict(vocab_size=300, hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                         num_attention_heads=4, num_key_value_heads=2,
                         rope_scaling={"type": "mrope", "mrope_section": [2, 3, 3]}, max_position_embeddings=512),
        vision_config=dict(depth=1, embed_dim=32, hidden_size=64, num_heads=2, mlp_ratio=2, patch_size=14,
                           spatial_merge_size=2, temporal_patch_size=2, in_channels=3),
        image_token_id=290, video_token_id=291, vision_start_token_id=292, vision_end_token_id=293)
    torch.manual_seed(0)
    return Qwen2VLForConditionalGeneration(cfg).eval()


def test_checkpoint_merge_and_special_token_pooling():
    vl = _tiny_vl()
    model = va.VideoAlignRewardModel(vl, output_dim=3, special_token_ids=[295, 296, 297], pad_token_id=0)
    base = model.state_dict_for_checkpoint()
    wkey = "model.language_model.layers.0.self_attn.q_proj.weight"
    A, Bm = torch.randn(4, 64), torch.randn(64, 4)
    head = torch.randn(3, 64)
    vis = torch.randn_like(base["model.visual.patch_embed.proj.weight"])
    tensors = {   # names as the VideoAlign trainer saves them (PEFT wrapper, pre-5.x layout)
        "base_model.model.model.layers.0.self_attn.q_proj.lora_A.default.weight": A,
        "base_model.model.model.layers.0.self_attn.q_proj.lora_B.default.weight": Bm,
        "base_model.model.rm_head.weight": head,
        "base_model.model.visual.patch_embed.proj.weight": vis,
    }
    sd = va.merge_training_state(base, tensors, lora_scale=2.0)
    assert torch.allclose(sd[wkey], base[wkey] + 2.0 * Bm @ A, atol=1e-5)
    assert torch.equal(sd["rm_head.weight"], head) and torch.equal(sd["model.visual.patch_embed.proj.weight"], vis)
    model.load_checkpoint_tensors(sd)
    assert torch.equal(model.rm_head.weight.detach(), head)
    ids = torch.randint(3, 280, (2, 24))
    ids[:, 10], ids[:, 15], ids[:, 20] = 295, 296, 297
    with torch.no_grad():
        out = model(ids, attention_mask=torch.ones_like(ids))
        h = vl.model(input_ids=ids, attention_mask=torch.ones_like(ids)).last_hidden_state
    assert out.shape == (2, 3)
    exp = torch.stack([h[:, 10] @ head[0], h[:, 15] @ head[1], h[:, 20] @ head[2]], 1)
    assert torch.allclose(out, exp, atol=1e-4)


def test_config_and_checkpoint_discovery(tmp_path):
    cfg = {"data_config": {"meta_data": "x", "data_dir": "y", "eval_dim": ["VQ", "MQ", "TA"], "fps": 2.0,
                           "max_frame_pixels": 76800, "prompt_template_type": "detailed_special"},
           "model_config": {"model_name_or_path": "/models/qwen2-vl", "output_dim": 3, "use_special_tokens": True,
                            "reward_token": "special"},
           "peft_lora_config": {"lora_enable": True, "lora_r": 64, "lora_alpha": 128},
           "inference_config": {"VQ_mean": 1.0, "VQ_std": 2.0, "MQ_mean": 0.0, "MQ_std": 1.0, "TA_mean": 0.5,
                                "TA_std": 0.5}}
    (tmp_path / "model_config.json").write_text(json.dumps(cfg))
    for s in (100, 2000, 300):
        (tmp_path / f"checkpoint-{s}").mkdir()
    c = va.VideoAlignConfig.from_dir(str(tmp_path))
    assert c.output_dim == 3 and c.use_special_tokens and c.lora_alpha == 128 and c.norm["VQ_std"] == 2.0
    assert va.find_checkpoint(str(tmp_path)).endswith("checkpoint-2000")
    assert va.find_checkpoint(str(tmp_path), 300).endswith("checkpoint-300")
    sc = va.VideoAlignScorer.__new__(va.VideoAlignScorer)
    sc.cfg, sc.use_norm = c, True
    s = sc.normalise({"VQ": 3.0, "MQ": 1.0, "TA": 1.0})
    assert s == {"VQ": 1.0, "MQ": 1.0, "TA": 1.0, "Overall": 3.0}
