"""bench.py's training-mode configuration (no GPU): layouts, overrides and the
synthetic-data shapes handed to the public trainer."""
import argparse
import importlib.util
import os

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench():
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_train_layouts_and_overrides(tmp_path):
    b = _bench()
    assert b.train_layout(1) == (1, 1) and b.train_layout(4) == (4, 4) and b.train_layout(8) == (8, 4)
    args = argparse.Namespace(model="14b", frames=81, height=768, width=1280, warmup=2, steps=3, quant="hif8",
                              loss_log=None, fsdp_comm="p2p")
    cfg = b.train_config(args, 8, str(tmp_path))
    assert cfg["fsdp_size"] == 8 and cfg["skiparse_sp_size"] == 4 and cfg["use_skiparse_sequence_parallel"]
    assert cfg["max_steps"] == 5 and cfg["gradient_checkpointing"] and cfg["fsdp_p2p_collectives"]
    mc = cfg["model_config"]
    assert mc["dim"] == 5120 and mc["num_layers"] == 40 and mc["num_full_blocks"] == 8 and mc["quant"] == "hif8"
    assert "pretrained_model_dir_or_checkpoint" not in mc
    dc = cfg["data_config"]
    assert dc["dataset_name"] == "t2v_random_latent"
    assert dc["dataset_config"] == dict(sample_height=768, sample_width=1280, sample_num_frames=81,
                                        text_max_length=512)


def test_inference_layouts_and_tokens():
    b = _bench()
    assert [b.layout_for(n) for n in (1, 2, 4, 8)] == [(1, 1), (2, 1), (2, 2), (2, 4)]
    args = argparse.Namespace(frames=81, height=768, width=1280)
    assert b.latent_shape(args) == (1, 16, 21, 96, 160)
    assert b.tokens(args) == 80640
