"""Mix-GRPO trainer end to end on CPU Gloo ranks (tiny model, synthetic prompts).

One epoch on 2 ranks with the policy FSDP2-sharded, the KL-to-reference loss (kl_beta)
and KL reward (kl_reward) through the adapter-disabled model, two inner epochs in
micro-batches with gradient accumulation, zero-advantage selection, the EMA eval loop,
checkpointing, and a resume that continues from the saved epoch.
"""
import json
import os
import socket
import sys
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _config(out_dir, fsdp, epochs=1, lora_path=None, resume_epoch=None):
    cfg = {
        "model_name": "osp_next", "seed": 3, "output_dir": out_dir, "num_epochs": epochs, "save_interval": 1000,
        "weight_dtype": "fp32", "ema_decay": 0.9, "init_max_grad_norm": 1.0, "fsdp_size": fsdp,
        "metrics_file": os.path.join(out_dir, "metrics.jsonl"), "gradient_accumulation_steps": 1,
        "model_config": dict(dim=128, ffn_dim=256, num_heads=4, num_layers=2, text_len=16, in_dim=16, out_dim=16,
                             skiparse_model_type="dual_end", sparse_ratio=2, num_full_blocks=0),
        "scheduler_config": {"scheduler_name": "flow_matching", "shift": 1.0},
        "lora_config": {"rank": 4, "alpha": 8, "target_modules": ["self_attn.q", "self_attn.v", "ffn.0"]},
        "rl_config": dict(synthetic_prompts=True, num_prompts=8, height=64, width=64, num_frames=5,
                          num_inference_steps=3, sde_steps=2, guidance_scale=3.0, kl_beta=0.1, kl_reward=0.1,
                          num_batches_per_epoch=1, num_image_per_prompt=2, sample_batch_size=2, train_batch_size=1,
                          num_inner_epochs=2, timestep_fraction=1.0, clip_range=0.2, adv_clip_max=5.0,
                          use_cfg_in_train=True, per_prompt_stat_tracking=True, reward_fn={"latent_mlp": 1.0},
                          eval_freq=1, eval_num_steps=2, num_eval_prompts=2),
        "optimizer_config": {"lr": 1e-3, "weight_decay": 0.0},
    }
    if lora_path:
        cfg["lora_config"]["lora_path"] = lora_path
    if resume_epoch is not None:
        cfg["resume_epoch"] = resume_epoch
    return cfg


def _worker(rank, world, port, cfg, res_file):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    sys.path.insert(0, os.path.join(ROOT, "train"))
    import train_osp_RL
    policy = train_osp_RL.main(cfg)
    n = sum(p.numel() for n_, p in policy.named_parameters() if "lora_" in n_)
    if rank == 0:
        with open(res_file, "w") as f:
            json.dump({"lora_numel_local": n}, f)
    dist.barrier()
    dist.destroy_process_group()


def _run(world, cfg):
    with tempfile.NamedTemporaryFile(suffix=".json", delete=False) as tf:
        res = tf.name
    mp.start_processes(_worker, args=(world, _port(), cfg, res), nprocs=world, join=True, start_method="spawn")
    with open(res) as f:
        return json.load(f)


def _records(out_dir):
    with open(os.path.join(out_dir, "metrics.jsonl")) as f:
        return [json.loads(l) for l in f]


@pytest.mark.parametrize("fsdp", [2, 1])
def test_rl_epoch_kl_inner_epochs_eval_resume(fsdp):
    with tempfile.TemporaryDirectory() as d:
        _run(2, _config(d, fsdp))
        recs = _records(d)
        steps = [r for r in recs if "policy_loss" in r]
        # 2 prompts × 2 repeats over 2 ranks → 2 samples per rank, 2 trained SDE steps, 2 inner
        # epochs, micro-batches of 1, accumulation over the 2 timesteps → 4 optimizer steps
        assert len(steps) == 4
        for r in steps:
            for key in ("kl_loss", "approx_kl", "clipfrac", "policy_loss", "loss", "grad_norm"):
                assert key in r and r[key] == r[key], key
        ep = [r for r in recs if "zero_std_ratio" in r]
        assert len(ep) == 1 and "kl" in ep[0] and ep[0]["samples_kept"] <= ep[0]["samples_total"]
        ck = os.path.join(d, "lora-checkpoint-4")
        assert os.path.exists(os.path.join(ck, "adapter_model.bin"))
        assert os.path.exists(os.path.join(d, "lora-checkpoint-4-ema", "adapter_model.bin"))
        with open(os.path.join(ck, "rl_training_state.json")) as f:
            assert json.load(f) == {"global_step": 4, "next_epoch": 1}
        sd = torch.load(os.path.join(ck, "adapter_model.bin"), weights_only=True)
        assert any(k.startswith("base_model.model.blocks.0.self_attn.q.lora_A.default") for k in sd)
        assert all(v.shape[0] in (4, 128, 256) for v in sd.values())          # full (unsharded) tensors
        evals = os.listdir(os.path.join(d, "eval"))
        assert evals and all(e.startswith("step_") for e in evals)
        # resume: the next epoch continues the step count from the checkpoint
        _run(2, _config(d, fsdp, epochs=2, lora_path=ck))
        with open(os.path.join(d, "lora-checkpoint-8", "rl_training_state.json")) as f:
            assert json.load(f) == {"global_step": 8, "next_epoch": 2}


def test_select_samples_pads_to_batch_multiple():
    sys.path.insert(0, os.path.join(ROOT, "train"))
    import train_osp_RL
    g = torch.Generator().manual_seed(0)
    adv = torch.tensor([[0.5, 0.5], [0.0, 0.0], [1.0, 1.0], [0.0, 0.0], [0.0, 0.0]])
    m = train_osp_RL.select_samples(adv.clone(), 2, g)
    assert int(m.sum()) == 2 and bool(m[0]) and bool(m[2])
    m = train_osp_RL.select_samples(adv.clone(), 3, g)
    assert int(m.sum()) == 3 and bool(m[0]) and bool(m[2])
    m = train_osp_RL.select_samples(torch.zeros(4, 2), 3, g)
    assert bool(m.all())
