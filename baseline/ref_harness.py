"""Import the unmodified reference (installed in ``baseline/_ref``) on this image.

The reference's third-party dependencies that are absent here (``diffusers``,
``accelerate``, ``ftfy``, ``imageio``, ``torchdata``) are replaced by minimal
stand-ins registered in ``sys.modules`` *before* the reference is imported;
the reference's own files are not modified.  Stand-ins provide only what the
reference's model / scheduler / distributed code paths touch:
``diffusers.ModelMixin`` (= ``nn.Module``), ``ConfigMixin`` + an identity
``register_to_config``, ``randn_tensor``, ``DiffusionPipeline``;
``accelerate.utils.is_npu_available`` (False); ``ftfy.fix_text`` (identity).
Gloo rejects 0-dim ``all_gather_into_tensor`` inputs that NCCL accepts, so on
Gloo that call is wrapped to reshape scalars to ``[1]``.
"""
from __future__ import annotations

import os
import sys
import types

REF_ROOT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_ref")


def _module(name, **attrs):
    m = types.ModuleType(name)
    for k, v in attrs.items():
        setattr(m, k, v)
    sys.modules[name] = m
    return m


def install_shims():
    import torch
    import torch.nn as nn

    try:
        import diffusers  # noqa: F401
    except Exception:
        class ConfigMixin:
            config_name = "config.json"

        def register_to_config(fn):
            return fn

        class ModelMixin(nn.Module):
            pass

        class DiffusionPipeline:
            def register_modules(self, **kw):
                for k, v in kw.items():
                    setattr(self, k, v)

        def randn_tensor(shape, generator=None, device=None, dtype=None):
            t = torch.randn(shape, generator=generator, dtype=dtype)
            return t.to(device) if device is not None else t

        _module("diffusers")
        _module("diffusers.configuration_utils", ConfigMixin=ConfigMixin, register_to_config=register_to_config)
        _module("diffusers.models")
        _module("diffusers.models.modeling_utils", ModelMixin=ModelMixin)
        _module("diffusers.utils")
        _module("diffusers.utils.torch_utils", randn_tensor=randn_tensor)
        _module("diffusers.pipelines", DiffusionPipeline=DiffusionPipeline)
    try:
        import accelerate  # noqa: F401
    except Exception:
        import transformers  # noqa: F401  (import before the accelerate stand-in)
        _module("accelerate")
        _module("accelerate.utils", is_npu_available=lambda *a, **k: False,
                load=lambda *a, **k: torch.load(*a, **k))
    try:
        import ftfy  # noqa: F401
    except Exception:
        _module("ftfy", fix_text=lambda s: s)
    try:
        import imageio  # noqa: F401
    except Exception:
        _module("imageio")
    try:
        import torchdata  # noqa: F401
    except Exception:
        _module("torchdata")
        _module("torchdata.stateful_dataloader", StatefulDataLoader=torch.utils.data.DataLoader)


def import_reference(disable_compile: bool = False, force_sdpa: bool = False):
    """Return the reference's ``(osp_next module, flow_matching module)``."""
    install_shims()
    if REF_ROOT not in sys.path:
        sys.path.insert(0, REF_ROOT)
    import ospnext.utils.compile as compile_mod
    if disable_compile:
        compile_mod.DISABLE_COMPILE = True
    import ospnext.modules.attention as attn
    if force_sdpa:
        attn.FLASH_ATTN_2_AVAILABLE = False
        attn.FLASH_ATTN_3_AVAILABLE = False
    import ospnext.distributed.communication as comm
    import torch.distributed as dist
    _orig = dist.all_gather_into_tensor

    def _ag(out, inp, group=None, async_op=False):
        if dist.get_backend(group) == "gloo" and inp.dim() == 0:
            return _orig(out.view(-1), inp.view(1), group=group, async_op=async_op)
        return _orig(out, inp, group=group, async_op=async_op)
    comm.dist = types.SimpleNamespace(**{k: getattr(dist, k) for k in dir(dist) if not k.startswith("__")})
    comm.dist.all_gather_into_tensor = _ag
    import ospnext.modules.osp_next as osp
    import ospnext.schedulers.flow_matching as fm
    return osp, fm


def fa2_usable() -> bool:
    """True when the installed flash_attn (FA2) runs on the current GPU.

    The reference prefers FA2 when importable (attention.py:8-27); its wheel may
    lack kernels for this architecture, in which case the reference's own SDPA
    branch is used instead (attention.py:479).
    """
    try:
        import torch
        from flash_attn import flash_attn_func
        q = torch.randn(1, 128, 1, 64, device="cuda", dtype=torch.bfloat16)
        flash_attn_func(q, q, q)
        torch.cuda.synchronize()
        return True
    except Exception:
        return False
