"""Model registries (reference: ospnext/modules/__init__.py:13-48)."""
from . import osp_next as _osp
from . import wan as _wan

models = {}
models.update(_wan.models)
models.update(_osp.models)

models_main_block = {}
models_main_block.update(_wan.models_main_block)
models_main_block.update(_osp.models_main_block)

models_blocks_to_float = {}
models_blocks_to_float.update(_wan.models_blocks_to_float)
models_blocks_to_float.update(_osp.models_blocks_to_float)

models_blocks_to_output_float = {}
models_blocks_to_output_float.update(_wan.models_blocks_to_output_float)
models_blocks_to_output_float.update(_osp.models_blocks_to_output_float)


def __getattr__(name):
    # heavy optional modules are imported lazily
    if name in ("T5EncoderModel", "T5Encoder", "T5Model", "T5Decoder"):
        from . import t5
        return getattr(t5, name)
    if name == "WanVAE":
        from .vae import WanVAE
        return WanVAE
    if name == "HuggingfaceTokenizer":
        from .tokenizers import HuggingfaceTokenizer
        return HuggingfaceTokenizer
    raise AttributeError(name)
