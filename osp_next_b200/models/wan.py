"""Dense Wan-2.1 DiT (registry name ``wan_t2v``; reference: ospnext/modules/want2v.py:291-519).

Every block is a full-attention block, i.e. the OSP-Next model with
``skiparse_model_type="full"``; parameter names are identical to Wan-2.1's.
"""
from .osp_next import Head, OSPNextAttentionBlock, OSPNextModel, WanLayerNorm, WanRMSNorm, sinusoidal_embedding_1d


class WanModel(OSPNextModel):
    def __init__(self, model_type="t2v", patch_size=(1, 2, 2), text_len=512, in_dim=16, dim=2048, ffn_dim=8192,
                 freq_dim=256, text_dim=4096, out_dim=16, num_heads=16, num_layers=32, window_size=(-1, -1),
                 qk_norm=True, cross_attn_norm=True, eps=1e-6, **kwargs):
        kwargs.pop("skiparse_model_type", None)
        super().__init__(model_type=model_type, patch_size=patch_size, text_len=text_len, in_dim=in_dim, dim=dim,
                         ffn_dim=ffn_dim, freq_dim=freq_dim, text_dim=text_dim, out_dim=out_dim, num_heads=num_heads,
                         num_layers=num_layers, window_size=window_size, qk_norm=qk_norm,
                         cross_attn_norm=cross_attn_norm, eps=eps, skiparse_model_type="full", **kwargs)


WanAttentionBlock = OSPNextAttentionBlock
models = {"wan_t2v": WanModel}
models_main_block = {"wan_t2v": OSPNextAttentionBlock}
models_blocks_to_float = {"wan_t2v": [WanLayerNorm, WanRMSNorm]}
models_blocks_to_output_float = {"wan_t2v": None}
__all__ = ["WanModel", "Head", "sinusoidal_embedding_1d"]
