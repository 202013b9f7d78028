"""Fake quantisation: HiF8 linears / attention (the OSP-Next model's quant path, hif8.py)
and the rest of the quant_cy_npu library surface (layers.py)."""
from .hif8 import (HIF8Linear, QLinear, QType, hif8_multi_linear, hif8_qkv, quant, quant_dequant_float,  # noqa: F401
                   quant_hif8, replace_linear)
from .layers import BlockFloatFormat, QConv2d, QSLinear, SLinear, quant_block_float, quant_py  # noqa: F401
