"""B200-native quantized matvec path for GGUF block weights (the hot path of the reference's
ggufengine): activation quantisation, fused dequant + int8 dot products for Q4_0, Q8_0, Q4_K, Q6_K,
TQ2_0 and IQ2_XXS, grouped MoE matvec and row / expert sharding across GPUs.

Module map (reference counterparts in ggufengine/):
    mmvq      -> mmvq.py          Eingang, mv, mm, verfuegbar
    cudakern  -> cudakern.py      expert gather mv, mm, verfuegbar, mm_bis
    qlinear   -> qlinear.py       QuantLinear, build_quant_linear, quantizable
    layers    -> models/common.py PackedLinear, PackedExperts
    moe       -> models/moe.py    MoE FFN, router (models/baukasten.py:_auswahl)
    shard     -> (new)            row-sharded projections and expert-sharded MoE over NCCL
The CUDA kernels sit in csrc/ behind the C ABI of include/nemicli_qmv.h (libnemiqmv.so).
"""
from .formats import FORMATS, TYPE_ID, TYPE_NAME  # noqa: F401

__version__ = "0.1.0"
