"""GGUF block formats of the quantized matvec path.

GGML type ids and block geometry follow the GGUF format (the reference's table is
ggufengine/gguf.py:64-77).  Only the twenty-six formats of the hot path have kernels here; asking for any
other format raises instead of computing elsewhere.
"""
from __future__ import annotations

# name -> (values per block, bytes per block)
FORMATS = {
    "Q4_0": (32, 18),
    "Q4_1": (32, 20),
    "Q5_0": (32, 22),
    "Q5_1": (32, 24),
    "IQ4_NL": (32, 18),
    "Q1_0": (128, 18),
    "Q2_0": (64, 18),
    "PQ2_0": (128, 34),
    "Q8_0": (32, 34),
    "Q2_K": (256, 84),
    "Q3_K": (256, 110),
    "Q4_K": (256, 144),
    "Q5_K": (256, 176),
    "Q6_K": (256, 210),
    "IQ2_XXS": (256, 66),
    "IQ2_XS": (256, 74),
    "IQ2_S": (256, 82),
    "IQ3_XXS": (256, 98),
    "IQ3_S": (256, 110),
    "IQ4_XS": (256, 136),
    "TQ2_0": (256, 66),
    "TQ1_0": (256, 54),
    "MXFP4": (32, 17),
    "IQ1_S": (256, 50),
    "IQ1_M": (256, 56),
    "PTQ1_0": (128, 28),
}

# name -> GGML type id
TYPE_ID = {"Q4_0": 2, "Q4_1": 3, "Q5_0": 6, "Q5_1": 7, "IQ4_NL": 20, "Q1_0": 41, "Q2_0": 42, "PQ2_0": 142, "Q2_K": 10, "Q3_K": 11, "TQ1_0": 34, "IQ2_XS": 17, "IQ2_S": 22, "Q8_0": 8, "Q4_K": 12, "Q5_K": 13, "Q6_K": 14, "IQ2_XXS": 16, "IQ3_XXS": 18, "IQ3_S": 21, "IQ4_XS": 23, "TQ2_0": 35, "MXFP4": 39,
           "IQ1_S": 19, "IQ1_M": 29, "PTQ1_0": 143}
TYPE_NAME = {v: k for k, v in TYPE_ID.items()}

# GGML types the reference knows but this path does not compute (for clear refusals)
GGML_TYPES = {
    0: ("F32", 1, 4), 1: ("F16", 1, 2), 2: ("Q4_0", 32, 18), 3: ("Q4_1", 32, 20),
    6: ("Q5_0", 32, 22), 7: ("Q5_1", 32, 24), 8: ("Q8_0", 32, 34), 9: ("Q8_1", 32, 36),
    10: ("Q2_K", 256, 84), 11: ("Q3_K", 256, 110), 12: ("Q4_K", 256, 144),
    13: ("Q5_K", 256, 176), 14: ("Q6_K", 256, 210), 15: ("Q8_K", 256, 292),
    16: ("IQ2_XXS", 256, 66), 17: ("IQ2_XS", 256, 74), 18: ("IQ3_XXS", 256, 98),
    19: ("IQ1_S", 256, 50), 20: ("IQ4_NL", 32, 18), 21: ("IQ3_S", 256, 110),
    22: ("IQ2_S", 256, 82), 23: ("IQ4_XS", 256, 136), 24: ("I8", 1, 1),
    25: ("I16", 1, 2), 26: ("I32", 1, 4), 27: ("I64", 1, 8), 28: ("F64", 1, 8),
    29: ("IQ1_M", 256, 56), 30: ("BF16", 1, 2), 34: ("TQ1_0", 256, 54),
    35: ("TQ2_0", 256, 66), 39: ("MXFP4", 32, 17), 41: ("Q1_0", 128, 18), 42: ("Q2_0", 64, 18),
    142: ("PQ2_0", 128, 34), 143: ("PTQ1_0", 128, 28),
}


def name_of(fmt) -> str:
    """Format name from a name or a GGML type id."""
    if isinstance(fmt, str):
        return fmt
    return GGML_TYPES[int(fmt)][0]


def row_bytes(fmt: str, n_in: int) -> int:
    bv, bb = FORMATS[fmt]
    return n_in // bv * bb


def supported(fmt) -> bool:
    return name_of(fmt) in FORMATS
