"""Offline weight preparation: the reference's byte formats for the W4A8 decode path."""

from asdsl_b200.quantization.core import QuantizedTensor, dequantize_weights, quantize_weights  # noqa: F401
from asdsl_b200.quantization.repack import (  # noqa: F401
    blocks_to_flat,
    repack_asymmetric_to_q4_32_blocks,
    repack_asymmetric_to_q4_128_blocks,
    repack_fp32_to_q4_128_blocks,
    repack_preq_blocks_to_preq2,
)
