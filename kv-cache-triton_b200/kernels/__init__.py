"""Drop-in replacements for the reference's ``kernels`` package, backed by
hand-written sm_100a CUDA in libkvint4.so (no Triton).

Re-exports the GPT-2 INT4 entry points like the reference's
``kernels/__init__.py:1-5`` (the unquantized ``attention_forward`` is not part
of the INT4 path and is not provided).
"""

from kernels.gpt2.attention_quant import attention_forward_quant
from kernels.gpt2.quantize import dequantize_int4, quantize_int4

__all__ = ["attention_forward_quant", "quantize_int4", "dequantize_int4"]
