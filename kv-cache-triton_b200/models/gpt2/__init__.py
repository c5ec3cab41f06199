"""GPT-2 model glue: quantized KV cache and attention module."""

__all__ = []
