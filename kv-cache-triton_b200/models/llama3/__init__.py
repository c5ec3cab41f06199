"""Llama 3.1 model glue: quantized KV cache and attention module."""
