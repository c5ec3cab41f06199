"""Llama 3.1 INT4 KV-cache kernels (sm_100a CUDA via libkvint4.so)."""
