"""Loader for the reference's own Triton kernels staged in ``oracle/_ref``.

Test infrastructure only (the checker, never the product).  The files are the
reference's unmodified ``kernels/{llama3,gpt2}/{quantize,attention_quant}.py``
copied by ``oracle/ref_recipe.py``.  Each is loaded under a private module
name from its file path, so it never shadows this repository's own
``kernels`` package.
"""

from __future__ import annotations

import importlib.util
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.path.join(HERE, "_ref")

_MODS: dict = {}


def available() -> bool:
    return os.path.isfile(os.path.join(REF, "kernels", "llama3", "quantize.py"))


def _load(rel: str):
    if rel in _MODS:
        return _MODS[rel]
    path = os.path.join(REF, rel)
    if not os.path.isfile(path):
        raise ImportError(f"reference kernel file not staged: {path} "
                          "(run oracle/ref_recipe.py where the reference checkout exists)")
    name = "_kv4_ref_" + rel.replace("/", "_").replace(".py", "")
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod  # Triton's JIT looks the module up by name
    spec.loader.exec_module(mod)
    _MODS[rel] = mod
    return mod


def llama3_quantize():
    """``kernels/llama3/quantize.py`` of the reference."""
    return _load("kernels/llama3/quantize.py")


def llama3_attention():
    """``kernels/llama3/attention_quant.py`` of the reference."""
    return _load("kernels/llama3/attention_quant.py")


def gpt2_quantize():
    return _load("kernels/gpt2/quantize.py")


def gpt2_attention():
    return _load("kernels/gpt2/attention_quant.py")
