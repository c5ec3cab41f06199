"""Recipe that stages the reference's own GPU kernels as a test checker.

Test infrastructure only.  The reference (johnchmura/kv-cache-triton) is
Python + Triton: its GPU quantizer (``kernels/llama3/quantize.py:27-75,
151-186``) and fused GQA decode attention
(``kernels/llama3/attention_quant.py:24-286``), plus the GPT-2 copies
(``kernels/gpt2/quantize.py``, ``kernels/gpt2/attention_quant.py``), cannot
be imported on the GPU box, where the reference checkout does not exist.
This recipe copies those four unmodified files from a reference checkout
into ``oracle/_ref/`` (git-ignored, shipped with the working tree like a
built library), together with a manifest of their SHA-256 digests.  Nothing
in the product imports them: ``oracle/triton_ref.py`` loads them for the
``-m gpu`` parity tests and for ``bench.py``'s reference-kernel timing leg.

    python oracle/ref_recipe.py [REFERENCE_CHECKOUT]
"""

from __future__ import annotations

import hashlib
import json
import os
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
FILES = [
    "kernels/llama3/quantize.py",
    "kernels/llama3/attention_quant.py",
    "kernels/gpt2/quantize.py",
    "kernels/gpt2/attention_quant.py",
]
DEFAULT_SRC = os.environ.get("KV4_REFERENCE_DIR", "/root/reference")


def stage(src: str = DEFAULT_SRC) -> str | None:
    """Copy the reference kernel files into ``oracle/_ref``; returns the output
    directory, or None when no reference checkout is present (the GPU box)."""
    if not all(os.path.isfile(os.path.join(src, f)) for f in FILES):
        return None
    manifest = {}
    for rel in FILES:
        dst = os.path.join(OUT, rel)
        os.makedirs(os.path.dirname(dst), exist_ok=True)
        shutil.copyfile(os.path.join(src, rel), dst)
        with open(dst, "rb") as f:
            manifest[rel] = hashlib.sha256(f.read()).hexdigest()
    with open(os.path.join(OUT, "MANIFEST.json"), "w") as f:
        json.dump({"source": "johnchmura/kv-cache-triton", "files": manifest}, f, indent=1)
    return OUT


if __name__ == "__main__":
    out = stage(sys.argv[1] if len(sys.argv) > 1 else DEFAULT_SRC)
    print(out or "reference checkout not found; nothing staged")
