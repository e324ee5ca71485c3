"""Drop-in replacements for the reference's kernel modules.

``install()`` registers these modules under the reference's own import names, so
``modeling_llama.py``'s ``from tritonModules import ...`` / ``from deltaFlashAttention
import ...`` / ``from flashAttention import ...`` / ``from deltaDecoding import ...``
(modeling_llama.py:104-112) resolve to the B200 kernels. Alternatively put this directory
first on ``sys.path``.
"""
import importlib
import os
import sys

MODULES = ["tritonModules", "deltaFlashAttention", "flashAttention", "deltaDecoding", "nmDeltaFlashAttention"]
PATH = os.path.dirname(os.path.abspath(__file__))


def install():
    for name in MODULES:
        sys.modules[name] = importlib.import_module(f"{__name__}.{name}")
    return [sys.modules[n] for n in MODULES]
