"""Where the upstream project's checkout (satyam19k/fast-cuda-cross-attention) is, for test
infrastructure only: the oracle's golden-vector generator, the recipe that compiles the
upstream CUDA sources into oracle/_ref, and the recipe that stages the upstream drivers for
an unchanged run against this library.  Nothing in the product imports this module.

The checkout is taken from the XATTN_UPSTREAM environment variable, else from a directory
named ``reference`` next to this repository's checkout; either must hold the upstream
``cuda_wrappers.py``.  Returns None when there is none (for example on a GPU box, which only
receives what was built and staged here).
"""

import os

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
STAGED = os.path.join(REPO, "oracle", "_ref", "upstream")  # staged upstream drivers


def _is_checkout(path):
    return bool(path) and os.path.isfile(os.path.join(path, "cuda_wrappers.py"))


def upstream_dir():
    env = os.environ.get("XATTN_UPSTREAM")
    if env:
        return env if _is_checkout(env) else None
    sibling = os.path.join(os.path.dirname(REPO), "reference")
    return sibling if _is_checkout(sibling) else None
