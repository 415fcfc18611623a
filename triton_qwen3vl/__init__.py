"""Drop-in import name: ``from triton_qwen3vl import install_qwen3vl_triton_attention``
(evaluation_wrapper.py:382 in the reference project) resolves to the sm_100a
backend in :mod:`aicas_b200`.  The package contains no Triton; the name is kept
so the reference's callers need no edit."""
import sys as _sys

from aicas_b200 import *  # noqa: F401,F403
from aicas_b200 import __all__  # noqa: F401
from aicas_b200 import backends, ops, patch  # noqa: F401

# the reference's submodule paths used by callers and tests
_sys.modules[__name__ + ".backends"] = backends
_sys.modules[__name__ + ".patch"] = patch
_sys.modules[__name__ + ".ops"] = ops
