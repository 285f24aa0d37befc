"""pi05_pytorch_fast_b200: the W4A4 prefix-LM path of pi05-pytorch-fast,
rebuilt for NVIDIA B200 (sm_100a).

Importing the package registers the ``pi05_w4a4::*`` custom ops on the B200
kernels (libw4a4_sm100.so, built by ``python -m pi05_pytorch_fast_b200.build``).
``prefix_lm.W4A4PrefixLM`` is the whole W4A4 Gemma prefix LM on those kernels.
"""

from . import w4a4  # noqa: F401  (registers the ops)

__version__ = "0.2.0"
