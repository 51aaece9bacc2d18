"""Drop-in import name: ``import rdnattention`` resolves to the B200 build.

The reference's public API (rdnattention/__init__.py:360-363 of
dmonkman/RDNAttention) re-exported from :mod:`rdnattention_b200`.
"""
from rdnattention_b200 import *  # noqa: F401,F403
from rdnattention_b200 import (RDNAttentionError, SUPPORTED_HEAD_DIMS, SUPPORTED_HEAD_DIMS_INT8, __all__,  # noqa: F401
                               __version__, flash_attn, flash_attn_int8qk, flash_attn_int8qk_quantized, has_device,
                               quantize_int8_perchannel_v, quantize_int8_qk_pertoken)
