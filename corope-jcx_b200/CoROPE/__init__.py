"""CoROPE -- B200-native CoRoPE attention with the call surface of the
reference package of the same name (N1-research/CoRoPE-jcx ``CoROPE/``).

    from CoROPE.forward import co_rope_forward
    from CoROPE.co_rope_backward import co_rope_backward
    from CoROPE.co_rope_mqa_forward import co_rope_mqa_forward
    from CoROPE.co_rope_attn import CoRoPEAttentionFunction, CoRoPEAttention
    from CoROPE.flash import flash_attention       # plain attention baseline

All compute runs in libcorope_b200.so (sm_100a CUDA kernels behind a C ABI,
include/corope.h); there is no CPU path.
"""
from .co_rope_attn import CoRoPEAttention, CoRoPEAttentionFunction
from .co_rope_backward import co_rope_backward
from .co_rope_mqa_forward import co_rope_mqa_forward
from .flash import FlashAttention, flash_attention
from .forward import co_rope_forward
from ._lib import load_library, LIB_PATH

__all__ = ["co_rope_forward", "co_rope_backward", "co_rope_mqa_forward",
           "CoRoPEAttentionFunction", "CoRoPEAttention", "flash_attention", "FlashAttention",
           "load_library", "LIB_PATH"]
