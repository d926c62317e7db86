"""Module alias: the reference's autograd wrapper and benchmark import
``CoROPE.co_rope_forward`` (CoROPE/co_rope_attn.py:2, benchmark.py:89), a
module that the reference does not ship; here it re-exports the forward."""
from .forward import co_rope_forward  # noqa: F401

__all__ = ["co_rope_forward"]
