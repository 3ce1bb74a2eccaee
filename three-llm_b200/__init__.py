"""B200-native attention hot path for three-llm.

Exports the host-side mirror of the reference's attention operator
(`CUDAAttention`, the `TSLAttention` surface) and the C-ABI binding of
libtla.so. Import this package as `three_llm_b200` (see `load()` in the
repository's `__graft_entry__.py`).
"""
from ._abi import EXPORTS, LIB_PATH, TlaError, lib  # noqa: F401
from .attention import Context, CUDAAttention, combine_lse, rope_parameters  # noqa: F401
