"""B200 (sm_100a) paged-attention hot path: ctypes front end of libpaged_attn_b200.so."""
from ._lib import LIB_PATH, PagedAttnError, load  # noqa: F401
from .ops import paged_attention, write_kv  # noqa: F401

__version__ = "0.1.0"
