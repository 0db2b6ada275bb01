"""suf_b200 -- B200-native PFSS evaluation engine (host side).

The compute path is libsufb200.so (CUDA, sm_100a) behind the C ABI in
include/sufb200.h; this package binds it (`_lib`) and wraps it (`engine`);
`host/` holds the C++ adapter that implements the reference backend
interface over the same C ABI.
"""
from ._lib import (  # noqa: F401
    GROUP_ADD,
    GROUP_XOR,
    TRUNC_FAITHFUL_ARS,
    TRUNC_FAITHFUL_TR,
    TRUNC_GAPARS,
    SufB200Error,
    TruncDesc,
)

__all__ = ["GROUP_ADD", "GROUP_XOR", "TRUNC_FAITHFUL_TR", "TRUNC_FAITHFUL_ARS", "TRUNC_GAPARS", "SufB200Error",
           "TruncDesc"]
