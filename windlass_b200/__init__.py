"""windlass_b200 — B200-native (sm_100a) GLM-5.2 DSA indexer + top-k + absorbed-MLA
attention substep behind a C ABI (``include/wl_attn.h``, ``libwl_attn.so``)."""
from ._lib import check_abi, lib  # noqa: F401

__all__ = ["lib", "check_abi"]
