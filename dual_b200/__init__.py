"""dual_b200 -- B200-native (sm_100a) tiered paged-KV attention hot path of Eyan-L/Dual.

Paged GQA decode over a KV pool split between local HBM and supplier GPUs'
HBM (read by direct peer loads over NVLink), the read-order packer for the
per-request tier/slot page tables, and the token-slot migration copy, behind
the FlashInfer wrapper API the reference patches (``wrapper``) and a C ABI
(``include/dual_b200.h``, library ``dual_b200/lib/libdual_b200.so``).
"""
from . import _lib, ops  # noqa: F401
from .wrapper import BatchDecodeWithPagedKVCacheWrapper, BatchPrefillWithPagedKVCacheWrapper, activate  # noqa: F401
from .remote_bank import RemoteBank, local_plane_pointers  # noqa: F401

__all__ = ["BatchDecodeWithPagedKVCacheWrapper", "BatchPrefillWithPagedKVCacheWrapper", "activate", "RemoteBank", "local_plane_pointers", "ops"]
