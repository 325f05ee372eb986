"""gadeon_b200 -- B200-native paged KV cache for the full-attention layers of
the Qwen3.5 Gated-DeltaNet hybrids (drop-in for leok7v/gadeon's PagePool /
hostFlashDecode path).

The compute lives in libgadeonkv.so (hand-written sm_100a CUDA behind the C
ABI of include/gadeon_kv.h); this package is its Python binding.
"""
from .kv import (  # noqa: F401
    EXPORTED,
    GKV_ATTEND_HEAD_MAJOR,
    GKV_ATTEND_OUT_F16,
    GKV_ATTEND_P_F16,
    GKV_ERR_BAD_SEQ,
    GKV_ERR_CAPACITY,
    GKV_ERR_CUDA,
    GKV_ERR_INVALID,
    GKV_ERR_NO_PAGES,
    GKV_ERR_UNSUPPORTED,
    GKV_OK,
    LIB_PATH,
    BlockPool,
    GkvError,
    PagePool,
    check_bounded_wait,
    conv_rollback,
    gdn_rollback,
    host_flash_decode,
    load_library,
    deserialize,
    mtp_rollback,
    paged_flash_batched,
    read_state_header,
    rope_table,
    serialize,
    state_header,
    verify_attn,
)
