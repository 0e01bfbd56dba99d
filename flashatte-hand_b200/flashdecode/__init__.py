"""flashdecode: B200 (sm_100a) paged-KV GQA flash-decode operator.

Host side of ``libflashdecode_sm100.so`` (C ABI in include/flashdecode.h).
Put the ``flashatte-hand_b200`` directory on ``sys.path`` and
``import flashdecode``.
"""
from ._lib import FlashDecodeError, LIB_PATH, load_library
from .ops import (DecodePlan, append_kv, combine_lse, device_status, flash_decode, last_error,
                  run_kernel, workspace_size)

__all__ = ["FlashDecodeError", "LIB_PATH", "load_library", "DecodePlan", "append_kv", "combine_lse",
           "device_status", "flash_decode", "last_error", "run_kernel", "workspace_size"]
