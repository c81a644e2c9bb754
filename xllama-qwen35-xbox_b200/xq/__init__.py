"""Host-side mirror of the reference's attention-path interface on B200.

The ggml ops GGML_OP_FLASH_ATTN_EXT and GGML_OP_GATED_DELTA_NET, the RKVA
range-attention call (RemoteAttnEngine::attend_range) and the split-partial /
LSE-merge pair, each a thin wrapper over one C-ABI entry point of
libxq_b200.so (include/xq_b200.h).  torch supplies device memory and streams;
every computation runs in the CUDA library.
"""
from ._lib import F16, F32, I32, I64, Q4_0, Q8_0, XqError, lib  # noqa: F401
from .ops import (attend_range, flash_attn_ext_plan, attend_range_kvarn4, attend_range_workspace,  # noqa: F401
                  dequantize_rows, fa_partials, flash_attn_ext, flash_attn_ext_workspace, gated_delta_net,
                  lse_merge, lse_merge_records, quantize_rows, row_bytes, set_rows, split_k)
