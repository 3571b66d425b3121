"""openasr_b200 -- B200-native (sm_100a) backend for OpenASR's inference hot
path: quantized GGML_OP_MUL_MAT and f16-KV GGML_OP_FLASH_ATTN_EXT behind a C
ABI (include/oasr_b200.h), with a Python host mirror in `backend`."""
from .backend import (  # noqa: F401
    F16, F32, I32, I64, OP_ARGMAX_FIRST, OP_FLASH_ATTN_EXT, OP_MUL_MAT, OP_SET_ROWS, PREC_DEFAULT, PREC_F32, Q4_0,
    Q4_K, Q8_0, Backend, GgmlBackendError, Weight, describe, device_count, lib, quantize, row_size, synth_normal,
)
