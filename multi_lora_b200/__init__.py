"""multi_lora_b200 — B200-native (sm_100a) per-token-batch multi-LoRA hot path.

Drop-in for the hot path of Rick0037/multi_lora: segment shrink/expand,
fused RMSNorm and slot-pool adapter loads, behind the reference's Python API
(batch_info / layers / backend / pool), backed by hand-written CUDA kernels in
``libmlora_b200.so`` (C ABI: include/mlora_b200.h) and ``torch.ops.mlora``.
"""

from multi_lora_b200.batch_info import (
    BatchLoRAInfo,
    KernelInputMetaData,
    empty_kernel_input_metadata,
    group_rows,
    segment_lens,
    write_kernel_input_metadata,
)

__all__ = [
    "BatchLoRAInfo",
    "KernelInputMetaData",
    "empty_kernel_input_metadata",
    "group_rows",
    "segment_lens",
    "write_kernel_input_metadata",
]
__version__ = "0.1.0"
