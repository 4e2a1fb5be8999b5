from multi_lora_b200.backend.base import LoRABackend
from multi_lora_b200.backend.cuda_backend import CudaLoRABackend
from multi_lora_b200.backend.registry import get_lora_backend

__all__ = ["LoRABackend", "CudaLoRABackend", "get_lora_backend"]
