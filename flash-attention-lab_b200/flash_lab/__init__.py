"""flash_lab on B200: the attention operators of tfan2437/flash-attention-lab (flash_lab.attention,
flash_lab.decode, torch.ops.flash_lab::*, the Hugging Face backend in flash_lab.hf) backed by
hand-written sm_100a kernels behind a C ABI (include/flash_lab_b200.h)."""

from flash_lab import reference
from flash_lab.ops import attention, available_impls, decode

__version__ = "0.1.0"
__all__ = ["attention", "available_impls", "decode", "reference"]
