"""metallora_b200 -- B200-native LoRA-linear kernels behind MetalLoRA's API."""

__version__ = "0.1.0"

from .exceptions import (  # noqa: F401
    AdapterError,
    ConfigurationError,
    DeviceError,
    DistributedError,
    MetalLoRAError,
    QuantizationError,
    ShapeError,
    validate_alpha,
    validate_probability,
    validate_rank,
)
from .kernels import is_metal_available, lora_backward_metal, lora_forward_metal  # noqa: F401
from . import torch_ops  # noqa: F401,E402  (registers torch.ops.metal_lora.*)
from .logging import disable_logging, enable_debug, get_logger, logger, set_log_level  # noqa: F401
