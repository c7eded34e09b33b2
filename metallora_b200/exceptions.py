"""Exception hierarchy and validators of the LoRA API.

Same names and behaviour as the reference (python/metal_lora/exceptions.py:1-71),
so code written against MetalLoRA catches the same errors here.
"""


class MetalLoRAError(Exception):
    """Base exception (exceptions.py:4)."""


class ConfigurationError(MetalLoRAError):
    """Invalid configuration (exceptions.py:9)."""


class ShapeError(MetalLoRAError):
    """Tensor shape, dtype or layout mismatch (exceptions.py:14)."""


class DeviceError(MetalLoRAError):
    """Device or CUDA extension not available (exceptions.py:19)."""


class AdapterError(MetalLoRAError):
    """Adapter-related error (exceptions.py:24)."""


class QuantizationError(MetalLoRAError):
    """Quantization error (exceptions.py:29)."""


class DistributedError(MetalLoRAError):
    """A data-parallel collective failed: a peer rank raised, left or did not
    arrive within the process group's timeout.  The reference is
    single-device and has no counterpart."""


def validate_rank(rank: int, min_rank: int = 1, max_rank: int = 256) -> None:
    """exceptions.py:34-39."""
    if not isinstance(rank, int):
        raise ConfigurationError(f"rank must be int, got {type(rank).__name__}")
    if rank < min_rank or rank > max_rank:
        raise ConfigurationError(f"rank must be in [{min_rank}, {max_rank}], got {rank}")


def validate_alpha(alpha: float) -> None:
    """exceptions.py:42-47."""
    if not isinstance(alpha, (int, float)):
        raise ConfigurationError(f"alpha must be numeric, got {type(alpha).__name__}")
    if alpha <= 0:
        raise ConfigurationError(f"alpha must be positive, got {alpha}")


def validate_shape(tensor, expected_shape: tuple, name: str = "tensor") -> None:
    """exceptions.py:50-53."""
    if tuple(tensor.shape) != tuple(expected_shape):
        raise ShapeError(f"{name} shape mismatch: expected {tuple(expected_shape)}, got {tuple(tensor.shape)}")


def validate_dtype(tensor, expected_dtype, name: str = "tensor") -> None:
    """exceptions.py:56-59."""
    if tensor.dtype != expected_dtype:
        raise ShapeError(f"{name} dtype mismatch: expected {expected_dtype}, got {tensor.dtype}")


def validate_positive(value: float, name: str = "value") -> None:
    """exceptions.py:62-65."""
    if value <= 0:
        raise ConfigurationError(f"{name} must be positive, got {value}")


def validate_probability(value: float, name: str = "probability") -> None:
    """exceptions.py:68-71."""
    if not 0 <= value <= 1:
        raise ConfigurationError(f"{name} must be in [0, 1], got {value}")
