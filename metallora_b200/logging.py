"""Package logger, shaped like the reference's (python/metal_lora/logging.py:1-43):
logger name ``metal_lora``, stdout handler, INFO by default."""

import logging
import sys


def get_logger(name: str = "metal_lora", level: int | None = None) -> logging.Logger:
    logger = logging.getLogger(name)
    if not logger.handlers:
        handler = logging.StreamHandler(sys.stdout)
        handler.setFormatter(logging.Formatter(
            "%(asctime)s - %(name)s - %(levelname)s - %(message)s", datefmt="%Y-%m-%d %H:%M:%S"))
        logger.addHandler(handler)
    if level is not None:
        logger.setLevel(level)
    elif logger.level == logging.NOTSET:
        logger.setLevel(logging.INFO)
    return logger


def set_log_level(level: int) -> None:
    get_logger().setLevel(level)


def enable_debug() -> None:
    set_log_level(logging.DEBUG)


def disable_logging() -> None:
    set_log_level(logging.CRITICAL + 1)


logger = get_logger()
