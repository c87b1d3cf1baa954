"""Optimizers over flat parameter spaces."""

from .adamw import FlatAdamW

__all__ = ["FlatAdamW"]
