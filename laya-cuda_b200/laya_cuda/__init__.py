"""Laya decision-model inference on NVIDIA B200 (sm_100a).

Importing the package is light: the execution library and the official SDK load only when an
Engine is constructed.
"""
from .engine import Engine
from .batching import BatchEngine

__all__ = ["Engine", "BatchEngine"]
__version__ = "0.1.0"
