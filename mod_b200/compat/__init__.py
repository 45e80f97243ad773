"""Compatibility surface for code written against the reference's tensor API."""
from .tensor import Tensor

__all__ = ["Tensor"]
