"""Operator wrappers (mirrors ``relmo.ops``)."""

from . import mp

__all__ = ["mp"]
