"""VC attention Config API with a B200 (sm_100a) backend."""

from .core import Config, LayoutCache, attention, expcast_codes

__all__ = ["Config", "LayoutCache", "attention", "expcast_codes"]
