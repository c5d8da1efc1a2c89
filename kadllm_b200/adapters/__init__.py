"""GRBeam model adapters."""

from .qwen3_5 import NativeGRBeamAdapter, Qwen35GRBeamAdapter

__all__ = ["Qwen35GRBeamAdapter", "NativeGRBeamAdapter"]
