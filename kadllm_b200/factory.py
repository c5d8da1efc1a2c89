"""Adapter factory for the reference's benchmark runner.

``benchmarks/grbeam.py --backend external --adapter-factory kadllm_b200.factory:make``
passes the loaded ``Qwen3_5ForConditionalGeneration``; ``make`` returns
``(adapter, search)`` (the runner's contract, ``benchmarks/grbeam.py:219-223``).
"""

from __future__ import annotations

from .adapters import Qwen35GRBeamAdapter
from .grbeam import grbeam_search


def make(model):
    text = model.model.language_model if hasattr(model, "model") else model
    return Qwen35GRBeamAdapter(text.eval(), model.lm_head.eval()), grbeam_search
