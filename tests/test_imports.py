"""Every host module imports on a CPU-only machine (no kernel is launched)."""

import importlib

import pytest


@pytest.mark.parametrize("name", ["kadllm_b200", "kadllm_b200.model", "kadllm_b200.adapters", "kadllm_b200.ops",
                                  "kadllm_b200.grbeam", "kadllm_b200.factory", "kadllm_b200.kernel_bench",
                                  "kadllm_b200.roofline", "kadllm_b200.shard", "bench"])
def test_module_imports(name):
    importlib.import_module(name)
