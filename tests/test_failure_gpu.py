"""Failure path of the tensor-core kernels, without a GPU fault: a bounded
mbarrier wait that nothing completes gives up, sets the status bit the kernels
report timeouts with, and the context keeps working."""

import pytest
import torch

from kadllm_b200 import _lib

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_and_context_survives():
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    # about 1 ms at B200 clocks
    _lib.call("kadllm_diag_wait_timeout", status.data_ptr(), 2_000_000, _lib.stream(status.device))
    torch.cuda.synchronize()
    assert int(status.item()) == 1
    # the context is still usable: a library kernel and a torch kernel run afterwards
    x = torch.randn(64, 1024, device="cuda").to(torch.bfloat16)
    normed = torch.empty_like(x)
    w = torch.zeros(1024, device="cuda")
    _lib.call("kadllm_add_rmsnorm", x.data_ptr(), None, 0, w.data_ptr(), 1e-6, normed.data_ptr(), 64, 1, 0, 1024,
              _lib.stream(x.device))
    ref = x.float() * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + 1e-6)
    torch.testing.assert_close(normed.float(), ref, rtol=1e-2, atol=1e-2)


def test_engine_check_raises_on_status():
    from kadllm_b200.config import TINY
    from kadllm_b200.model import HybridModel
    from kadllm_b200.synthetic import torch_weights

    engine = HybridModel(TINY, torch_weights(TINY, seed=0, device="cuda"), device="cuda")
    engine.check()  # clean
    _lib.call("kadllm_diag_wait_timeout", engine.status.data_ptr(), 100_000, _lib.stream(engine.device))
    with pytest.raises(RuntimeError, match="timed out"):
        engine.check()


def test_search_raises_on_engine_status():
    """A timed-out tensor-core wait surfaces from the search itself, not only from
    an explicit ``check()``: the drop-in ``grbeam_search`` and the graphed search both raise."""
    from kadllm_b200 import grbeam_search
    from kadllm_b200.adapters import NativeGRBeamAdapter
    from kadllm_b200.config import TINY
    from kadllm_b200.grbeam import GraphedSearch
    from kadllm_b200.model import HybridModel
    from kadllm_b200.synthetic import torch_weights

    engine = HybridModel(TINY, torch_weights(TINY, seed=0, device="cuda"), device="cuda")
    adapter = NativeGRBeamAdapter(engine)
    ids = torch.randint(0, TINY.vocab_size, (2, 16), device="cuda")
    grbeam_search(adapter, ids, [4, 4])  # clean
    graphed = GraphedSearch(adapter, 2, 16, [4, 4], torch.device("cuda"))
    graphed(ids)
    graphed.check()
    _lib.call("kadllm_diag_wait_timeout", engine.status.data_ptr(), 100_000, _lib.stream(engine.device))
    with pytest.raises(RuntimeError, match="timed out"):
        grbeam_search(adapter, ids, [4, 4])
    graphed(ids)
    with pytest.raises(RuntimeError, match="timed out"):
        graphed.check()
