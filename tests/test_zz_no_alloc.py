"""The allocation-free beam selection gives the same results as the workspace one.

Some callers cannot allocate device memory where they select beams (a host
that only lends the library its own tensors, a runtime whose memory budget is
fixed when the model loads).
``kadllm_beam_select_noalloc`` serves them from a fixed scratch array in the
library's device image.  This file is collected last so a failure here does not
hide the rest of the suite; it must pass alone and after the other tests.
"""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _case(seed, B, Wp, V, depth):
    g = torch.Generator(device="cuda").manual_seed(seed)
    logits = (2 * torch.randn(B, Wp, V, device="cuda", generator=g)).to(torch.bfloat16)
    parent = -torch.rand(B, Wp, device="cuda", generator=g) * 3
    hist = torch.randint(0, V, (B, Wp, depth), device="cuda", generator=g)
    return logits, parent, hist


def test_noalloc_matches_workspace_selection_twice():
    from kadllm_b200 import _lib
    from kadllm_b200.grbeam import BeamSelector

    dev = torch.device("cuda")
    cases = [(4, 64, 3000, 48, 2, False), (32, 16, 5000, 16, 1, False), (2, 256, 4096, 64, 1, False),
             (4, 32, 3000, 40, 2, True)]
    for seed, (B, Wp, V, W, depth, masked) in enumerate(cases):
        logits, parent, hist = _case(seed, B, Wp, V, depth)
        mask = None
        if masked:  # a constraint: every third token and all of beam 0 disallowed
            mask = torch.ones(B, Wp, V, dtype=torch.bool, device=dev)
            mask[..., 1::3] = False
            mask[:, 0, :] = False
        ref_scores, ref_hist = BeamSelector(B, Wp, dev).step(logits, parent, hist, W, mask)
        scores = torch.empty(B, W, dtype=torch.float32, device=dev)
        new_hist = torch.empty(B, W, depth + 1, dtype=torch.int64, device=dev)
        flags = torch.ones(1, dtype=torch.int32, device=dev)  # the entry point clears it
        _lib.call("kadllm_beam_select_noalloc", logits.data_ptr(), _lib.dtype_code(logits), V,
                  parent.data_ptr(), None if mask is None else mask.view(torch.uint8).data_ptr(), hist.data_ptr(),
                  scores.data_ptr(), new_hist.data_ptr(),
                  flags.data_ptr(), B, Wp, V, W, depth, _lib.stream(dev))
        torch.cuda.synchronize()
        np.testing.assert_allclose(scores.cpu().numpy(), ref_scores.cpu().numpy(), rtol=0, atol=1e-6)
        np.testing.assert_array_equal(new_hist.cpu().numpy(), ref_hist.cpu().numpy())
        assert int(flags.item()) == 0


def test_noalloc_rejects_sizes_beyond_its_scratch():
    from kadllm_b200 import _lib

    lib = _lib.lib()
    rc = lib.kadllm_beam_select_noalloc(None, 2, 10, None, None, None, None, None,
                                        ctypes.c_void_p(16), 64, 256, 10, 4, 0, None)
    assert rc == 1
    assert b"static" in lib.kadllm_last_error()
