"""The C-ABI library builds, loads without a GPU and exports every declared symbol."""

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "kadllm_b200.h"


def declared_functions() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(kadllm_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def library():
    from kadllm_b200 import build

    path = build.build()
    return ctypes.CDLL(str(path))


def test_header_declares_entry_points():
    names = declared_functions()
    assert "kadllm_last_error" in names and "kadllm_gated_delta_replay" in names
    assert len(names) >= 4


def test_library_exports_every_declared_symbol(library):
    missing = [n for n in declared_functions() if not hasattr(library, n)]
    assert missing == []


def test_signatures_cover_every_compute_entry_point():
    from kadllm_b200 import _lib

    compute = [n for n in declared_functions()
               if n not in ("kadllm_last_error", "kadllm_abi_version", "kadllm_beam_select_workspace",
                            "kadllm_gdn_prefill_workspace", "kadllm_kv_tile_bytes",
                            "kadllm_beam_select_workspace_fused", "kadllm_attention_split_workspace",
                            "kadllm_gdn_mixer_record_bytes")]
    assert sorted(compute) == sorted(_lib.SIGNATURES)


def test_argument_errors_are_reported_without_a_gpu(library):
    from kadllm_b200 import _lib

    lib = _lib.lib()
    # T = 9 exceeds the replay limit: rejected on the host, before any launch
    rc = lib.kadllm_gated_delta_replay(None, None, None, 2, None, 0, None, 0, None, 2, None,
                                       1, 1, 9, 1, 1, 32, 32, 0.0, None, None)
    assert rc == 3
    assert b"suffix steps" in lib.kadllm_last_error()
    rc = lib.kadllm_gated_delta_replay(None, None, None, 7, None, 0, None, 0, None, 2, None,
                                       1, 1, 1, 1, 1, 32, 32, 0.0, None, None)
    assert rc == 2


def test_mixer_record_bytes_without_a_gpu(library):
    from kadllm_b200 import _lib

    lib = _lib.lib()
    # one fp32 delta per (beam row, value head, value column)
    assert lib.kadllm_gdn_mixer_record_bytes(32, 256, 16, 128) == 32 * 256 * 16 * 128 * 4
    assert lib.kadllm_gdn_mixer_record_bytes(3, 8, 4, 64) == 3 * 8 * 4 * 64 * 4
    assert lib.kadllm_gdn_mixer_record_bytes(0, 8, 4, 64) == 0
    # null operands are refused on the host, before any launch (the record pointer is never read there)
    rc = lib.kadllm_gdn_mixer_replay(None, 0, None, 4, None, None, None, None, None, 1e-6, None, 1, 1, 2, 1, 1, 128,
                                     128, 1, None, None)
    assert rc != 0


def test_mixer_records_need_one_suffix_step(library):
    """First-step records are refused on the host (EUNSUPPORTED) for a two-token replay.
    The pointers are aligned placeholders: the host checks reject the call before any is used."""
    from kadllm_b200 import _lib

    lib = _lib.lib()
    fake = 1 << 20  # 16-byte aligned, never dereferenced on the host
    rc = lib.kadllm_gdn_mixer_replay(fake, 520, fake, 4, fake, fake, fake, fake, fake, 1e-6, fake, 1, 8, 2, 1, 1, 128,
                                     128, fake, fake, None)
    assert rc == 3
    assert b"records" in lib.kadllm_last_error()


def test_gemm_output_row_width_multiple_of_8(library):
    """The GEMM's tensor-map store writes 16-byte granules, so an output row width that is
    not a multiple of 8 (padding past it in a wider row) is refused on the host (EINVAL)."""
    from kadllm_b200 import _lib

    lib = _lib.lib()
    fake = 1 << 20  # 16-byte aligned, never dereferenced on the host
    rc = lib.kadllm_gemm(fake, 64, fake, 64, fake, 64, None, 0, 64, 62, 64, 62, 0, fake, None)
    assert rc == 1
    assert b"multiple of 8" in lib.kadllm_last_error()
