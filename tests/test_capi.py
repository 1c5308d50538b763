"""The C ABI (include/jeffb200.h) on the CPU: the library loads without a GPU, exports every declared entry point,
and refuses bad arguments with JB_EINVAL and a message before touching the device."""

from __future__ import annotations

import ctypes

import pytest

from jeff_b200 import _lib


@pytest.fixture(scope="module")
def lib() -> ctypes.CDLL:
    from jeff_b200 import build

    build.build()
    return _lib.load()


def test_every_declared_entry_point_is_exported(lib: ctypes.CDLL) -> None:
    names = _lib.header_symbols()
    assert len(names) >= 19
    for name in names:
        assert hasattr(lib, name), name
    assert lib.jb_abi_version() == 2


def test_bad_arguments_are_refused_before_any_launch(lib: ctypes.CDLL) -> None:
    p = ctypes.c_void_p(16)
    # k not a multiple of 64
    assert lib.jb_w4a16_lora(p, 64, 100, p, p, None, 64, 128, 128, None, None, 0, 0, None, 64, p, 128, 0, None) == -1
    assert b"multiple of 64" in lib.jb_last_error()
    # group must be 64 or 128
    assert lib.jb_int4_dequant(p, p, None, 128, 128, 32, p, None) == -1
    assert b"group" in lib.jb_last_error()
    # a pass must hold whole rows
    assert lib.jb_gdn_prep_rows(p, 8224, 100, 32, p, 393216, p, 434, 48, 0, p, p, p, p, p, p, p, p, None, None, 0,
                                None) == -1
    assert b"rows of 32" in lib.jb_last_error()
    # rows whose length is not a multiple of 128 gather the LoRA expand from a per-tile set of at most 256 pool rows,
    # kept for at most 128 row tiles (32768 tokens)
    assert lib.jb_w4a16_lora(p, 128, 1024, p, p, None, 64, 128, 128, p, p, 16, 300, p, 1, p, 128, 0, None) == -1
    assert b"at most 256" in lib.jb_last_error()
    assert lib.jb_w4a16_lora(p, 40000, 1024, p, p, None, 64, 128, 128, p, p, 16, 3, p, 48, p, 128, 0, None) == -1
    assert b"at most 32768 tokens" in lib.jb_last_error()
    # K not a multiple of 128 takes the 16-row shrink, whose blocks hold one adapter each
    assert lib.jb_lora_shrink(p, 32, 64, p, 16, 1, p, 1, p, None) == -1
    assert b"multiples of 16" in lib.jb_last_error()
    with pytest.raises(_lib.ArgumentError, match="rank 20"):
        _lib.call("jb_lora_shrink", p, 32, 64, p, 20, 1, p, 32, p, None)


def test_the_product_library_has_no_stage_trace(lib: ctypes.CDLL) -> None:
    out = (ctypes.c_uint64 * (16 * 256))()
    assert lib.jb_stage_trace_read(out) == -1
    assert b"built without the stage trace" in lib.jb_last_error()


def test_stage_trace_statistics_of_a_regular_schedule() -> None:
    """A stamp table of a made-up schedule (K block every 1000 cycles, MMAs issued in 600, data 300 cycles after the
    TMA, dequantisation 500, warps 10 apart) gives back those intervals."""
    import numpy as np

    from jeff_b200.stage_trace import steady_state_stats

    kg = np.arange(256, dtype=np.int64)
    t = np.zeros((16, 256), dtype=np.int64)
    t[4] = 10_000 + 1000 * kg                 # MMA waits return
    t[5] = t[4] + 600                          # MMAs and commit issued
    t[0] = t[5] - 4 * 1000 + 250               # stage freed 250 cycles after the commit of the block 4 earlier
    t[1] = t[0] + 500                          # TMA issued
    t[2] = t[1] + 300                          # full seen
    t[3] = t[2] + 500                          # first warp dequantised
    for w in range(4):
        t[12 + w] = t[2] + 5 * w
        t[8 + w] = t[3] + 10 * w
    t[6, :16] = 50_000 + 20_000 * np.arange(16)
    t[7, :16] = t[6, :16] + 6000
    stats = steady_state_stats(t.astype(np.uint64))
    assert stats["k_block"][0] == 1000 and stats["mma_issue"][0] == 600
    assert stats["mma_wait_between_blocks"][0] == 400 and stats["tma_issue_to_full_seen"][0] == 300
    assert stats["commit_to_stage_free"][0] == 250 and stats["dequant_arrive_skew"][0] == 30
    assert stats["epilogue_per_tile"][0] == 6000
