"""The product kernel's stage trace on the cfg4 GDN in_proj shape (M 8192, K 1024, N 8224, g128z, no LoRA).

    python -m jeff_b200.build --trace && python -m jeff_b200.stage_trace

Loads libjeffb200_trace.so (the product library with -DJB_TRACE) instead of the product library, runs the product
five times, reads CTA 0's clock64() stamps of its last launch (jb_stage_trace_read) and prints one JSON line of
medians, 10th and 90th percentiles in SM cycles over its steady-state K blocks (tiles 2 to 7 of CTA 0): the time per
K block, how long the MMA thread takes to issue a block's MMAs and how long it waits between blocks, the TMA latency
as the dequantisers see it, the dequantisation, the gaps between the dequantisers' arrival and the MMA thread's
wait returning, the commit-to-free latency of a stage, the skew between the warps of a dequantiser group, and the
epilogue's time per tile."""

from __future__ import annotations

import ctypes
import json

import numpy as np
import torch

from jeff_b200 import _lib, build


def steady_state_stats(t: np.ndarray, per_tile: int = 16) -> dict[str, list[float]]:
    """Statistics of a (16, 256) stamp table (0 = not stamped) over K blocks of tiles 2 .. 7."""
    t = t.astype(np.int64)
    ks = np.arange(per_tile * 2, per_tile * 8)

    def d(a: np.ndarray, b: np.ndarray) -> list[float]:
        v = np.asarray(a, dtype=np.float64) - np.asarray(b, dtype=np.float64)
        return [float(np.median(v)), float(np.percentile(v, 10)), float(np.percentile(v, 90))]

    last_arrive = t[8:12, ks].max(0)
    return {
        "k_block": d(t[5][ks], t[5][ks - 1]),
        "mma_issue": d(t[5][ks], t[4][ks]),
        "mma_wait_between_blocks": d(t[4][ks], t[5][ks - 1]),
        "tma_issue_to_full_seen": d(t[2][ks], t[1][ks]),
        "dequant_first_warp": d(t[3][ks], t[2][ks]),
        "last_dequant_arrive_to_mma_ready": d(t[4][ks], last_arrive),
        "commit_to_stage_free": d(t[0][ks + 4], t[5][ks]),
        "producer_free_to_issued": d(t[1][ks], t[0][ks]),
        "stage_free_to_mma_ready": d(t[4][ks + 4], t[0][ks + 4]),
        "dequant_arrive_skew": d(last_arrive, t[8:12, ks].min(0)),
        "epilogue_per_tile": d(t[7][2:8], t[6][2:8]),
    }


def main() -> None:
    if not torch.cuda.is_available():
        raise SystemExit("stage_trace needs a CUDA GPU")
    if not build.TRACE_LIB.exists():
        raise SystemExit(f"{build.TRACE_LIB} is missing: python -m jeff_b200.build --trace")
    _lib.LIB_PATH = build.TRACE_LIB
    lib = _lib.load()
    from jeff_b200 import int4, kernels, synthetic

    m, k, n = 8192, 1024, 8224
    packed, _ = int4.quantize_pack(synthetic.normal(4, "trace/w", (n, k), 0.02), "g128z")
    words = kernels.int4_repack(packed.words.cuda())
    scales, zeros = packed.scales.cuda(), packed.zeros.cuda()
    x = synthetic.normal(4, "trace/x", (m, k), 1.0).to(torch.bfloat16).cuda()
    y = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    for _ in range(5):
        kernels.int4_product(x, words, scales, zeros, 128, n, None, None, None, 128, y=y)
    torch.cuda.synchronize()
    stamps = np.zeros((16, 256), dtype=np.uint64)
    if lib.jb_stage_trace_read(ctypes.c_void_p(stamps.ctypes.data)) != 0:
        raise SystemExit(lib.jb_last_error().decode())
    print(json.dumps({"shape": "M8192 K1024 N8224 g128z, no LoRA", "unit": "SM cycles [median, p10, p90]",
                      **steady_state_stats(stamps)}), flush=True)


if __name__ == "__main__":
    main()
