"""Hardware ceilings for roofline fractions, with a B200 entry.

Same lookup interface as the upstream experiments' table (GPU_SPECS[key][...],
PRECISION_PEAK_KEY, detect_gpu_name(), ridge_point()), so sweeps written against it run
unchanged.  FLOP/s and bytes/s, not T-units.  For the B200 the tensor and HBM peaks come
from the repository's MEASURED_PEAKS.json when it exists (a cuBLAS bf16 GEMM burst and a
STREAM-style copy on this pool's GPUs; TF32 is half the bf16 rate on tcgen05), otherwise
from NVIDIA's nominal dense figures.  The other entries are nominal spec-sheet values.
"""

import json
import os

TFLOP = 1.0e12
GBs = 1.0e9


def _b200():
    spec = {"arch": "Blackwell", "sm_count": 148, "smem_per_sm_kb": 228,
            "peak_fp32_flops": 80.0 * TFLOP,        # CUDA cores, nominal
            "peak_fp16_tc_flops": 2250.0 * TFLOP,   # dense, nominal
            "peak_tf32_tc_flops": 1125.0 * TFLOP,
            "peak_fp8_tc_flops": 4500.0 * TFLOP,
            "peak_bw_bytes": 7700.0 * GBs, "source": "nominal"}
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                        "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            m = json.load(f)
        spec.update(peak_fp16_tc_flops=m["bf16_tflops"] * TFLOP,
                    peak_tf32_tc_flops=m["bf16_tflops"] / 2 * TFLOP,
                    peak_bw_bytes=m["hbm_gbs"] * GBs, source="measured")
    return spec


GPU_SPECS = {
    "B200": _b200(),
    "H200": {"arch": "Hopper", "sm_count": 132, "smem_per_sm_kb": 228,
             "peak_fp32_flops": 67.0 * TFLOP, "peak_fp16_tc_flops": 989.0 * TFLOP,
             "peak_tf32_tc_flops": 494.5 * TFLOP, "peak_fp8_tc_flops": 1979.0 * TFLOP,
             "peak_bw_bytes": 4800.0 * GBs, "source": "nominal"},
    "L40S": {"arch": "Ada", "sm_count": 142, "smem_per_sm_kb": 100,
             "peak_fp32_flops": 91.6 * TFLOP, "peak_fp16_tc_flops": 362.0 * TFLOP,
             "peak_tf32_tc_flops": 183.0 * TFLOP, "peak_fp8_tc_flops": 733.0 * TFLOP,
             "peak_bw_bytes": 864.0 * GBs, "source": "nominal"},
}

# precision -> peak key; the fp32 API of this library computes on TF32 tensor cores
PRECISION_PEAK_KEY = {"fp32": "peak_fp32_flops", "tf32": "peak_tf32_tc_flops",
                      "fp16": "peak_fp16_tc_flops", "bf16": "peak_fp16_tc_flops",
                      "fp8": "peak_fp8_tc_flops"}


def raw_gpu_name():
    try:
        import torch

        if torch.cuda.is_available():
            return torch.cuda.get_device_name(0)
    except Exception:
        pass
    return None


def detect_gpu_name():
    """GPU_SPECS key of the current device, or None."""
    name = (raw_gpu_name() or "").upper()
    for key in ("B200", "H200", "L40S"):
        if key in name:
            return key
    return None


def ridge_point(gpu_key, precision="fp32"):
    spec = GPU_SPECS[gpu_key]
    peak = spec.get(PRECISION_PEAK_KEY[precision])
    return None if peak is None else peak / spec["peak_bw_bytes"]
