"""snai_b200: B200 (sm_100a) decode engine behind SnAI's libcortex C ABI.

The product is libcortex.so (built from snai_b200/csrc, declared in
include/cortex.h).  This package only binds it: see engine.py.
"""
from ._lib import (CortexError, PREC_BF16, PREC_FP32, PREC_TF32, LIB_PATH, SampleParams, last_error, load)
from .engine import (Cortex, CortexGroup, SnaiCortexBridge, VARIANT_A, VARIANT_B, average_states, merge_files,
                     run_inference, sample_device, sample_params, upscale_file)

__all__ = ["CortexError", "PREC_BF16", "PREC_FP32", "PREC_TF32", "LIB_PATH", "SampleParams", "last_error", "load",
           "Cortex", "CortexGroup", "SnaiCortexBridge", "VARIANT_A", "VARIANT_B", "average_states", "merge_files",
           "run_inference", "sample_device", "sample_params", "upscale_file"]
