"""GPU entry points (the drop-in for the reference's `pck.cuda`, src/pck/cuda/__init__.py)."""

from pck.cuda import ops
from pck.cuda._lib import device_status
from pck.cuda.checker import (
    DEFAULT_BLOCK,
    CheckResult,
    GpuBlockedChecker,
    PendingCheck,
    SideStreamChecker,
    check_many,
    checked_gemvs,
    gemv_checked,
    round_up_bf16,
)
from pck.cuda.gemv import gemv_coalesced, gemv_fp8, gemv_naive, gemv_tc, quantize_fp8, tc_height
from pck.cuda.sampling import (
    SamplingCheck,
    check_topk_gpu,
    check_topp_gpu,
    sharded_topk_gpu,
    topk_sample,
    topp_select,
)

__all__ = [
    "DEFAULT_BLOCK",
    "CheckResult",
    "GpuBlockedChecker",
    "PendingCheck",
    "SamplingCheck",
    "SideStreamChecker",
    "check_many",
    "check_topk_gpu",
    "check_topp_gpu",
    "checked_gemvs",
    "device_status",
    "gemv_checked",
    "gemv_coalesced",
    "gemv_fp8",
    "gemv_naive",
    "gemv_tc",
    "ops",
    "quantize_fp8",
    "round_up_bf16",
    "tc_height",
    "sharded_topk_gpu",
    "topk_sample",
    "topp_select",
]
