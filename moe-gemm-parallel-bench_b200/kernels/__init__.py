"""B200-native MoE expert GEMM kernels behind the reference's kernels/ API.

Exports the names of the reference's kernels/__init__.py:1-41 that belong to
the hot path (grouped GEMM and masked single GEMM).  The torch grouped_mm
comparison provider of the reference is not part of this package.
"""

from .grouped_gemm import (
    GroupedWorkspace,
    build_fused_gate_up_workspace,
    build_fused_swiglu_workspace,
    build_grouped_workspace,
    last_aggregate_launch_info,
    launch_grouped_mm,
    launch_grouped_mm_scatter,
    check_device_errors,
    grouped_candidate_configs,
    launch_grouped,
    workspace_from_tensors,
)
from .fp8 import (
    Fp8GroupedWorkspace,
    build_fp8_workspace,
    fp8_workspace_from_tensors,
    launch_grouped_fp8,
    quantize_activations,
    quantize_weight,
)
from .matmul import (
    KernelConfig,
    last_matmul_config,
    launch_matmul,
    matmul_candidate_configs,
    native_candidates,
    select_config,
)

__all__ = [
    "Fp8GroupedWorkspace",
    "GroupedWorkspace",
    "build_fp8_workspace",
    "fp8_workspace_from_tensors",
    "launch_grouped_fp8",
    "quantize_activations",
    "quantize_weight",
    "KernelConfig",
    "build_fused_gate_up_workspace",
    "build_fused_swiglu_workspace",
    "last_aggregate_launch_info",
    "launch_grouped_mm",
    "launch_grouped_mm_scatter",
    "build_grouped_workspace",
    "check_device_errors",
    "grouped_candidate_configs",
    "last_matmul_config",
    "launch_grouped",
    "launch_matmul",
    "matmul_candidate_configs",
    "native_candidates",
    "select_config",
    "workspace_from_tensors",
]
