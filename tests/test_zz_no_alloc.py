"""GPU test of grouped_gemm_launch_noalloc, the grouped launch for callers
that cannot allocate device memory.

Such callers -- a plugin whose host framework owns all device memory and hands
it only its input and output tensors, or a launch path that must never enter
the driver's allocator -- cannot hand the library a scratch buffer, so this
entry point takes the tensor-map scratch from a fixed array inside the
library.  This file is collected last (its name sorts last), so a run that
stops at the first failure has already run every other test; it also passes
alone in a fresh process, where its first call performs the once-per-device
set-up.

The checks, through the C ABI, on two calls in a row: the no-alloc entry
point gives the same output as the existing grouped_gemm_launch on the same
inputs and matches the float64 oracle (both within the bf16 tolerance the
parity tests use: relative Frobenius <= 1e-2), the device error word stays
clear, and the second call (after the set-up) changes neither torch's
allocated bytes nor the device's free memory.
"""

from __future__ import annotations

import numpy as np
import pytest

from tests.conftest import cuda_ready

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_ready(), reason="needs a CUDA GPU")]

REL_FRO_BF16 = 1e-2


def _inputs(shapes, seed):
    import torch

    from kernels import workspace_from_tensors

    gen = torch.Generator(device="cuda").manual_seed(seed)
    a = [torch.randn((m, k), device="cuda", generator=gen).to(torch.bfloat16) for m, k, _ in shapes]
    b = [(torch.randn((k, n), device="cuda", generator=gen) / k**0.5).to(torch.bfloat16) for _, k, n in shapes]
    c = [torch.full((m, n), float("nan"), device="cuda", dtype=torch.bfloat16) for m, _, n in shapes]
    return workspace_from_tensors(a, b, c)


def _rel_fro(got, expected) -> float:
    return float((got.double() - expected.double()).norm() / expected.double().norm())


@pytest.mark.parametrize("shapes", [[(16, 512, 256)] * 4, [(16, 256, 256), (40, 192, 128), (130, 64, 384)]],
                         ids=["homogeneous", "heterogeneous"])
def test_noalloc_entry_matches_existing_entry_on_two_calls(shapes):
    import torch

    from kernels import KernelConfig, _native, launch_grouped
    from kernels.grouped_gemm import operands_tma_aligned
    from oracle import gemm as oracle

    ws = _inputs(shapes, seed=31)
    config = KernelConfig(16, 128, 64, 4, 4, 3)
    device = torch.cuda.current_device()
    _native.read_and_clear_error_word(device)

    launch_grouped(ws, config=config, autotune=False)  # the existing entry point
    torch.cuda.synchronize()
    expected = [c.clone() for c in ws.c]
    assert ws.launch_info["path"].startswith("tcgen05_tma")
    oracle_out = [oracle.matmul(a.double().cpu().numpy(), b.double().cpu().numpy(), "bf16")
                  for a, b in zip(ws.a, ws.b)]

    if ws.homogeneous:
        m, k, n = ws.shapes[0]
    else:
        m, k, n = ws.max_m, ws.max_k, ws.max_n
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        for c in ws.c:
            c.fill_(float("nan"))
        torch.cuda.synchronize()
        allocated, (free, _) = torch.cuda.memory_allocated(), torch.cuda.mem_get_info()
        info = _native.grouped_launch_noalloc(
            ws.a_ptrs.data_ptr(), ws.b_ptrs.data_ptr(), ws.c_ptrs.data_ptr(), ws.dims.data_ptr(),
            ws.strides.data_ptr(), ws.problem_count, ws.homogeneous, m, n, k, "bf16", "ieee",
            operands_tma_aligned(ws), config, stream,
        )
        torch.cuda.synchronize()
        if call == 1:  # after the once-per-device set-up of the first call
            assert torch.cuda.memory_allocated() == allocated
            assert torch.cuda.mem_get_info()[0] == free, "the no-alloc launch changed the device's free memory"
        assert info.path == 0, "the no-alloc entry point must run the tensor-core kernel"
        assert _native.read_and_clear_error_word(device) == 0
        for e, (got, want) in enumerate(zip(ws.c, expected)):
            assert torch.isfinite(got.float()).all(), f"call {call}: unwritten outputs"
            assert _rel_fro(got, want) <= REL_FRO_BF16, f"call {call}"
            got_np = got.double().cpu().numpy()
            err = float(np.linalg.norm(got_np - oracle_out[e]) / np.linalg.norm(oracle_out[e]))
            assert err <= REL_FRO_BF16, f"call {call}, problem {e}: {err:.3e} against the oracle"
