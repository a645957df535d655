"""Regenerates tests/golden/bf16_checker_cases.npz: bf16 outputs of the
reference's own correctness checker on DeepSeek-V3 miniature rank groups.

The reference checks every grouped launch against per-expert torch.matmul on
the same bf16 tensors; for the packed W13 weight it multiplies the gate and up
halves separately and concatenates them (benchmark_moe.py:255-266 of the
reference):

    W1:  reference = cat(matmul(a, b[:, :F]), matmul(a, b[:, F:]), dim=1)
    W2:  reference = matmul(a, b)

This script runs exactly that computation with torch on host bf16 tensors (the
reference runs it on the GPU; torch.matmul on the host is the same operation
with fp32 accumulation and one bf16 rounding) and stores its outputs.

Inputs follow BASELINE.json's distributions: A ~ N(0, 1), B ~ N(0, 1/sqrt(K)),
drawn in bf16 from a CPU torch.Generator seeded per case (draw order: A of
every expert, then B of every expert).  Only outputs are stored, with SHA-256
digests of the inputs' bytes: the tests regenerate the inputs from the seed
and refuse to compare if a digest differs.  K is the real DeepSeek-V3 depth of
each projection; experts and N are cut down so the fixture stays small.

    python tests/golden/make_bf16_golden.py
"""

from __future__ import annotations

import hashlib
import json
import math
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
OUT = HERE / "bf16_checker_cases.npz"

# (name, projection, K, N, experts): DeepSeek-V3 P = 8 rank projections with
# their real K.  W13 N is a packed [gate | up] width.
GROUPS = (
    ("W13_EP", "W1", 7168, 512, 2),   # rank: 32 x [M, 7168] @ [7168, 4096]
    ("W13_TP", "W1", 7168, 512, 2),   # rank: 256 x [M, 7168] @ [7168, 512]
    ("W2_EP", "W2", 2048, 512, 2),    # rank: 32 x [M, 2048] @ [2048, 7168]
    ("W2_TP", "W2", 256, 512, 2),     # rank: 256 x [M, 256] @ [256, 7168]
)
M_VALUES = (16, 17, 129, 256)


def case_seed(group_index: int, m: int) -> int:
    return 1000 * (group_index + 1) + m


def make_inputs(seed: int, m: int, k: int, n: int, experts: int):
    """Seeded bf16 inputs of one case (CPU generator; see the module docstring)."""
    gen = torch.Generator().manual_seed(seed)
    a = [torch.randn((m, k), generator=gen, dtype=torch.float32).to(torch.bfloat16) for _ in range(experts)]
    b = [(torch.randn((k, n), generator=gen, dtype=torch.float32) / math.sqrt(k)).to(torch.bfloat16)
         for _ in range(experts)]
    return a, b


def digest(tensors) -> str:
    h = hashlib.sha256()
    for t in tensors:
        h.update(t.contiguous().view(torch.uint16).numpy().tobytes())
    return h.hexdigest()


def checker(a: torch.Tensor, b: torch.Tensor, projection: str) -> torch.Tensor:
    """The reference's per-expert check (benchmark_moe.py:259-266)."""
    if projection == "W1":
        local_ffn = b.shape[1] // 2
        return torch.cat((torch.matmul(a, b[:, :local_ffn]), torch.matmul(a, b[:, local_ffn:])), dim=1)
    return torch.matmul(a, b)


def main() -> None:
    torch.set_num_threads(max(1, torch.get_num_threads()))
    arrays, index = {}, []
    for g, (name, projection, k, n, experts) in enumerate(GROUPS):
        for m in M_VALUES:
            seed = case_seed(g, m)
            a, b = make_inputs(seed, m, k, n, experts)
            key = f"{name}_M{m}"
            for e in range(experts):
                c = checker(a[e], b[e], projection)
                assert c.dtype == torch.bfloat16 and c.shape == (m, n)
                arrays[f"{key}/c{e}"] = c.view(torch.uint16).numpy()
            index.append({"name": key, "group": name, "projection": projection, "m": m, "k": k, "n": n,
                          "experts": experts, "seed": seed, "a_sha256": digest(a), "b_sha256": digest(b)})
    arrays["_index"] = np.frombuffer(json.dumps(index).encode(), dtype=np.uint8)
    np.savez_compressed(OUT, **arrays)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes, {len(index)} cases)")


if __name__ == "__main__":
    main()
