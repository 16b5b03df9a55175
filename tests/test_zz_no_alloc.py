"""The allocation-free GroupNorm entry point (GPU).

``ldb_group_norm_affine_noalloc`` serves callers that cannot allocate device
memory when they call (an engine that reserves all of its device memory up
front, or a binding with no device allocator), so they cannot hand the
library a workspace.  It keeps its partial sums in a fixed device array
inside the library.  This test calls it through the C ABI twice in a row, on
different inputs, and checks each result against the workspace-based
``ldb_group_norm_affine`` at the tolerance the other GroupNorm tests use.
The file is named to be collected last.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _noalloc_affine(x1: torch.Tensor, x2: torch.Tensor | None, gamma: torch.Tensor, beta: torch.Tensor,
                    groups: int, eps: float) -> torch.Tensor:
    from lesiondiffusion_mlx_b200 import _lib

    b = int(x1.shape[0])
    voxels = int(np.prod(x1.shape[1:-1]))
    c1, ld1 = int(x1.shape[-1]), int(x1.stride(-2))
    c2, ld2 = (0, 0) if x2 is None else (int(x2.shape[-1]), int(x2.stride(-2)))
    affine = torch.full((b, c1 + c2, 2), float("nan"), dtype=torch.float32, device=x1.device)
    _lib.call(
        "ldb_group_norm_affine_noalloc", torch.cuda.current_stream(x1.device).cuda_stream, x1.data_ptr(), c1, ld1,
        None if x2 is None else x2.data_ptr(), c2, ld2, _lib.LDB_F16 if x1.dtype == torch.float16 else _lib.LDB_F32,
        b, voxels, groups, gamma.data_ptr(), beta.data_ptr(), float(eps), affine.data_ptr(),
    )
    return affine


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_noalloc_group_norm_matches_workspace_entry_point_twice(cuda_device, dtype):
    from lesiondiffusion_mlx_b200 import ops

    # The last two cases hold batch x 1024 channels over 20480 voxels: the fixed
    # array cannot take one partial per planned chunk there, so the entry point
    # reduces the chunk count (512 and 256 chunks instead of the workspace
    # path's count) and the sums are formed over longer chunks.
    cases = [((2, 6, 10, 12, 256), None, 32), ((1, 4, 20, 20, 512), 256, 32), ((1, 16, 32, 40, 1024), None, 32),
             ((2, 16, 32, 40, 1024), 512, 32)]
    for i, (shape, split, groups) in enumerate(cases):
        rng = np.random.default_rng(40 + i)
        x = torch.from_numpy((rng.normal(size=shape) * 2 + 0.5).astype(np.float32)).to(dtype).to(cuda_device)
        gamma = torch.from_numpy(rng.normal(size=shape[-1]).astype(np.float32)).to(cuda_device)
        beta = torch.from_numpy(rng.normal(size=shape[-1]).astype(np.float32)).to(cuda_device)
        x1, x2 = (x, None) if split is None else (x[..., :split].contiguous(), x[..., split:].contiguous())
        got = _noalloc_affine(x1, x2, gamma, beta, groups, 1e-5)
        want = ops.group_norm_affine(x1, gamma, beta, groups=groups, eps=1e-5, x2=x2)
        torch.cuda.synchronize()
        assert torch.isfinite(got).all()
        np.testing.assert_allclose(got.cpu().numpy(), want.cpu().numpy(), rtol=2e-5, atol=2e-5)


def test_noalloc_group_norm_rejects_oversized_calls(cuda_device):
    from lesiondiffusion_mlx_b200 import _lib

    x = torch.zeros((1, 1, 1, 1, 8), dtype=torch.float16, device=cuda_device)
    g = torch.ones(8, device=cuda_device)
    affine = torch.empty((1 << 17, 8, 2), device=cuda_device)
    with pytest.raises(_lib.LdbError, match="exceeds the fixed scratch"):
        # batch * channels = 2^17 * 8 > 2^19 entries
        _lib.call("ldb_group_norm_affine_noalloc", torch.cuda.current_stream().cuda_stream, x.data_ptr(), 8, 8,
                  None, 0, 0, _lib.LDB_F16, 1 << 17, 1, 1, g.data_ptr(), g.data_ptr(), 1e-5, affine.data_ptr())
