"""``GPUKernels.mv_bf16`` / ``mv_f32`` -- the BF16 dense GEMV and the FP32
router GEMV of the reference's kernel wrapper (kennydd001/ervf
src/moe_lab/lightningstream_nemotron/gpu_kernels.py:1549-1555) on the B200 C
ABI, plus a batched BF16 form.

Only the GEMVs that lie on the expert-decode path are provided; the
reference's attention / Mamba / norm kernels are out of scope.
"""

from __future__ import annotations

import torch

from . import _lib
from .fused_nvfp4 import _need, ptr


class GPUKernels:
    def __init__(self, block: int = 256, device=None):
        _lib.load()
        self.block = block
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None \
            else torch.device(device)
        self.stream = None

    def _s(self) -> int:
        if self.stream is not None:
            return int(self.stream.cuda_stream)
        return int(torch.cuda.current_stream(self.device).cuda_stream)

    def mv_bf16(self, out, W, x, rows: int, cols: int) -> None:
        """out[rows] = bf16 W[rows, cols] @ x[cols] (fp32), bit-exact to the
        reference's gemv_bf16."""
        self.mv_bf16_batched(out, W, x, rows, cols, 1)

    def mm_bf16_tc(self, out, W, x, rows: int, cols: int, batch: int) -> None:
        """out[b*rows + r] for x[b*cols + k], b < batch <= 8, on the tensor
        cores (tolerance path: rel-L2 <= 1e-3, not gemv_bf16's chain order)."""
        _need(out, batch * rows, "out")
        _need(W, rows * cols, "W")
        _need(x, batch * cols, "x")
        _lib.call("ervf_bf16_gemm_tc", ptr(W), ptr(x), ptr(out), int(rows), int(cols), int(batch),
                  self._s())

    def mv_bf16_batched(self, out, W, x, rows: int, cols: int, batch: int) -> None:
        """out[b*rows + r] for x[b*cols + k], b < batch <= 8."""
        _need(out, batch * rows, "out")
        _need(W, rows * cols, "W")
        _need(x, batch * cols, "x")
        _lib.call("ervf_bf16_gemv", ptr(W), ptr(x), ptr(out), int(rows), int(cols), int(batch),
                  self._s())

    def mv_f32(self, out, W, x, rows: int, cols: int) -> None:
        """out[rows] = fp32 W[rows, cols] @ x[cols], bit-exact to the
        reference's gemv_f32 (the router projection, gpu_kernels.py:51-74)."""
        _need(out, rows, "out")
        _need(W, rows * cols, "W")
        _need(x, cols, "x")
        _lib.call("ervf_f32_gemv", ptr(W), ptr(x), ptr(out), int(rows), int(cols), self._s())
