"""``SweepMoE`` -- the reference's expert-major block API on the B200 C ABI.

Drop-in for ``lightningstream_nemotron.sweepspec.SweepMoE``
(kennydd001/ervf src/moe_lab/lightningstream_nemotron/sweepspec.py:244-375):
same constructor, ``plan`` / ``compile_plan`` / ``alloc_state`` /
``gemm_into`` / ``down_union`` / ``moe_block`` with the same argument order,
in-place outputs and ``None`` returns.  Buffers are torch tensors (or CuPy
arrays through ``__cuda_array_interface__``); raw addresses are ints.

Numerics, per node (activation row):
  * ``gemm_into`` returns what the reference's ``gemm_nvfp4_rows_b`` returns,
    bit for bit: each column is ``gemv_nvfp4_rows`` (the legacy 256-chain
    tree) on that node's row, which is what the reference's batched kernel
    computes per column (ervf_nvfp4_gemm_rows_b).
  * ``down_union`` returns the reference's ``down_union`` bit for bit: the
    masked panel-major down projection of every node over the UNION panel
    list and masks of the expert's nodes (ervf_down_union), scattered to
    ``contrib[dst[b]]``.  The union matters: the masked path assigns panels
    to its chunks by their position in the active list, so a node's bits
    depend on the other nodes' zero pattern.
  * ``moe_block`` ends with ``reduce_slots``: out[b] = fmaf(w, contrib, out)
    over the route slots in order (the token-major path's order).

This surface keeps the reference's semantics; the B200 throughput path for a
decode batch is ``MoEDecoder.step_batch`` / ``FusedNVFP4.moe_batched`` (one
tensor-core launch per projection for all experts, held to rel-L2 1e-3).
"""

from __future__ import annotations

import numpy as np
import torch

from . import _lib
from .fused_nvfp4 import FusedNVFP4, _numel, ptr

MAX_B = 16


class SweepMoE:
    """Expert-major block execution of the routed experts."""

    def __init__(self, fused: FusedNVFP4, kernels=None, block: int = 256):
        self.fused = fused
        self.k = kernels
        self.block = block
        self.max_shared = 0  # no shared-memory limit on the batch here (the reference's cap)

    # ------------------------------------------------------------- planning
    @staticmethod
    def plan(routes, top_k: int):
        """Group (node, slot) pairs by expert, experts in first-seen order."""
        groups: dict[int, list[tuple[int, int]]] = {}
        for b, r in enumerate(routes):
            for s in range(top_k):
                groups.setdefault(int(r[s]), []).append((b, s))
        return groups

    def compile_plan(self, groups, top_k: int):
        """Device-side index arrays for one layer's plan, built once:
        (expert, nodes int32[n], dst int32[n] = node*top_k + slot, n)."""
        d = self.fused.device
        out = []
        for e, pairs in groups.items():
            nodes = torch.tensor([b for b, _ in pairs], dtype=torch.int32, device=d)
            dst = torch.tensor([b * top_k + s for b, s in pairs], dtype=torch.int32, device=d)
            out.append((int(e), nodes, dst, len(pairs)))
        return out

    def alloc_state(self, hidden: int, inter: int, top_k: int, B: int):
        d = self.fused.device
        z = lambda n, dt=torch.float32: torch.zeros(n, dtype=dt, device=d)  # noqa: E731
        npanel = inter // 16
        nb = max(B, MAX_B)
        state = self.fused.alloc_masked_state(hidden, inter)
        state.update({
            "acts": z(nb * inter),
            "act_sum": z(inter),
            "contrib": z(B * top_k * hidden),
            "weights": z(B * top_k),
            "xbuf": z(nb * max(hidden, inter)),
            "tmp": z(nb * hidden),
            "nchunks": self.fused.nchunks, "npanel": npanel, "top_k": top_k, "B": B,
        })
        return state

    # -------------------------------------------------------------- kernels
    def gemm_into(self, out, codes, scales, x, nodes, global_scale: float, rows: int, cols: int,
                  n: int, apply_relu2: bool = False, xbuf=None) -> None:
        """out[b*rows + r] = op(W x[nodes[b]])[r], b < n (gemm_nvfp4_rows_b,
        sweepspec.py:317-329)."""
        if n < 1 or n > MAX_B:
            raise ValueError(f"n must be in [1, {MAX_B}], got {n}")
        if xbuf is None:
            xbuf = self._xbuf(n * cols)
        elif (_numel(xbuf) or 0) < n * cols:
            raise ValueError("xbuf holds fewer than n * cols floats")
        _lib.call("ervf_nvfp4_gemm_rows_b", ptr(codes), ptr(scales), ptr(x), ptr(nodes), ptr(out),
                  float(np.float32(global_scale)), int(rows), int(cols), int(n),
                  int(bool(apply_relu2)), ptr(xbuf), self.fused._s())

    def down_union(self, dst, bank_ptr: int, state, global_scale: float, hidden: int, inter: int,
                   n: int, gather_from_host: bool = True) -> None:
        """contrib[dst[b]] = masked down of state["acts"][b] over the
        panel-major record at bank_ptr, b < n (sweepspec.py:331-360).  The
        record is read where it lies (device or mapped host memory), so
        ``gather_from_host`` changes nothing in the result."""
        _lib.call("ervf_down_union", ptr(bank_ptr), ptr(state["acts"]), int(n), ptr(dst),
                  ptr(state["contrib"]), float(np.float32(global_scale)), int(hidden), int(inter),
                  int(state["nchunks"]), ptr(state["act_sum"]), ptr(state["masks"]), ptr(state["plist"]),
                  ptr(state["pcount"]), ptr(state["nz"]), ptr(state["nzc"]), ptr(state["tmp"]),
                  self.fused._s())

    def reduce_slots(self, state, out, hidden: int, top_k: int, B: int) -> None:
        """out[b] = fmaf(w[b,s], contrib[b,s], out[b]) over s in route order."""
        _lib.call("ervf_reduce_slots", ptr(state["contrib"]), ptr(state["weights"]), ptr(out),
                  int(hidden), int(top_k), int(B), self.fused._s())

    def moe_block(self, out, rt, layer: int, x_all, compiled_plan, state, B: int) -> None:
        """Expert-major MoE for B nodes of one layer (sweepspec.py:362-375).
        ``rt`` carries the reference runtime's layer state: ``hidden``,
        ``moe_inter``, ``top_k``, ``bank[layer]`` ("globals" [E][2] host,
        "down_base_ptr") and ``cache[layer]`` ("map", "codes", "scales")."""
        hidden, inter, top_k = rt.hidden, rt.moe_inter, rt.top_k
        up_code, up_scale = inter * hidden // 2, inter * hidden // 16
        down_panel_bytes = hidden * inter // 2 + hidden * inter // 16
        bank, cache = rt.bank[layer], rt.cache[layer]
        for e, nodes, dst, n in compiled_plan:
            slot = int(cache["map"][e])
            self.gemm_into(state["acts"], cache["codes"][slot * up_code:(slot + 1) * up_code],
                           cache["scales"][slot * up_scale:(slot + 1) * up_scale], x_all, nodes,
                           float(bank["globals"][e, 1]), inter, hidden, n, apply_relu2=True,
                           xbuf=state["xbuf"])
            self.down_union(dst, int(bank["down_base_ptr"]) + e * down_panel_bytes, state,
                            float(bank["globals"][e, 0]), hidden, inter, n)
        self.reduce_slots(state, out, hidden, top_k, B)

    def _xbuf(self, n: int):
        buf = getattr(self, "_xb", None)
        if buf is None or buf.numel() < n:
            self._xb = buf = torch.empty(n, dtype=torch.float32, device=self.fused.device)
        return buf
