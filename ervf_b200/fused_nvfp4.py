"""``FusedNVFP4`` -- the reference's kernel-wrapper class on the B200 C ABI.

Drop-in for ``lightningstream_nemotron.fused_nvfp4.FusedNVFP4``
(kennydd001/ervf src/moe_lab/lightningstream_nemotron/fused_nvfp4.py:748-984):
same method names, argument order and meaning, same in-place outputs and
``None`` returns, same attribute flags.  Buffers are caller-owned CUDA
tensors (torch tensors, or any object exposing ``__cuda_array_interface__``
such as CuPy arrays); raw device / mapped-host addresses are Python ints, as
in the reference.  Launches go on ``self.stream`` if set, else on CuPy's
current stream when CuPy is in use (as in the reference runtime), else on
torch's current stream.

Differences a caller can observe:
  * ``ervf_width`` selects a schedule: 0 (default) is the TMA-staged B200
    schedule, 4/8/16/32 the reference's subwarp widths.  All return the same
    bits (the reference proved its widths bit-identical; so are these).
  * Shapes the reference silently assumed (cols % 16 == 0, aligned rows) are
    checked and raise ``ValueError``.
  * ``down_masked_into`` reads the panel-major record where it lies (device
    or mapped host memory); ``gather_from_host`` and ``gatherless_down`` are
    accepted and change nothing in the result (the reference's gather only
    moved the same bytes into a mirror first).
"""

from __future__ import annotations

import sys

import numpy as np
import torch

from . import _lib
from .formats import e2m1_table, e4m3_device_table


def ptr(a) -> int:
    """Device address of a tensor / CUDA array, or an int passed through."""
    if a is None:
        return 0
    if isinstance(a, int):
        return a
    if isinstance(a, torch.Tensor):
        return a.data_ptr()
    cai = getattr(a, "__cuda_array_interface__", None)
    if cai is not None:
        return int(cai["data"][0])
    raise TypeError(f"expected a CUDA tensor, CUDA array or int address, got {type(a)!r}")


def current_stream(explicit, device) -> int:
    """Stream handle for a launch: an explicit stream (torch / CuPy stream
    object or raw handle), else CuPy's current stream when the caller runs
    on CuPy (as the reference runtime does), else torch's current stream."""
    if explicit is not None:
        if hasattr(explicit, "cuda_stream"):
            return int(explicit.cuda_stream)
        if hasattr(explicit, "ptr"):
            return int(explicit.ptr)
        return int(explicit)
    cp = sys.modules.get("cupy")
    if cp is not None:
        return int(cp.cuda.get_current_stream().ptr)
    return int(torch.cuda.current_stream(device).cuda_stream)


def _numel(a) -> int | None:
    if isinstance(a, torch.Tensor):
        return a.numel()
    cai = getattr(a, "__cuda_array_interface__", None)
    if cai is not None:
        return int(np.prod(cai["shape"]))
    return None


def _need(a, n: int, what: str) -> None:
    k = _numel(a)
    if k is not None and k < n:
        raise ValueError(f"{what} holds {k} elements, needs {n}")


class FusedNVFP4:
    """NVFP4 expert GEMV, fused expert, route-order accumulate, masked down,
    device router, device LRU and expert fetch on B200."""

    def __init__(self, block: int = 256, device=None):
        _lib.load()
        self.block = block
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None \
            else torch.device(device)
        self.e2m1 = torch.tensor(e2m1_table(), dtype=torch.float32, device=self.device)
        self.e4m3 = torch.tensor(e4m3_device_table(), dtype=torch.float32, device=self.device)
        self.use_ervf = True
        self.ervf_width = 0
        self.gatherless_down = False
        self.nchunks = 8
        self.stream = None

    # ------------------------------------------------------------ plumbing
    def _s(self) -> int:
        return current_stream(self.stream, self.device)

    def _width(self) -> int:
        w = int(self.ervf_width)
        if w not in (0, 4, 8, 16, 32):
            raise ValueError(f"ervf_width must be 0, 4, 8, 16 or 32, got {w}")
        return w

    # ------------------------------------------------------------- GEMV
    def gemv_into(self, out, codes, scales, x, global_scale: float, rows: int, cols: int,
                  apply_relu2: bool = False, out_scale: float = 1.0) -> None:
        """out[rows] = op(W[rows, cols] @ x[cols]) without materialising W
        (fused_nvfp4.py:944-968)."""
        _need(out, rows, "out")
        _need(codes, rows * cols // 2, "codes")
        _need(scales, rows * cols // 16, "scales")
        _need(x, cols, "x")
        width = self._width() if self.use_ervf else 0
        _lib.call("ervf_nvfp4_gemv", ptr(codes), ptr(scales), ptr(x), ptr(out),
                  float(np.float32(global_scale)), int(rows), int(cols), int(bool(apply_relu2)),
                  float(np.float32(out_scale)), width, 0 if self.use_ervf else 1, self._s())

    def expert(self, up_codes, up_scales, up_gscale: float, down_codes, down_scales,
               down_gscale: float, x, act_buf, out_buf, hidden: int, intermediate: int) -> None:
        """One routed expert: up -> ReLU^2 -> down (fused_nvfp4.py:970-978)."""
        self.gemv_into(act_buf, up_codes, up_scales, x, up_gscale, rows=intermediate,
                       cols=hidden, apply_relu2=True)
        self.gemv_into(out_buf, down_codes, down_scales, act_buf, down_gscale, rows=hidden,
                       cols=intermediate, apply_relu2=False)

    def accumulate_into(self, dst, src, weight: float, n: int) -> None:
        """dst = fmaf(src, weight, dst) (fused_nvfp4.py:980-984)."""
        _need(dst, n, "dst")
        _need(src, n, "src")
        _lib.call("ervf_weighted_accumulate", ptr(dst), ptr(src), float(np.float32(weight)),
                  int(n), self._s())

    # ------------------------------------------------------ masked down
    def alloc_masked_state(self, hidden: int, intermediate: int):
        """Device scratch for the masked down path (fused_nvfp4.py:884-900)."""
        npanel = intermediate // 16
        z = lambda n, dt: torch.zeros(n, dtype=dt, device=self.device)  # noqa: E731
        return {
            "masks": z(npanel, torch.int32),
            "plist": z(npanel, torch.int32),
            "pcount": z(1, torch.int32),
            "nz": z(intermediate, torch.int32),
            "nzc": z(1, torch.int32),
            "partials": z(self.nchunks * hidden, torch.float32),
            "mirror": z(npanel * (hidden + 16 * (hidden // 2)), torch.uint8),
        }

    def down_masked_into(self, out, bank_ptr: int, act, state, global_scale: float,
                         hidden: int, intermediate: int, nchunks: int | None = None,
                         gather_from_host: bool = True) -> None:
        """out[hidden] = masked down GEMV over one panel-major record, in the
        reference's chunk / panel / column order (fused_nvfp4.py:902-942)."""
        nc = nchunks or self.nchunks
        _lib.call("ervf_down_masked", ptr(out), ptr(bank_ptr), ptr(act), ptr(state["masks"]),
                  ptr(state["plist"]), ptr(state["pcount"]), ptr(state["nz"]), ptr(state["nzc"]),
                  float(np.float32(global_scale)), int(hidden), int(intermediate), int(nc),
                  self._s())

    # -------------------------------------------- device routing + cache
    def route_topk(self, rlog, gate_b, ids, w, n, top_k, scaling, bad_pick: int = 0) -> None:
        _lib.call("ervf_route_topk", ptr(rlog), ptr(gate_b), ptr(ids), ptr(w), int(n),
                  int(top_k), float(np.float32(scaling)), int(bad_pick), self._s())

    def route_gemv_topk(self, rlog, gate_w, x, gate_b, ids, w, n: int, hidden: int, top_k: int,
                        scaling: float, bad_pick: int = 0, counter=None, flags: int = 0) -> None:
        """The reference's ``mv_f32(rlog, gate_w, x)`` + ``route_topk`` pair
        (runtime.py:710-713) in one launch, same rlog / ids / w bit for bit.
        ``counter``: a zero int32 device word (one owned by this object by
        default; every call leaves it zero)."""
        if counter is None:
            if getattr(self, "_rcounter", None) is None:
                self._rcounter = torch.zeros(1, dtype=torch.int32, device=self.device)
            counter = self._rcounter
        _lib.call("ervf_route_gemv_topk", ptr(gate_w), ptr(x), ptr(rlog), ptr(gate_b), ptr(ids),
                  ptr(w), int(n), int(hidden), int(top_k), float(np.float32(scaling)),
                  int(bad_pick), ptr(counter), int(flags), self._s())

    def cache_assign(self, dev, ids, cap: int, top_k: int) -> None:
        _lib.call("ervf_cache_assign", ptr(dev["slot_of"]), ptr(dev["expert_of"]),
                  ptr(dev["last_used"]), ptr(dev["state2"]), ptr(ids), ptr(dev["slots"]),
                  ptr(dev["need"]), ptr(dev["stats2"]), int(cap), int(top_k), self._s())

    def cache_fetch(self, bank_c_ptr: int, bank_s_ptr: int, cache_c, cache_s, dev,
                    code_bytes: int, scale_bytes: int, top_k: int) -> None:
        _lib.call("ervf_cache_fetch", ptr(bank_c_ptr), ptr(bank_s_ptr), ptr(cache_c),
                  ptr(cache_s), ptr(dev["ids"]), ptr(dev["slots"]), ptr(dev["need"]),
                  int(code_bytes), int(scale_bytes), int(top_k), self._s())

    def gemv_ervf_indirect(self, out, cache_c, cache_s, dev, s: int, globals_dev, gsel: int, x,
                           rows: int, cols: int, apply_relu2: bool, code_stride: int,
                           scale_stride: int) -> None:
        slots = ptr(dev["slots"]) + 4 * int(s)
        ids = ptr(dev["ids"]) + 4 * int(s)
        _lib.call("ervf_nvfp4_gemv_ind", ptr(cache_c), ptr(cache_s), slots, ids,
                  ptr(globals_dev), int(gsel), ptr(x), ptr(out), int(rows), int(cols),
                  int(bool(apply_relu2)), 1.0, int(code_stride), int(scale_stride),
                  self._width(), self._s())

    def down_masked_into_indirect(self, out, down_base_ptr: int, dev, s: int, globals_dev, act,
                                  state, hidden: int, intermediate: int,
                                  panel_bytes: int) -> None:
        ids = ptr(dev["ids"]) + 4 * int(s)
        _lib.call("ervf_down_masked_ind", ptr(out), ptr(down_base_ptr), ids, int(panel_bytes),
                  ptr(globals_dev), ptr(act), ptr(state["masks"]), ptr(state["plist"]),
                  ptr(state["pcount"]), ptr(state["nz"]), ptr(state["nzc"]), int(hidden),
                  int(intermediate), int(self.nchunks), self._s())

    def accumulate_indirect(self, dst, src, w_ptr_elem, n: int) -> None:
        _lib.call("ervf_weighted_accumulate_ind", ptr(dst), ptr(src), ptr(w_ptr_elem), int(n),
                  self._s())

    def alloc_device_cache(self, n_experts: int, cap: int, top_k: int, globals_host):
        """Per-layer device state of the graph-safe MoE path
        (fused_nvfp4.py:867-882)."""
        d = self.device
        return {
            "ids": torch.zeros(top_k, dtype=torch.int32, device=d),
            "w": torch.zeros(top_k, dtype=torch.float32, device=d),
            "slots": torch.zeros(top_k, dtype=torch.int32, device=d),
            "need": torch.zeros(top_k, dtype=torch.int32, device=d),
            "slot_of": torch.full((n_experts,), -1, dtype=torch.int32, device=d),
            "expert_of": torch.full((cap,), -1, dtype=torch.int32, device=d),
            "last_used": torch.full((cap,), -1, dtype=torch.int32, device=d),
            "state2": torch.zeros(2, dtype=torch.int32, device=d),
            "stats2": torch.zeros(2, dtype=torch.int32, device=d),
            "globals": torch.as_tensor(np.asarray(globals_host, dtype=np.float32),
                                       device=d).contiguous(),
        }

    # -------------------------------------------------- grouped (B200)
    def moe_up_grouped(self, up_codes, up_scales, up_code_stride: int, up_scale_stride: int,
                       ids, globals_dev, top_k: int, x, act, inter: int, hidden: int,
                       flags: int = 0) -> None:
        """All routed up projections of a token in one launch (relu^2).
        ``flags``: ervf_b200._lib.LAUNCH_PDL | LAUNCH_IDS_READY (see the header)."""
        _lib.call("ervf_moe_up_grouped", ptr(up_codes), ptr(up_scales), int(up_code_stride),
                  int(up_scale_stride), ptr(ids), ptr(globals_dev), int(top_k), ptr(x), ptr(act),
                  int(inter), int(hidden), self._width(), int(flags), self._s())

    def moe_down_routesum(self, dn_codes, dn_scales, dn_code_stride: int, dn_scale_stride: int,
                          ids, globals_dev, route_w, top_k: int, act, out, hidden: int,
                          inter: int, base=None, resid=None, flags: int = 0, scratch=None) -> None:
        """All routed down projections plus the route-order weighted sum.
        ``scratch``: a zero-initialised uint8 device buffer of
        ``routesum_scratch_bytes(hidden, top_k)`` bytes; by default one owned
        by this object is used (so calls through one FusedNVFP4 on different
        streams must not overlap)."""
        if scratch is None:
            scratch = self._scratch(hidden, top_k)
        _lib.call("ervf_moe_down_routesum", ptr(dn_codes), ptr(dn_scales), int(dn_code_stride),
                  int(dn_scale_stride), ptr(ids), ptr(globals_dev), ptr(route_w), int(top_k),
                  ptr(act), ptr(base), ptr(resid), ptr(out), int(hidden), int(inter),
                  ptr(scratch), int(_numel(scratch) or 0), self._width(), int(flags), self._s())

    def device_status(self) -> int:
        """Read and clear the library's device error words (waits for the
        device: ervf_device_status).  After a bounded device wait ran out
        (``_lib.ERR_TIMEOUT``) the counters in this object's cached scratch
        buffers can be left non-zero, so they are zeroed again here and the
        next call starts clean.  Returns the status (0 = no error)."""
        st = int(_lib.load().ervf_device_status())
        if st == _lib.ERR_TIMEOUT:
            for buf in self.__dict__.get("_scratch_cache", {}).values():
                buf.zero_()
            if getattr(self, "_bscratch", None) is not None:
                self._bscratch.zero_()
        return st

    def routesum_scratch_bytes(self, hidden: int, top_k: int) -> int:
        return int(_lib.load().ervf_routesum_scratch_bytes(int(hidden), int(top_k)))

    def _scratch(self, hidden: int, top_k: int):
        key = (int(hidden), int(top_k))
        cache = self.__dict__.setdefault("_scratch_cache", {})
        if key not in cache:
            cache[key] = torch.zeros(self.routesum_scratch_bytes(*key), dtype=torch.uint8,
                                     device=self.device)
        return cache[key]

    def moe_batched(self, up_codes, up_scales, up_code_stride: int, up_scale_stride: int,
                    dn_codes, dn_scales, dn_code_stride: int, dn_scale_stride: int, globals_,
                    ids, w, tokens: int, top_k: int, n_experts: int, x, out, hidden: int,
                    inter: int, scratch=None, ksplit: int = 1, swiglu: bool = False) -> None:
        """Expert-major batched routed-MoE block of `tokens` decode tokens on
        the tensor cores: out[t] = x[t] + sum over route slots (in order) of
        w[t,s] * down(relu(up(x[t]))^2) with each expert read once.
        ``ksplit`` 2 splits the columns of every tensor-core unit over two CTAs
        (deterministic; more parallelism for small batches or expert shards).
        ``swiglu``: up records of 2*inter rows (gate / up interleaved),
        act = silu(gate) * up (the Qwen3-shaped block)."""
        nbytes = _lib.load().ervf_moe_batched_scratch_bytes(int(tokens), int(top_k), int(hidden),
                                                            int(inter))
        if scratch is None:
            if getattr(self, "_bscratch", None) is None or self._bscratch.numel() < nbytes:
                self._bscratch = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
            scratch = self._bscratch
        _lib.call("ervf_moe_batched_ex", ptr(up_codes), ptr(up_scales), int(up_code_stride),
                  int(up_scale_stride), ptr(dn_codes), ptr(dn_scales), int(dn_code_stride),
                  int(dn_scale_stride), ptr(globals_), ptr(ids), ptr(w), int(tokens), int(top_k),
                  int(n_experts), ptr(x), ptr(out), int(hidden), int(inter), int(ksplit),
                  _lib.UP_SWIGLU if swiglu else 0, ptr(scratch), int(nbytes), self._s())

    def gemm_tc(self, out, codes, scales, x, global_scale: float, rows: int, cols: int,
                n: int) -> None:
        """Batched NVFP4 GEMM on the tensor cores for n <= 16 activation rows:
        out[j*rows + r] = g * (W @ x[j])[r] (tolerance path, fp32 accumulate,
        deterministic).  Uses a scratch buffer owned by this object per shape
        (calls through one FusedNVFP4 on different streams must not overlap)."""
        key = ("tc", int(rows), int(cols), int(n))
        cache = self.__dict__.setdefault("_scratch_cache", {})
        if key not in cache:
            nb = int(_lib.load().ervf_nvfp4_gemm_tc_scratch_bytes(int(rows), int(cols), int(n)))
            cache[key] = torch.zeros(nb, dtype=torch.uint8, device=self.device)
        scr = cache[key]
        _lib.call("ervf_nvfp4_gemm_tc", ptr(codes), ptr(scales), float(np.float32(global_scale)),
                  ptr(x), ptr(out), int(rows), int(cols), int(n), ptr(scr), scr.numel(), self._s())

    def route_topk_softmax(self, rlogs, ids, w, layers: int, n: int, top_k: int) -> None:
        """Softmax top-k routing (Qwen-shaped experts) of `layers` logit rows:
        ids[l][s], w[l][s] = renormalised softmax of the selected experts."""
        _lib.call("ervf_route_topk_softmax", ptr(rlogs), ptr(ids), ptr(w), int(layers), int(n),
                  int(top_k), self._s())

    def route_topk_batched(self, rlogs, gate_b, ids, w, layers: int, n: int, top_k: int,
                           scaling: float, bad_pick: int = 0, bias_stride: int = 0) -> None:
        """route_topk for `layers` independent logit rows in one launch."""
        _lib.call("ervf_route_topk_batched", ptr(rlogs), ptr(gate_b), ptr(ids), ptr(w),
                  int(layers), int(n), int(top_k), float(np.float32(scaling)), int(bad_pick),
                  int(bias_stride), self._s())
