"""HBM-resident routed experts and the MoE decode step on the C ABI.

``ExpertBank`` is the residency / upload path: every routed expert of every
MoE layer lives in HBM for the life of the process, uploaded once, in the
layout the grouped kernels read directly (replaces the reference's pinned
host bank + LRU device cache, runtime.py:216-267, :324-381, whose slot map
becomes the identity when everything is resident).  Per layer:

    up_codes   u8[E][inter * hidden / 2]    row-major, low nibble first
    up_scales  u8[E][inter * hidden / 16]   E4M3
    dn_codes   u8[E][hidden * inter / 2]
    dn_scales  u8[E][hidden * inter / 16]
    globals    f32[E][2] = (g_down, g_up)   (runtime.py:246-247)

Every record starts on a 16-byte boundary (the per-expert byte counts of
the supported shapes are multiples of 16), so the TMA schedule streams them
with 1-D bulk copies.

``MoEDecoder`` runs routed MoE layers of one token: device router
(route_topk), one launch for the top-k up projections with relu^2, one
launch for the top-k down projections fused with the route-order weighted
sum and the residual add x + moe(x).  With expert parallelism (``ep_ranks``
> 1) each rank owns experts e with e % ep_ranks == rank and computes only
its slots' down outputs; one exchange kernel per layer then reads every
slot from its owner's memory over NVLink (or, with ``exchange="nccl"``, an
all-gather collects them) before the same route-order sum -- so every
rank's result is bit-identical to one GPU.
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib
from .formats import quantize_nvfp4_torch
from .fused_nvfp4 import FusedNVFP4, ptr


class ExpertBank:
    def __init__(self, n_layers: int, n_experts: int, hidden: int, inter: int, device=None,
                 layers=None):
        self.n_layers, self.n_experts = n_layers, n_experts
        self.hidden, self.inter = hidden, inter
        self.device = torch.device(device or "cuda")
        self.up_code_bytes = inter * hidden // 2
        self.up_scale_bytes = inter * hidden // 16
        self.dn_code_bytes = hidden * inter // 2
        self.dn_scale_bytes = hidden * inter // 16
        for b in (self.up_code_bytes, self.up_scale_bytes, self.dn_code_bytes, self.dn_scale_bytes):
            if b % 16:
                raise ValueError("per-expert record sizes must be multiples of 16 bytes")
        self.owned = list(range(n_experts)) if layers is None else layers
        E, d = n_experts, self.device
        u8 = torch.uint8
        self.up_codes = [torch.empty(E * self.up_code_bytes, dtype=u8, device=d) for _ in range(n_layers)]
        self.up_scales = [torch.empty(E * self.up_scale_bytes, dtype=u8, device=d) for _ in range(n_layers)]
        self.dn_codes = [torch.empty(E * self.dn_code_bytes, dtype=u8, device=d) for _ in range(n_layers)]
        self.dn_scales = [torch.empty(E * self.dn_scale_bytes, dtype=u8, device=d) for _ in range(n_layers)]
        self.globals = [torch.zeros(E, 2, dtype=torch.float32, device=d) for _ in range(n_layers)]

    @property
    def nbytes(self) -> int:
        per = self.up_code_bytes + self.up_scale_bytes + self.dn_code_bytes + self.dn_scale_bytes
        return self.n_layers * self.n_experts * per

    def expert_bytes(self) -> int:
        return self.up_code_bytes + self.up_scale_bytes + self.dn_code_bytes + self.dn_scale_bytes

    # -------------------------------------------------------------- upload
    def upload_expert(self, layer: int, e: int, up, dn, non_blocking: bool = False) -> None:
        """up / dn = (codes, scales, g) as numpy arrays or tensors (host or
        device, row-major as in the checkpoint)."""
        for (c, s, g), codes, scales, cb, sb, gi in (
                (up, self.up_codes, self.up_scales, self.up_code_bytes, self.up_scale_bytes, 1),
                (dn, self.dn_codes, self.dn_scales, self.dn_code_bytes, self.dn_scale_bytes, 0)):
            ct = torch.as_tensor(c).reshape(-1)
            st = torch.as_tensor(s).reshape(-1)
            if ct.numel() != cb or st.numel() != sb:
                raise ValueError("record size does not match the bank shape")
            codes[layer][e * cb:(e + 1) * cb].copy_(ct, non_blocking=non_blocking)
            scales[layer][e * sb:(e + 1) * sb].copy_(st, non_blocking=non_blocking)
            self.globals[layer][e, gi] = float(np.float32(g.item() if hasattr(g, "item") else g))

    def expert_host(self, layer: int, e: int):
        """(up, dn) records of one expert, copied back to numpy."""
        cb, sb = self.up_code_bytes, self.up_scale_bytes
        db, ds = self.dn_code_bytes, self.dn_scale_bytes
        g = self.globals[layer][e].cpu().numpy()
        up = (self.up_codes[layer][e * cb:(e + 1) * cb].cpu().numpy(),
              self.up_scales[layer][e * sb:(e + 1) * sb].cpu().numpy(), np.float32(g[1]))
        dn = (self.dn_codes[layer][e * db:(e + 1) * db].cpu().numpy(),
              self.dn_scales[layer][e * ds:(e + 1) * ds].cpu().numpy(), np.float32(g[0]))
        return up, dn

    @classmethod
    def synthetic(cls, n_layers: int, n_experts: int, hidden: int, inter: int, device=None,
                  seed: int = 0, std: float = 0.02, rank: int = 0,
                  world: int = 1) -> "ExpertBank":
        """Seeded synthetic bank built on the device: weights ~ N(0, std)
        from a torch generator seeded with seed*1e6 + 1000*layer + expert
        (+0 up, +500 down), quantised by ``quantize_nvfp4_torch``.  With
        world > 1 only the experts this rank owns (e % world == rank) are
        built; the others stay uninitialised."""
        bank = cls(n_layers, n_experts, hidden, inter, device)
        gen = torch.Generator(device=bank.device)
        for layer in range(n_layers):
            for e in range(rank, n_experts, world):
                recs = []
                for off, (r, c) in ((0, (inter, hidden)), (500, (hidden, inter))):
                    gen.manual_seed(seed * 1_000_000 + 1000 * layer + e + off)
                    w = torch.randn(r, c, generator=gen, device=bank.device) * std
                    recs.append(quantize_nvfp4_torch(w))
                bank.upload_expert(layer, e, recs[0], recs[1])
        torch.cuda.synchronize(bank.device)
        return bank


class MoEDecoder:
    """Routed MoE layers of one token on a resident ``ExpertBank``."""

    def __init__(self, bank: ExpertBank, top_k: int, scaling: float = 1.0, fused=None,
                 ep_ranks: int = 1, ep_rank: int = 0, group=None, exchange: str = "p2p",
                 exchange_timeout_ms: int = 5000):
        self.bank, self.top_k, self.scaling = bank, top_k, scaling
        self.fused = fused or FusedNVFP4(device=bank.device)
        self.ep_ranks, self.ep_rank, self.group = ep_ranks, ep_rank, group
        d, L, k = bank.device, bank.n_layers, top_k
        self.ids = torch.zeros(L, k, dtype=torch.int32, device=d)
        self.w = torch.zeros(L, k, dtype=torch.float32, device=d)
        self.act = torch.zeros(k * bank.inter, dtype=torch.float32, device=d)
        self.gate_b = torch.zeros(bank.n_experts, dtype=torch.float32, device=d)
        # x after layer l lives in xbuf[l & 1]
        self.xbuf = torch.zeros(2, bank.hidden, dtype=torch.float32, device=d)
        self.xs = [self.xbuf[0], self.xbuf[1]]
        # exchange of the slot outputs between ranks: "p2p" = peer-memory
        # exchange kernel fused with the route-order sum (one launch, no
        # collective); "nccl" = NCCL all-gather + route-sum launch
        if exchange not in ("p2p", "nccl"):
            raise ValueError(f"exchange must be 'p2p' or 'nccl', not {exchange!r}")
        self.exchange, self.exchange_timeout_ms = exchange, int(exchange_timeout_ms)
        self.xchg = None
        self._bxchg = None  # exchange regions of the batched block (sized per batch)
        # K-split of the batched block's tensor-core launches: with 8 ranks a
        # rank's expert shard (~13 experts per layer at batch 32) leaves most
        # of the GPU idle at one CTA per (expert chunk, row tile), and two CTAs
        # per unit cut the shard's time by 15 % (98 -> 83 us per layer on
        # B200); at 4 ranks the units already fill the GPU and the split costs
        # 8 %.  Results are the same on every rank for the same ksplit.
        self.batch_ksplit = 2 if ep_ranks >= 8 else 1
        if ep_ranks > 1 and exchange == "nccl":
            self.contrib = torch.zeros(k * bank.hidden, dtype=torch.float32, device=d)
            self.gathered = torch.zeros(ep_ranks * k * bank.hidden, dtype=torch.float32, device=d)
        elif ep_ranks > 1:
            from .ep import PeerExchange

            if L < 2:
                # one layer would reuse one slot buffer in consecutive steps
                raise ValueError("the peer-memory exchange needs at least two MoE layers; "
                                 "use exchange='nccl'")

            self.xchg = PeerExchange(group, ep_ranks, ep_rank, bank.hidden, k, d)
        self.graph = None
        self.pdl = True
        # L2 prefetch of the next launch's routed expert records (a hint:
        # results are the same with it off)
        self.prefetch = True
        nb = _lib.load().ervf_routesum_scratch_bytes(bank.hidden, k)
        self.scratch = torch.zeros(nb, dtype=torch.uint8, device=d)
        # One launch per token on one GPU (ervf_moe_token: every layer's up
        # and down rows as one claimed work list, bit-identical to the
        # per-layer launches); False runs the per-layer launches.
        # With expert parallelism over peer memory (exchange "p2p", up to 8
        # ranks) the token is one launch per rank too (ervf_moe_token_ep: each
        # rank's slot rows go to every rank over NVLink inside the launch),
        # bit-identical to one GPU; False runs the per-layer launches and one
        # exchange kernel per layer.  B200, batch 1, through the public API:
        # 1604 / 1568 / 1595 tok/s at 2 / 4 / 8 ranks for the one launch,
        # 1457 / 1530 / 1602-1606 for the per-layer launches.
        token_ep = exchange == "p2p" and 1 < ep_ranks <= 8
        self.token = ep_ranks == 1 or token_ep
        # step_with_router in one launch too (router items inside the token
        # kernel): bit-identical to the per-layer router + expert launches and,
        # on B200, 0.896 ms per 24-layer token against 0.930 ms for them
        self.token_router = ep_ranks == 1
        self.layer_ptrs = self.tok_scratch = self.tok_xchg = None
        if self.token or token_ep:
            addrs = ([ptr(t) for t in bank.up_codes] + [ptr(t) for t in bank.up_scales]
                     + [ptr(t) for t in bank.dn_codes] + [ptr(t) for t in bank.dn_scales]
                     + [ptr(t) for t in bank.globals])
            self.layer_ptrs = torch.tensor(addrs, dtype=torch.int64, device=d)
            if ep_ranks == 1:
                nb = _lib.load().ervf_moe_token_scratch_bytes(L, bank.hidden, bank.inter, k)
                self.tok_scratch = torch.zeros(nb, dtype=torch.uint8, device=d)
            else:
                from .ep import PeerExchange

                nb = int(_lib.load().ervf_moe_token_ep_scratch_bytes(L, bank.hidden, bank.inter, k))
                # every rank's token scratch, mapped on this GPU (CUDA IPC)
                self.tok_xchg = PeerExchange(group, ep_ranks, ep_rank, bank.hidden, k, d, nbytes=nb)
                self._tok_peers = (ctypes.c_uint64 * ep_ranks)(*self.tok_xchg.peers.cpu().tolist())
                self.prepare_token_ep()

    def prepare_token_ep(self) -> None:
        """Resets this rank's expert-parallel token scratch (counters, entry
        flags, unwritten slot rows) and waits until every rank has: before the
        first token, and on every rank after a timeout.  Collective."""
        import torch.distributed as dist

        b = self.bank
        _lib.call("ervf_moe_token_ep_prepare", self.tok_xchg.own, self.tok_xchg.nbytes, b.n_layers,
                  b.hidden, b.inter, self.top_k, self._s())
        torch.cuda.synchronize(b.device)
        dist.barrier(group=self.group)

    def _s(self) -> int:
        return int(torch.cuda.current_stream(self.bank.device).cuda_stream)

    def route(self, rlogs: torch.Tensor) -> None:
        """Routes every layer of the token in one launch (rlogs f32[L][E])."""
        b = self.bank
        self.fused.route_topk_batched(rlogs, None, self.ids, self.w, b.n_layers, b.n_experts,
                                      self.top_k, self.scaling)

    def layer(self, l: int, x: torch.Tensor, out: torch.Tensor, first: bool = False) -> None:
        """out = x + sum_s w_s * down_{e_s}(relu2(up_{e_s}(x))) in route order,
        with layer l's route already in self.ids[l] / self.w[l]."""
        b, f, k = self.bank, self.fused, self.top_k
        ids, w = self.ids[l], self.w[l]
        if self.ep_ranks == 1:
            # The routing launch precedes the first up launch directly, so
            # that one must wait before reading ids; every later launch may
            # start streaming its experts while its predecessor drains.  The
            # up launch queues this layer's down records into L2, the down
            # launch the next layer's up records (routes of every layer are
            # known before the step).
            flags = _lib.LAUNCH_PDL | (0 if first else _lib.LAUNCH_IDS_READY)
            if not self.pdl:
                flags = 0
            nxt = l + 1 if (self.prefetch and l + 1 < b.n_layers) else None
            pf = (ptr(b.up_codes[nxt]), ptr(b.up_scales[nxt]), ptr(self.ids[nxt])) if nxt is not None \
                else (0, 0, 0)
            _lib.call("ervf_moe_layer", ptr(b.up_codes[l]), ptr(b.up_scales[l]), int(b.up_code_bytes),
                      int(b.up_scale_bytes), ptr(b.dn_codes[l]), ptr(b.dn_scales[l]),
                      int(b.dn_code_bytes), int(b.dn_scale_bytes), ptr(ids), ptr(b.globals[l]),
                      ptr(w), k, ptr(x), ptr(self.act), ptr(out), b.hidden, b.inter, b.n_experts,
                      ptr(self.scratch), self.scratch.numel(), *pf, flags, self._s())
            return
        if self.xchg is not None:
            from .ep import exchange_buffer

            buf = exchange_buffer(l, b.n_layers)
            up_flags = (_lib.LAUNCH_PDL | (0 if first else _lib.LAUNCH_IDS_READY)) if self.pdl else 0
            _lib.call("ervf_ep_expert_slots_ex", ptr(b.up_codes[l]), ptr(b.up_scales[l]),
                      int(b.up_code_bytes), int(b.up_scale_bytes), ptr(b.dn_codes[l]),
                      ptr(b.dn_scales[l]), int(b.dn_code_bytes), int(b.dn_scale_bytes), ptr(ids),
                      ptr(b.globals[l]), k, ptr(x), ptr(self.act), self.xchg.slots(buf), b.hidden,
                      b.inter, self.ep_ranks, self.ep_rank, f._width(), up_flags, self._s())
            _lib.call("ervf_ep_exchange_route_sum", ptr(self.xchg.peers), self.ep_ranks,
                      self.ep_rank, buf, ptr(ids), ptr(w), k, ptr(x), ptr(out), b.hidden,
                      self.exchange_timeout_ms, _lib.LAUNCH_PDL if self.pdl else 0, self._s())
            return
        import torch.distributed as dist

        _lib.call("ervf_ep_expert_slots", ptr(b.up_codes[l]), ptr(b.up_scales[l]),
                  int(b.up_code_bytes), int(b.up_scale_bytes), ptr(b.dn_codes[l]),
                  ptr(b.dn_scales[l]), int(b.dn_code_bytes), int(b.dn_scale_bytes), ptr(ids),
                  ptr(b.globals[l]), k, ptr(x), ptr(self.act), ptr(self.contrib), b.hidden, b.inter,
                  self.ep_ranks, self.ep_rank, f._width(), self._s())
        dist.all_gather_into_tensor(self.gathered, self.contrib, group=self.group)
        _lib.call("ervf_ep_route_sum", ptr(self.gathered), ptr(ids), ptr(w), k, ptr(x), ptr(out),
                  b.hidden, self.ep_ranks, self._s())

    def close(self) -> None:
        """Releases the peer-exchange regions (collective over the ranks)."""
        if self.xchg is not None:
            self.xchg.close()
            self.xchg = None
        if self._bxchg is not None:
            self._bxchg.close()
            self._bxchg = None
        if self.tok_xchg is not None:
            self.tok_xchg.close()
            self.tok_xchg = None

    def step_batch(self, x_in: torch.Tensor, rlogs: torch.Tensor) -> torch.Tensor:
        """A decode batch of T tokens through every layer, expert-major on the
        tensor cores (tolerance path).  x_in f32[T][hidden], rlogs
        f32[L][T][E].  Returns the buffer holding x after the last layer.
        With expert parallelism every rank streams only the experts it owns
        for all T tokens, and one exchange kernel per layer reads each pair's
        output from its owner over NVLink before the route-order sum (same
        result as one GPU).  The first call with a new T sets up the exchange
        regions (a collective over the ranks), so make it outside graph
        capture."""
        b, k = self.bank, self.top_k
        L, T = b.n_layers, x_in.shape[0]
        d = b.device
        if getattr(self, "_bt", None) != T:
            self._bt = T
            self.bids = torch.zeros(L * T, k, dtype=torch.int32, device=d)
            self.bw = torch.zeros(L * T, k, dtype=torch.float32, device=d)
            self.bx = torch.zeros(2, T, b.hidden, dtype=torch.float32, device=d)
            if self.ep_ranks > 1:
                from .ep import PeerExchange

                if self._bxchg is not None:
                    self._bxchg.close()
                self._bxchg = PeerExchange(self.group, self.ep_ranks, self.ep_rank, b.hidden, T * k, d)
                self._bnb = int(_lib.load().ervf_moe_batched_scratch_bytes(T, k, b.hidden, b.inter))
                self._bscr = torch.empty(self._bnb, dtype=torch.uint8, device=d)
        self.fused.route_topk_batched(rlogs, None, self.bids, self.bw, L * T, b.n_experts, k,
                                      self.scaling)
        cur = x_in
        for l in range(L):
            nxt = self.bx[l & 1]
            ids, w = self.bids[l * T:(l + 1) * T], self.bw[l * T:(l + 1) * T]
            if self.ep_ranks == 1:
                self.fused.moe_batched(b.up_codes[l], b.up_scales[l], b.up_code_bytes,
                                       b.up_scale_bytes, b.dn_codes[l], b.dn_scales[l],
                                       b.dn_code_bytes, b.dn_scale_bytes, b.globals[l], ids, w, T, k,
                                       b.n_experts, cur, nxt, b.hidden, b.inter,
                                       ksplit=self.batch_ksplit)
            else:
                from .ep import exchange_buffer

                buf = exchange_buffer(l, L)
                _lib.call("ervf_moe_batched_ep_slots_ex", ptr(b.up_codes[l]), ptr(b.up_scales[l]),
                          int(b.up_code_bytes), int(b.up_scale_bytes), ptr(b.dn_codes[l]),
                          ptr(b.dn_scales[l]), int(b.dn_code_bytes), int(b.dn_scale_bytes),
                          ptr(b.globals[l]), ptr(ids), T, k, b.n_experts, ptr(cur),
                          self._bxchg.slots(buf), b.hidden, b.inter, self.ep_ranks, self.ep_rank,
                          self.batch_ksplit, ptr(self._bscr), self._bnb, self._s())
                _lib.call("ervf_ep_batch_exchange_route_sum", ptr(self._bxchg.peers), self.ep_ranks,
                          self.ep_rank, buf, ptr(ids), ptr(w), T, k, ptr(cur), ptr(nxt), b.hidden,
                          b.inter, ptr(self._bscr), self._bnb, self.exchange_timeout_ms, self._s())
            cur = nxt
        return cur

    def step_with_router(self, x_in: torch.Tensor, gate_w: torch.Tensor,
                         gate_b: torch.Tensor | None = None) -> torch.Tensor:
        """One decode token through all layers with the router on the device
        between them: per layer one launch computes the router logits from
        the current hidden state (gate_w f32[L][E][hidden], the reference's
        mv_f32) and routes them (route_topk, gate_b f32[L][E] or None), then
        the grouped up and down launches follow -- the reference's per-layer
        mv_f32 + route_topk + experts sequence (runtime.py:705-746), single
        GPU, PDL-chained.  Returns the buffer holding x after the last layer."""
        b, f, k = self.bank, self.fused, self.top_k
        if self.ep_ranks != 1:
            raise ValueError("step_with_router runs on one GPU")
        if self.token and self.token_router and b.n_experts <= 256:
            # routers and experts of every layer in one launch (the token
            # kernel's router items route up to 256 experts per layer)
            out = self.xs[(b.n_layers - 1) & 1]
            self.token_step_router(x_in, out, gate_w, gate_b)
            return out
        if getattr(self, "rlog", None) is None:
            self.rlog = torch.zeros(b.n_experts, dtype=torch.float32, device=b.device)
        pdl = _lib.LAUNCH_PDL if self.pdl else 0
        cur = x_in
        for l in range(b.n_layers):
            nxt = self.xs[l & 1]
            ids, w = self.ids[l], self.w[l]
            f.route_gemv_topk(self.rlog, gate_w[l], cur, None if gate_b is None else gate_b[l], ids,
                              w, b.n_experts, b.hidden, k, self.scaling, flags=pdl)
            # the router launch directly precedes the up launch: up waits
            # before reading ids; down may read them early
            f.moe_up_grouped(b.up_codes[l], b.up_scales[l], b.up_code_bytes, b.up_scale_bytes, ids,
                             b.globals[l], k, cur, self.act, b.inter, b.hidden, flags=pdl)
            f.moe_down_routesum(b.dn_codes[l], b.dn_scales[l], b.dn_code_bytes, b.dn_scale_bytes,
                                ids, b.globals[l], w, k, self.act, nxt, b.hidden, b.inter, resid=cur,
                                flags=pdl | (_lib.LAUNCH_IDS_READY if self.pdl else 0))
            cur = nxt
        return cur

    def step(self, x_in: torch.Tensor, rlogs: torch.Tensor) -> torch.Tensor:
        """One decode token through all layers; rlogs f32[L][E] are the
        router logits of every layer.  Returns the buffer holding x after
        the last layer."""
        self.route(rlogs)
        if self.token:
            out = self.xs[(self.bank.n_layers - 1) & 1]
            if self.ep_ranks == 1:
                self.token_step(x_in, out)
            else:
                self.token_step_ep(x_in, out)
            return out
        cur = x_in
        for l in range(self.bank.n_layers):
            nxt = self.xs[l & 1]
            self.layer(l, cur, nxt, first=(l == 0))
            cur = nxt
        return cur

    def device_status(self) -> int:
        """Read and clear the library's device error words; after a timeout
        zero this decoder's scratch buffers (and the FusedNVFP4 caches) so the
        next step starts from clean counters.  Returns the status.  With
        expert parallelism the token scratch is shared by all ranks: after a
        timeout every rank calls ``prepare_token_ep()`` (collective) before
        the next token."""
        st = self.fused.device_status()
        if st == _lib.ERR_TIMEOUT:
            self.scratch.zero_()
            if self.tok_scratch is not None:
                self.tok_scratch.zero_()
        return st

    def token_step_router(self, x_in: torch.Tensor, out: torch.Tensor, gate_w: torch.Tensor,
                          gate_b: torch.Tensor | None = None) -> None:
        """One token through every layer in one launch with the router on the
        device (ervf_moe_token_router): per layer rlog = gemv_f32(gate_w[l],
        x_l) and route_topk into self.ids[l] / self.w[l], then the layer's
        experts; out = x_L, bit-identical to the per-layer router + expert
        launches.  gate_w f32[L][E][hidden], gate_b f32[L][E] or None."""
        b = self.bank
        if gate_w.dtype != torch.float32 or gate_w.shape != (b.n_layers, b.n_experts, b.hidden):
            raise ValueError("gate_w must be f32 [n_layers][n_experts][hidden]")
        if gate_b is not None and (gate_b.dtype != torch.float32 or gate_b.shape != (b.n_layers, b.n_experts)):
            raise ValueError("gate_b must be f32 [n_layers][n_experts] or None")
        gw = gate_w.contiguous()
        gb = None if gate_b is None else gate_b.contiguous()
        key = (ptr(gw), 0 if gb is None else ptr(gb))
        if getattr(self, "_router_key", None) != key:
            rows = [ptr(gw[l]) for l in range(b.n_layers)]
            rows += [0] * b.n_layers if gb is None else [ptr(gb[l]) for l in range(b.n_layers)]
            self._router_ptrs = torch.cat([self.layer_ptrs,
                                           torch.tensor(rows, dtype=torch.int64, device=b.device)])
            self._router_key = key
            self._router_hold = (gw, gb)  # the addresses stay valid while held
        _lib.call("ervf_moe_token_router", ptr(self._router_ptrs), b.n_layers, int(b.up_code_bytes),
                  int(b.up_scale_bytes), int(b.dn_code_bytes), int(b.dn_scale_bytes), ptr(self.ids),
                  ptr(self.w), self.top_k, b.n_experts, float(np.float32(self.scaling)), 0, ptr(x_in),
                  ptr(out), b.hidden, b.inter, ptr(self.tok_scratch), self.tok_scratch.numel(),
                  _lib.LAUNCH_PDL if self.pdl else 0, self._s())

    def token_step_ep(self, x_in: torch.Tensor, out: torch.Tensor) -> None:
        """Every layer of one token in one launch on this rank of the
        expert-parallel group (ervf_moe_token_ep), routes in self.ids /
        self.w: every rank ends with the same out, bit-identical to one GPU.
        Every rank must run the same tokens in the same order."""
        b = self.bank
        _lib.call("ervf_moe_token_ep", ptr(self.layer_ptrs), b.n_layers, int(b.up_code_bytes),
                  int(b.up_scale_bytes), int(b.dn_code_bytes), int(b.dn_scale_bytes), ptr(self.ids),
                  ptr(self.w), self.top_k, b.n_experts, ptr(x_in), ptr(out), b.hidden, b.inter,
                  ctypes.cast(self._tok_peers, ctypes.c_void_p), self.ep_ranks, self.ep_rank,
                  self.tok_xchg.nbytes, self.exchange_timeout_ms,
                  _lib.LAUNCH_PDL if self.pdl else 0, self._s())

    def token_step(self, x_in: torch.Tensor, out: torch.Tensor, ids: torch.Tensor | None = None,
                   w: torch.Tensor | None = None) -> None:
        """Every layer of one token in one launch with the routes in
        self.ids / self.w (or the given int32 [L][top_k] ids and f32 weights):
        out = x_L, bit-identical to the per-layer chain (out may be x_in)."""
        b = self.bank
        ids = self.ids if ids is None else ids
        w = self.w if w is None else w
        _lib.call("ervf_moe_token", ptr(self.layer_ptrs), b.n_layers, int(b.up_code_bytes),
                  int(b.up_scale_bytes), int(b.dn_code_bytes), int(b.dn_scale_bytes), ptr(ids),
                  ptr(w), self.top_k, b.n_experts, ptr(x_in), ptr(out), b.hidden, b.inter,
                  ptr(self.tok_scratch), self.tok_scratch.numel(),
                  _lib.LAUNCH_PDL if self.pdl else 0, self._s())
