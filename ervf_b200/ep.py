"""Expert-parallel partition and exchange layout (host side).

Experts are sharded by id: expert e of every layer lives on rank
``e % world``.  Per layer and token every rank knows the route (ids, w) --
the router runs redundantly on every rank from the same logits -- computes
the down outputs y_s of the slots it owns into ``contrib[slot][hidden]``,
and one all-gather builds ``gathered[rank][slot][hidden]``.  The route-order
sum then reads slot s from rank ``owner(ids[s])``, so every rank ends with
the same x_{L+1}, bit-identical to one GPU (the reference is single-GPU;
its route-order contract is runtime.py:588-596).
"""

from __future__ import annotations


def owner(expert: int, world: int) -> int:
    return int(expert) % int(world)


def owned_slots(ids, world: int, rank: int) -> list[int]:
    return [s for s, e in enumerate(ids) if owner(int(e), world) == rank]


def gathered_index(ids, slot: int, world: int, top_k: int, hidden: int) -> int:
    """Flat offset of slot `slot`'s output in the gathered buffer."""
    return (owner(int(ids[slot]), world) * top_k + slot) * hidden


def experts_of_rank(n_experts: int, world: int, rank: int) -> list[int]:
    return list(range(rank, n_experts, world))


class PeerExchange:
    """Exchange regions of every rank, mapped over NVLink (CUDA IPC).

    Each rank allocates one region (``ervf_ep_region_alloc``), the 64-byte
    IPC handles are all-gathered over ``group``, and every peer's region is
    mapped here (``ervf_ep_region_open``).  ``peers`` is the device table
    u64[world] the exchange kernel reads; ``slots(buf)`` the address of slot
    buffer ``buf`` (``n_slots`` rows of ``hidden`` floats: top_k for one
    token, tokens * top_k for a batch) where this rank's down launch writes
    the slots it owns.  Set-up only: the
    per-layer exchange (``ervf_ep_exchange_route_sum``) is one kernel with no
    collective call.  ``close()`` unmaps the peers, waits for every rank and
    frees the own region.
    """

    def __init__(self, group, world: int, rank: int, hidden: int, n_slots: int, device,
                 nbytes: int | None = None):
        import ctypes

        import torch
        import torch.distributed as dist

        from . import _lib

        self.world, self.rank, self.hidden, self.n_slots = world, rank, hidden, n_slots
        self.group, self.device = group, device
        lib = _lib.load()
        # nbytes: a region of another layout (the one-launch token's scratch)
        self.nbytes = int(lib.ervf_ep_region_bytes(hidden, n_slots)) if nbytes is None else int(nbytes)
        if self.nbytes == 0:
            raise ValueError("unsupported exchange shape")
        own = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(64)
        with torch.cuda.device(device):
            _lib.call("ervf_ep_region_alloc", self.nbytes, ctypes.byref(own), handle)
        self.own = int(own.value)
        mine = torch.frombuffer(bytearray(handle.raw), dtype=torch.uint8).to(device)
        allh = torch.empty(world * 64, dtype=torch.uint8, device=device)
        dist.all_gather_into_tensor(allh, mine, group=group)
        allh = allh.cpu().numpy().tobytes()
        self.mapped = []
        ptrs = []
        with torch.cuda.device(device):
            for q in range(world):
                if q == rank:
                    ptrs.append(self.own)
                    continue
                p = ctypes.c_void_p()
                _lib.call("ervf_ep_region_open", allh[q * 64:(q + 1) * 64], ctypes.byref(p))
                self.mapped.append(int(p.value))
                ptrs.append(int(p.value))
        self.peers = torch.tensor(ptrs, dtype=torch.int64, device=device)
        # every rank has zeroed its region before anyone's first exchange
        dist.barrier(group=group)

    def slots(self, buf: int) -> int:
        return self.own + 1024 + buf * self.n_slots * self.hidden * 4

    def close(self) -> None:
        import torch.distributed as dist

        from . import _lib

        if self.own is None:
            return
        for p in self.mapped:
            _lib.call("ervf_ep_region_close", p)
        self.mapped = []
        dist.barrier(group=self.group)
        _lib.call("ervf_ep_region_free", self.own)
        self.own = None


def exchange_buffer(layer: int, n_layers: int) -> int:
    """Slot buffer of a layer: consecutive exchanges (the wrap from the last
    layer of one step to layer 0 of the next included) use different
    buffers -- alternate 0 / 1, and the last layer of an odd count takes 2.
    Needs n_layers >= 2."""
    if n_layers % 2 == 1 and layer == n_layers - 1:
        return 2
    return layer & 1
