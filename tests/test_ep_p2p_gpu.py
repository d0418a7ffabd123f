"""Expert-parallel exchange over peer memory (ervf_ep_exchange_route_sum).

One GPU: the exchange kernel as a single rank reads the slot outputs the
grouped launches wrote into its region and sums them in route order --
bit-identical to the single-GPU routed sum (the oracle), through every slot
buffer in turn; and a wait on a flag that nothing sets runs out after its
limit, reports ERVF_ERR_TIMEOUT and leaves the context usable.

The batched block as one rank equals ervf_moe_batched bit for bit.

Two or more GPUs (skipped otherwise): one process per GPU over NCCL, experts
sharded by id, every layer's slots exchanged over NVLink -- inside the
one-launch token kernel (ervf_moe_token_ep) and by the per-layer exchange
kernel; each rank's x after the last layer must equal one GPU's bit for bit,
eager and in a CUDA graph, and the batched block's likewise.
"""

from __future__ import annotations

import ctypes
import datetime
import os
import socket
import sys
import traceback
from pathlib import Path

import numpy as np
import pytest
import torch

from conftest import bits_equal, random_nvfp4, x_regime

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
HIDDEN, INTER, K, E = 2688, 1856, 6, 8


def _t(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _stream(dev):
    return int(torch.cuda.current_stream(dev).cuda_stream)


class _Region:
    """One exchange region of this process (alloc / free through the C ABI)."""

    def __init__(self, hidden, k):
        from ervf_b200 import _lib

        self.lib = _lib
        self.nbytes = int(_lib.load().ervf_ep_region_bytes(hidden, k))
        own = ctypes.c_void_p()
        self.handle = ctypes.create_string_buffer(64)
        _lib.call("ervf_ep_region_alloc", self.nbytes, ctypes.byref(own), self.handle)
        self.ptr = int(own.value)

    def slots(self, buf, k, hidden):
        return self.ptr + 1024 + buf * k * hidden * 4

    def free(self):
        self.lib.call("ervf_ep_region_free", self.ptr)


@pytest.fixture(scope="module")
def experts():
    ups = [random_nvfp4(INTER, HIDDEN, seed=3000 + e) for e in range(E)]
    dns = [random_nvfp4(HIDDEN, INTER, seed=3500 + e) for e in range(E)]
    return ups, dns


def test_single_rank_exchange_matches_oracle(oracle, experts, cuda):
    from ervf_b200 import _lib

    ups, dns = experts
    up_c = _t(np.concatenate([u[0] for u in ups]), cuda)
    up_s = _t(np.concatenate([u[1] for u in ups]), cuda)
    dn_c = _t(np.concatenate([d[0] for d in dns]), cuda)
    dn_s = _t(np.concatenate([d[1] for d in dns]), cuda)
    glob = _t(np.array([[d[2], u[2]] for u, d in zip(ups, dns)], np.float32), cuda)
    cb, sb = ups[0][0].size, ups[0][1].size
    reg = _Region(HIDDEN, K)
    try:
        peers = torch.tensor([reg.ptr], dtype=torch.int64, device=cuda)
        act = torch.zeros(K * INTER, device=cuda)
        r = np.random.default_rng(5)
        for step, buf in enumerate((0, 1, 2, 0, 1)):
            rlog = r.standard_normal(E).astype(np.float32)
            ids, w = oracle.route_topk(rlog, np.zeros(E, np.float32), K)
            x = x_regime(HIDDEN, "bf16", seed=40 + step)
            xd, idsd, wd = _t(x, cuda), _t(ids, cuda), _t(w, cuda)
            out = torch.full((HIDDEN,), float("nan"), device=cuda)
            flags = _lib.LAUNCH_PDL if step % 2 else 0
            _lib.call("ervf_ep_expert_slots_ex", up_c.data_ptr(), up_s.data_ptr(), cb, sb,
                      dn_c.data_ptr(), dn_s.data_ptr(), cb, sb, idsd.data_ptr(), glob.data_ptr(),
                      K, xd.data_ptr(), act.data_ptr(), reg.slots(buf, K, HIDDEN), HIDDEN, INTER,
                      1, 0, 0, flags, _stream(cuda))
            _lib.call("ervf_ep_exchange_route_sum", peers.data_ptr(), 1, 0, buf, idsd.data_ptr(),
                      wd.data_ptr(), K, xd.data_ptr(), out.data_ptr(), HIDDEN, 2000, flags,
                      _stream(cuda))
            torch.cuda.synchronize()
            ex = {e: (*ups[e], *dns[e]) for e in range(E)}
            want = (x + oracle.moe_block(x, ex, ids, w, HIDDEN, INTER)).astype(np.float32)
            assert bits_equal(out.cpu().numpy(), want), (step, buf)
        assert _lib.load().ervf_device_status() == _lib.OK
    finally:
        reg.free()


def test_single_rank_batched_exchange_matches_moe_batched(fused, cuda):
    """The expert-parallel batched block as one rank (slots into the exchange
    region, then the batched exchange + route sum) equals ervf_moe_batched
    bit for bit, through three slot buffers in turn, without and with the
    K-split."""
    from ervf_b200 import _lib
    from ervf_b200.moe import ExpertBank

    T, k, E2 = 8, 6, 16
    eb = ExpertBank.synthetic(1, E2, HIDDEN, INTER, cuda, seed=9)
    g = torch.Generator(device=cuda)
    g.manual_seed(4)
    reg = _Region(HIDDEN, T * k)
    try:
        peers = torch.tensor([reg.ptr], dtype=torch.int64, device=cuda)
        nb = int(_lib.load().ervf_moe_batched_scratch_bytes(T, k, HIDDEN, INTER))
        scr = torch.empty(nb, dtype=torch.uint8, device=cuda)
        for buf, ks in ((0, 1), (1, 2), (2, 2)):
            x = torch.randn(T, HIDDEN, generator=g, device=cuda)
            rl = torch.randn(T, E2, generator=g, device=cuda)
            ids = torch.zeros(T, k, dtype=torch.int32, device=cuda)
            w = torch.zeros(T, k, device=cuda)
            fused.route_topk_batched(rl, None, ids, w, T, E2, k, 1.0)
            want = torch.full((T, HIDDEN), float("nan"), device=cuda)
            fused.moe_batched(eb.up_codes[0], eb.up_scales[0], eb.up_code_bytes, eb.up_scale_bytes,
                              eb.dn_codes[0], eb.dn_scales[0], eb.dn_code_bytes, eb.dn_scale_bytes,
                              eb.globals[0], ids, w, T, k, E2, x, want, HIDDEN, INTER, ksplit=ks)
            out = torch.full((T, HIDDEN), float("nan"), device=cuda)
            _lib.call("ervf_moe_batched_ep_slots_ex", eb.up_codes[0].data_ptr(),
                      eb.up_scales[0].data_ptr(), eb.up_code_bytes, eb.up_scale_bytes,
                      eb.dn_codes[0].data_ptr(), eb.dn_scales[0].data_ptr(), eb.dn_code_bytes,
                      eb.dn_scale_bytes, eb.globals[0].data_ptr(), ids.data_ptr(), T, k, E2,
                      x.data_ptr(), reg.slots(buf, T * k, HIDDEN), HIDDEN, INTER, 1, 0, ks,
                      scr.data_ptr(), nb, _stream(cuda))
            _lib.call("ervf_ep_batch_exchange_route_sum", peers.data_ptr(), 1, 0, buf,
                      ids.data_ptr(), w.data_ptr(), T, k, x.data_ptr(), out.data_ptr(), HIDDEN,
                      INTER, scr.data_ptr(), nb, 2000, _stream(cuda))
            torch.cuda.synchronize()
            assert torch.isfinite(want).all()
            assert torch.equal(want.view(torch.int32), out.view(torch.int32)), buf
        assert _lib.load().ervf_device_status() == _lib.OK
    finally:
        reg.free()


def test_exchange_wait_times_out_on_unset_flag(cuda):
    """Two ranks declared, both table entries this process's own region: the
    flag of rank 1 is never published, so the bounded wait runs out (0.2 s),
    the output stays unwritten and the status reads ERVF_ERR_TIMEOUT."""
    from ervf_b200 import _lib

    k, hidden = 2, 256
    reg = _Region(hidden, k)
    try:
        peers = torch.tensor([reg.ptr, reg.ptr], dtype=torch.int64, device=cuda)
        ids = torch.tensor([0, 1], dtype=torch.int32, device=cuda)
        w = torch.tensor([0.5, 0.25], device=cuda)
        x = torch.ones(hidden, device=cuda)
        out = torch.full((hidden,), -7.0, device=cuda)
        _lib.call("ervf_ep_exchange_route_sum", peers.data_ptr(), 2, 0, 0, ids.data_ptr(),
                  w.data_ptr(), k, x.data_ptr(), out.data_ptr(), hidden, 200, 0, _stream(cuda))
        torch.cuda.synchronize()
        assert _lib.load().ervf_device_status() == _lib.ERR_TIMEOUT
        assert torch.all(out == -7.0)
        # the context is intact: a single-rank exchange on the same region works
        one = torch.tensor([reg.ptr], dtype=torch.int64, device=cuda)
        _lib.call("ervf_ep_exchange_route_sum", one.data_ptr(), 1, 0, 1, ids.data_ptr(),
                  w.data_ptr(), k, None, out.data_ptr(), hidden, 200, 0, _stream(cuda))
        torch.cuda.synchronize()
        assert _lib.load().ervf_device_status() == _lib.OK
        assert torch.all(out == 0.0)  # slots are zero: acc = 0, no residual
    finally:
        reg.free()


def test_exchange_rejects_bad_arguments(cuda):
    from ervf_b200 import _lib

    reg = _Region(256, 2)
    try:
        peers = torch.tensor([reg.ptr], dtype=torch.int64, device=cuda)
        ids = torch.zeros(2, dtype=torch.int32, device=cuda)
        w = torch.zeros(2, device=cuda)
        out = torch.zeros(256, device=cuda)
        args = [peers.data_ptr(), 1, 0, 0, ids.data_ptr(), w.data_ptr(), 2, None, out.data_ptr(),
                256, 100, 0, _stream(cuda)]
        for i, bad in ((3, 3), (1, 0), (2, 1), (9, 254), (10, 0), (6, 17)):
            a = list(args)
            a[i] = bad
            with pytest.raises(ValueError):
                _lib.call("ervf_ep_exchange_route_sum", *a)
    finally:
        reg.free()


# ---------------------------------------------------------------- 2+ GPUs

def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    try:
        sys.path.insert(0, str(ROOT))
        import torch.distributed as dist

        from ervf_b200.moe import ExpertBank, MoEDecoder

        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=60))
        L = 5  # odd: the last layer takes the third slot buffer
        bank = ExpertBank.synthetic(L, E, HIDDEN, INTER, dev, seed=7)
        one = MoEDecoder(bank, K)
        ep = MoEDecoder(bank, K, ep_ranks=world, ep_rank=rank, group=dist.group.WORLD,
                        exchange_timeout_ms=5000)
        g = torch.Generator(device=dev)
        g.manual_seed(11)
        xs = torch.randn(4, HIDDEN, generator=g, device=dev)
        rls = torch.randn(4, L, E, generator=g, device=dev)
        bad = []
        x_in = torch.zeros(HIDDEN, device=dev)
        r_in = torch.zeros(L, E, device=dev)
        # the one-launch token (ervf_moe_token_ep, the default) and the
        # per-layer launches with one exchange kernel per layer
        for token in (True, False):
            ep.token = token
            for t in range(2):  # eager steps
                x_in.copy_(xs[t])
                r_in.copy_(rls[t])
                want = one.step(x_in, r_in).clone()
                got = ep.step(x_in, r_in).clone()
                torch.cuda.synchronize()
                if not torch.equal(want.view(torch.int32), got.view(torch.int32)):
                    bad.append(("eager", token, t))
            graph = torch.cuda.CUDAGraph()
            s = torch.cuda.Stream(dev)
            s.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(s):
                ep.step(x_in, r_in)
            torch.cuda.current_stream(dev).wait_stream(s)
            with torch.cuda.graph(graph):
                y = ep.step(x_in, r_in)
            for t in range(2, 4):
                x_in.copy_(xs[t])
                r_in.copy_(rls[t])
                want = one.step(x_in, r_in).clone()
                graph.replay()
                torch.cuda.synchronize()
                if not torch.equal(want.view(torch.int32), y.view(torch.int32)):
                    bad.append(("graph", token, t))
            del graph
        # the batched block (expert-major, tensor cores), odd layer count; the
        # same K-split on both sides (results depend on it, not on the rank)
        one.batch_ksplit = ep.batch_ksplit
        T = 8
        xb = torch.randn(T, HIDDEN, generator=g, device=dev)
        rb = torch.randn(L, T, E, generator=g, device=dev)
        for t in range(2):
            want = one.step_batch(xb, rb).clone()
            got = ep.step_batch(xb, rb).clone()
            torch.cuda.synchronize()
            if not torch.equal(want.view(torch.int32), got.view(torch.int32)):
                bad.append(("batch", t))
            xb = want
        from ervf_b200 import _lib

        status = _lib.load().ervf_device_status()
        torch.cuda.synchronize()
        ep.close()
        dist.destroy_process_group()
        q.put((rank, "ok", (bad, status)))
    except Exception as exc:  # noqa: BLE001
        q.put((rank, "error", f"{type(exc).__name__}: {exc}\n{traceback.format_exc()[-600:]}"))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs (one process per GPU)")
def test_multi_gpu_exchange_bit_identical_to_one_gpu():
    import torch.multiprocessing as mp

    world = min(torch.cuda.device_count(), 8)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(300)
    res = {}
    while not q.empty():
        rank, status, payload = q.get()
        res[rank] = (status, payload)
    for p in ps:
        if p.is_alive():
            p.kill()
    assert [p.exitcode for p in ps] == [0] * world, res
    for rank in range(world):
        status, payload = res[rank]
        assert status == "ok", payload
        bad, dev_status = payload
        assert bad == [] and dev_status == 0, (rank, bad, dev_status)
