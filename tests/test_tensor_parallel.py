"""Tensor parallelism: the shard layout on the CPU (exact algebra), and the
NCCL-backed TP DiT forward against the single-GPU forward on 2 GPUs."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

import __graft_entry__

__graft_entry__.load_package()  # spawned workers import this module without conftest
from oasis_b200 import _lib  # noqa: E402
from oasis_b200 import tensor_parallel as TP  # noqa: E402
from tests.helpers import rel_l2  # noqa: E402


def test_shards_reassemble_the_projections():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(5, 1024, generator=g, dtype=torch.float64)
    wqkv = torch.randn(3072, 1024, generator=g, dtype=torch.float64)
    wo = torch.randn(1024, 1024, generator=g, dtype=torch.float64)
    w1 = torch.randn(4096, 1024, generator=g, dtype=torch.float64)
    w2 = torch.randn(1024, 4096, generator=g, dtype=torch.float64)
    for n in (2, 4, 8):
        full = x @ wqkv.T
        dl = 1024 // n
        for r in range(n):  # rank r's q | k | v columns are the heads [16 r / n, 16 (r + 1) / n)
            loc = x @ TP.shard_qkv(wqkv, n, r).T
            for sec in range(3):
                assert torch.equal(loc[:, sec * dl:(sec + 1) * dl],
                                   full[:, sec * 1024 + r * dl:sec * 1024 + (r + 1) * dl])
        a = torch.randn(5, 1024, generator=g, dtype=torch.float64)
        parts = sum(a[:, r * dl:(r + 1) * dl] @ TP.shard_cols(wo, n, r).T for r in range(n))
        assert torch.allclose(parts, a @ wo.T)
        parts = sum((x @ TP.shard_rows(w1, n, r).T) @ TP.shard_cols(w2, n, r).T for r in range(n))
        assert torch.allclose(parts, (x @ w1.T) @ w2.T)


def test_shard_struct_points_at_the_shards():
    """The OasisDitWeights handed to oasis_dit_forward_tp: sub-block pointers are
    this rank's shards (1/n of the QKV / FC1 rows, O / FC2 columns), everything
    else is the replicated full struct."""
    from oasis_b200.weights import init_dit_weights

    sd = init_dit_weights(seed=3, n_blocks=2)
    n, r = 4, 1
    tpw = TP.TPDitWeights(sd, n, r, "cpu")
    st, full = tpw.struct, tpw.full.struct
    assert tpw.heads == 4 and st.num_subblocks == full.num_subblocks == 4
    for f in ("adaln_w", "adaln_b", "final_w", "final_b", "embed_w", "embed_b", "rope_spatial", "rope_temporal"):
        assert getattr(st, f) == getattr(full, f), f
    for i, blk in enumerate(tpw.sub):
        for k, t in blk.items():
            assert getattr(st.sub[i], k) == t.data_ptr(), (i, k)
        assert tuple(blk["qkv_w"].shape) == (3 * 1024 // n, 1024)
        assert tuple(blk["out_w"].shape) == (1024, 1024 // n)
        assert tuple(blk["fc1_w"].shape) == (4096 // n, 1024) and tuple(blk["fc1_b"].shape) == (4096 // n,)
        assert tuple(blk["fc2_w"].shape) == (1024, 4096 // n)
    # rank r's q rows are heads [16 r / n, 16 (r + 1) / n) of the checkpoint's q block
    q = sd["blocks.0.s_attn.to_qkv.weight"][:1024]
    assert torch.equal(tpw.sub[0]["qkv_w"][:256].float(), q[256:512].to(torch.bfloat16).float())
    with pytest.raises(ValueError):
        TP.TPDitWeights(sd, 3, 0, "cpu")


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tp_worker(rank, world, port, q):
    import torch.distributed as dist

    from oasis_b200 import engine as E
    from oasis_b200 import host as H
    from oasis_b200.weights import DitDeviceWeights, init_dit_weights

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        dev = torch.device("cuda", rank)
        sd = init_dit_weights(seed=3, n_blocks=2, bias_std=0.02)
        B, T = 4, 3
        g = torch.Generator().manual_seed(1)
        z = torch.randn(B, T, H.N_PATCHES, H.D_MODEL, generator=g).to(dev)
        cond = torch.randn(B, T, H.D_MODEL, generator=g).to(dev)
        tpw = TP.TPDitWeights(sd, world, rank, dev)
        sc = TP.TPScratch(tpw, B, T, dev)
        v_tp = torch.empty(B, H.N_PATCHES, H.OUT_DIM, device=dev)
        TP.dit_forward_tp(tpw, z.clone(), cond, v_tp, sc)
        dw = DitDeviceWeights(sd, dev)
        v_1 = torch.empty_like(v_tp)
        E.dit_forward(dw, z.clone(), cond, v_1, E.workspace(E.dit_workspace_bytes(B, T), dev))
        # the sequence-parallel form over NCCL (reduce-scatter + all-gather, bf16 partials)
        bufs = TP.TPSpBuffers(tpw, B, T, dev)
        Bl = B // world
        v_sp = torch.empty_like(v_tp)
        TP.dit_forward_tp_sp(tpw, z[rank * Bl:(rank + 1) * Bl].clone(), cond[rank * Bl:(rank + 1) * Bl].contiguous(),
                             v_sp, bufs)
        # overlapped: collectives on a second stream, one session per group
        v_ov = torch.empty_like(v_tp)
        TP.dit_forward_tp_sp(tpw, z[rank * Bl:(rank + 1) * Bl].clone(), cond[rank * Bl:(rank + 1) * Bl].contiguous(),
                             v_ov, bufs, comm_stream=torch.cuda.Stream(dev), chunks=Bl)
        # the same over peer memory: copy-engine transfers + the library's handshake kernels
        pc = TP.PeerCollectives(bufs)
        v_pc = torch.empty_like(v_tp)
        TP.dit_forward_tp_sp(tpw, z[rank * Bl:(rank + 1) * Bl].clone(), cond[rank * Bl:(rank + 1) * Bl].contiguous(),
                             v_pc, bufs, collectives=pc.callbacks)
        v_pco = torch.empty_like(v_tp)
        TP.dit_forward_tp_sp(tpw, z[rank * Bl:(rank + 1) * Bl].clone(), cond[rank * Bl:(rank + 1) * Bl].contiguous(),
                             v_pco, bufs, collectives=pc.callbacks, comm_stream=torch.cuda.Stream(dev), chunks=Bl)
        # the callbacks alone, as the library calls them: exact small integers
        st = torch.cuda.current_stream().cuda_stream
        rs, ag = pc.callbacks
        prims = {}
        for dt, code in ((torch.float32, _lib.OASIS_DTYPE_F32), (torch.bfloat16, _lib.OASIS_DTYPE_BF16)):
            count = 4096
            send = ((torch.arange(world * count, device=dev) % 17) * (rank + 1)).to(dt)
            recv = torch.full((count,), -1.0, device=dev, dtype=dt)
            rc1 = rs(send.data_ptr(), recv.data_ptr(), count, code, None, st)
            exp = (torch.arange(count, device=dev) + rank * count) % 17 * sum(range(1, world + 1))
            mine = torch.full((count,), float(rank + 1), device=dev, dtype=dt)
            into = torch.zeros(world * count, device=dev, dtype=dt)  # outside the shared region: staged
            rc2 = ag(mine.data_ptr(), into.data_ptr(), count, code, None, st)
            prims[str(dt)] = (rc1, rc2, torch.equal(recv.float(), exp.float()),
                              torch.equal(into.float(), torch.arange(world, device=dev).repeat_interleave(count) + 1.0))
        torch.cuda.synchronize()
        pc.check()
        pc.close()
        from oracle import oasis_oracle as O
        ref = O.dit_forward(z.cpu(), cond.cpu(), sd)[:, -1]
        q.put((rank, rel_l2(v_tp, v_1), rel_l2(v_tp, ref), rel_l2(v_sp, ref), rel_l2(v_ov, ref), rel_l2(v_pc, ref),
               rel_l2(v_pco, ref), rel_l2(v_pc, v_sp), prims))
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp2_matches_single_gpu():
    """2 GPUs: the all-reduce TP forward (NCCL) against the single-GPU forward and
    the oracle; the sequence-parallel forward against the oracle over NCCL and
    over peer memory (copy engines + handshake kernels), in order and
    overlapped; the peer-memory reduce-scatter / all-gather callbacks on exact
    small integers."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_tp_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for _, err, err_tp, err_sp, err_ov, err_pc, err_pco, pc_vs_nccl, prims in res:
        assert err < 5e-3, res  # bf16 operands; partial sums re-associated across ranks
        # every TP form against the fp32 oracle (NCCL and peer-memory collectives)
        assert max(err_tp, err_sp, err_ov, err_pc, err_pco) < 1e-2, res
        assert pc_vs_nccl < 5e-3, res  # the two collective back ends differ only in summation rounding
        for rc1, rc2, rs_ok, ag_ok in prims.values():
            assert rc1 == 0 and rc2 == 0 and rs_ok and ag_ok, prims


# ----------------------------------------------------------------- sequence-parallel TP
def _cb_worker(rank, world, port, q):
    """gloo rank: the reduce-scatter / all-gather callbacks of OasisTpSpArgs, called
    through their C function pointers as the library calls them."""
    import ctypes as C

    import torch.distributed as dist

    from oasis_b200 import _lib

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        out = {}
        for dtype, code in ((torch.float32, _lib.OASIS_DTYPE_F32), (torch.bfloat16, _lib.OASIS_DTYPE_BF16)):
            count = 6
            send = (torch.arange(world * count, dtype=torch.float32) * (rank + 1)).to(dtype)
            recv = torch.full((count,), -1.0, dtype=dtype)
            xl = torch.full((count,), float(rank), dtype=dtype)
            xg = torch.zeros(world * count, dtype=dtype)
            reg = {t.data_ptr(): t for t in (send, recv, xl, xg)}
            errors = []
            rs, ag = TP.dist_collectives(reg, None, errors)
            f_rs = C.cast(rs, C.c_void_p).value
            f_ag = C.cast(ag, C.c_void_p).value
            rs_c = _lib.COLLECTIVE_FN(f_rs)
            ag_c = _lib.COLLECTIVE_FN(f_ag)
            rc1 = rs_c(send.data_ptr(), recv.data_ptr(), count, code, None, None)
            rc2 = ag_c(xl.data_ptr(), xg.data_ptr(), count, code, None, None)
            rc3 = ag_c(12345, xg.data_ptr(), count, code, None, None)  # a buffer the registry does not know
            out[str(dtype)] = (rc1, rc2, rc3, recv.float().tolist(), xg.float().tolist(), len(errors))
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


def test_tp_sp_collective_callbacks_gloo_world2():
    """The callback contract on two gloo ranks (CPU): reduce_scatter sums every
    rank's send and leaves rank r its r-th slice, all_gather lays the ranks' sends
    out rank-major, an unknown buffer returns a non-zero status (which aborts the
    library's forward) and is recorded."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_cb_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    world, count = 2, 6
    for rank in range(world):
        for dt, (rc1, rc2, rc3, recv, xg, nerr) in res[rank].items():
            assert (rc1, rc2) == (0, 0) and rc3 != 0 and nerr == 1, (rank, dt)
            total = [i * sum(k + 1 for k in range(world)) for i in range(world * count)]
            assert recv == total[rank * count:(rank + 1) * count], (rank, dt)
            assert xg == [float(k) for k in range(world) for _ in range(count)], (rank, dt)


def test_tp_sp_entry_validates_without_a_gpu():
    import ctypes as C

    from oasis_b200 import _lib

    lib = _lib.load()
    w = _lib.OasisDitWeights()
    cb = _lib.COLLECTIVE_FN(lambda *a: 0)
    a = _lib.OasisTpSpArgs(5, 2, 8, 0, 2, 16, 16, 16, 1, 16, 16, 16, 16, 16, cb, cb, None, 16, 1 << 40)
    # 5 sessions are not a multiple of the 2 ranks
    assert lib.oasis_dit_forward_tp_sp(C.byref(w), C.byref(a), None) == -1
    assert b"multiple of world" in lib.oasis_last_error()
    a.batch, a.heads = 6, 4  # 4 heads x 2 ranks != 16
    assert lib.oasis_dit_forward_tp_sp(C.byref(w), C.byref(a), None) == -1
    a.heads, a.partial_dtype = 8, 7  # unknown partial type
    assert lib.oasis_dit_forward_tp_sp(C.byref(w), C.byref(a), None) == -1
    a.partial_dtype, a.reduce_scatter = 1, _lib.COLLECTIVE_FN()  # no collective
    assert lib.oasis_dit_forward_tp_sp(C.byref(w), C.byref(a), None) == -1
    assert lib.oasis_tp_sp_workspace_size(6, 2, 8, 2) > 0
    assert lib.oasis_tp_sp_workspace_size(5, 2, 8, 2) == 0


class _EmulatedGroup:
    """`world` tensor-parallel ranks in one process on one GPU: one host thread and
    one CUDA stream per rank, each inside its own oasis_dit_forward_tp_sp call.
    A collective callback records an event on its rank's stream and meets the
    other ranks at a host barrier; rank 0's thread then does the whole
    collective with torch copies/adds on a separate stream after every rank's
    event, and each rank's stream waits for that before its next kernel. No kernel
    waits on another kernel: the ranks rendezvous on the host only."""

    def __init__(self, world: int):
        import threading

        self.world = world
        self.barrier = threading.Barrier(world, timeout=300)
        self.slots = [None] * world
        self.comm = torch.cuda.Stream()
        self.done = None

    def collectives(self, rank: int, registry: dict):
        from oasis_b200 import _lib

        def make(kind):
            def cb(send, recv, count, dtype, user, st):
                try:
                    stream = torch.cuda.ExternalStream(st)  # the stream the library orders this collective on
                    n = self.world
                    s = TP.buffer_view(registry, send, count * (n if kind == "rs" else 1))
                    r = TP.buffer_view(registry, recv, count * (1 if kind == "rs" else n))
                    ev = torch.cuda.Event()
                    ev.record(stream)
                    self.slots[rank] = (s, r, ev, count)
                    self.barrier.wait()
                    if rank == 0:
                        with torch.cuda.stream(self.comm):
                            for *_, e, _ in self.slots:
                                self.comm.wait_event(e)
                            if kind == "rs":
                                total = sum(s2.reshape(self.world, -1).float() for s2, *_ in self.slots)
                                for k, (_, r2, _, _) in enumerate(self.slots):
                                    r2.reshape(-1).copy_(total[k])
                            else:
                                for _, r2, _, _ in self.slots:
                                    for j, (s2, *_) in enumerate(self.slots):
                                        r2.reshape(self.world, -1)[j].copy_(s2.reshape(-1))
                            self.done = torch.cuda.Event()
                            self.done.record(self.comm)
                    self.barrier.wait()
                    stream.wait_event(self.done)
                    self.barrier.wait()  # everyone has queued the wait before `done` is replaced
                    return 0
                except Exception:  # noqa: BLE001
                    self.barrier.abort()
                    return -2
            return _lib.COLLECTIVE_FN(cb)

        return make("rs"), make("ag")


def _tp_sp_emulated(sd, world, z, cond, partial_dtype, chunks=1):
    import threading

    B, T = z.shape[0], z.shape[1]
    dev = torch.device("cuda")
    grp = _EmulatedGroup(world)
    outs, errs = [None] * world, []
    ranks = []
    for r in range(world):
        tpw = TP.TPDitWeights(sd, world, r, dev)
        bufs = TP.TPSpBuffers(tpw, B, T, dev, partial_dtype)
        v = torch.empty(B, 144, 64, device=dev)
        Bl = B // world
        zl = z[r * Bl:(r + 1) * Bl].contiguous().to(dev)
        cl = cond[r * Bl:(r + 1) * Bl].contiguous().to(dev)
        ranks.append((tpw, bufs, v, zl, cl, torch.cuda.Stream(), torch.cuda.Stream() if chunks > 1 else None))
    torch.cuda.synchronize()

    def run(r):
        tpw, bufs, v, zl, cl, st, cst = ranks[r]
        try:
            with torch.cuda.stream(st):
                TP.dit_forward_tp_sp(tpw, zl, cl, v, bufs, grp.collectives(r, bufs.registry(v)), stream=st,
                                     comm_stream=cst, chunks=chunks, reserve_sms=16 if chunks > 1 else 0)
            st.synchronize()
            outs[r] = v.cpu()
        except Exception as e:  # noqa: BLE001
            errs.append(e)
            grp.barrier.abort()

    th = [threading.Thread(target=run, args=(r,)) for r in range(world)]
    for t in th:
        t.start()
    for t in th:
        t.join(timeout=600)
    assert not errs, errs
    return outs


@pytest.mark.gpu
@pytest.mark.parametrize("world,dtype,chunks", [(2, torch.bfloat16, 1), (2, torch.float32, 1), (4, torch.bfloat16, 1),
                                                (2, torch.bfloat16, 2)])
def test_tp_sp_emulated_ranks_match_oracle(world, dtype, chunks):
    """Sequence-parallel TP, full 16-block DiT, `world` ranks emulated on one GPU
    (host threads + streams; the collectives as torch ops), against the fp32
    oracle: every rank's gathered v of the last frame."""
    from oracle import oasis_oracle as O
    from oasis_b200 import host as H
    from oasis_b200.weights import init_dit_weights
    from tests.helpers import COS_TOL, REL_L2_TOL, cosine

    sd = init_dit_weights(seed=3, bias_std=0.02)
    B, T = 4, 3
    g = torch.Generator().manual_seed(5)
    z = torch.randn(B, T, H.N_PATCHES, H.D_MODEL, generator=g)
    cond = torch.randn(B, T, H.D_MODEL, generator=g)
    outs = _tp_sp_emulated(sd, world, z, cond, dtype, chunks)  # chunks > 1: communication stream + 2 groups
    ref = O.dit_forward(z, cond, sd)[:, -1]
    for r, v in enumerate(outs):
        assert rel_l2(v, ref) < REL_L2_TOL and cosine(v, ref) > COS_TOL, (r, rel_l2(v, ref), cosine(v, ref))
        assert torch.equal(v, outs[0])  # the gathered result is the same on every rank
