"""The host side of tensor_parallel.PeerCollectives without a GPU: 2 and 3 ranks
as threads over one simulated unified address space, the library's peer entry
points replaced by a fake that performs each operation at once (copies,
flag stores, rank-ordered fp32 sums) and blocks a wait until the flags reach the
epoch (with a time limit). Checks the offsets each rank writes to, the
epoch / READY / DONE protocol across consecutive collectives, the direct and the
staged all-gather and the reduce-scatter sums."""
from __future__ import annotations

import ctypes as C
import threading

import numpy as np
import pytest

from oasis_b200 import _lib
from oasis_b200 import tensor_parallel as TP

BASE = 1 << 20  # simulated device addresses start here


class FakeDevice:
    """One flat byte heap standing for every rank's memory (unified addressing)."""

    def __init__(self, nbytes: int):
        self.mem = np.zeros(nbytes, dtype=np.uint8)
        self.top = 0
        self.cv = threading.Condition()
        self.log: list = []

    def alloc(self, nbytes: int) -> int:
        addr = BASE + self.top
        self.top += (nbytes + 255) // 256 * 256
        assert self.top <= self.mem.size
        return addr

    def view(self, addr: int, nbytes: int, dtype=np.uint8) -> np.ndarray:
        o = addr - BASE
        assert 0 <= o and o + nbytes <= self.mem.size, (addr, nbytes)
        return self.mem[o:o + nbytes].view(dtype)

    def call(self, name, *args):
        a = [x.value if isinstance(x, C.c_void_p) else x for x in args]
        if name == "oasis_peer_signal":
            flag, value, _ = a
            with self.cv:
                self.view(flag, 4, np.int32)[0] = value
                self.log.append(("signal", flag, value))
                self.cv.notify_all()
        elif name == "oasis_peer_wait":
            flags, n, skip, target, _, _ = a
            with self.cv:
                ok = self.cv.wait_for(
                    lambda: all(self.view(flags, 4 * n, np.int32)[i] >= target for i in range(n) if i != skip),
                    timeout=10)
            if not ok:
                raise RuntimeError(f"fake peer wait timed out (flags {self.view(flags, 4 * n, np.int32)}, {target})")
        elif name == "oasis_peer_copy":
            dst, src, nbytes, _ = a
            with self.cv:
                self.view(dst, nbytes)[:] = self.view(src, nbytes)
        elif name == "oasis_reduce_slots":
            dst, staging, stride, own, own_slot, n, count, dtype, _ = a
            assert dtype == _lib.OASIS_DTYPE_F32
            with self.cv:
                acc = np.zeros(count, np.float32)
                for k in range(n):
                    src = own if k == own_slot else staging + k * stride * 4
                    acc += self.view(src, 4 * count, np.float32)
                self.view(dst, 4 * count, np.float32)[:] = acc
        else:
            raise AssertionError(f"unexpected library call {name}")
        return 0


def _ranks(dev: FakeDevice, n: int, xn_elems: int, slot_bytes: int):
    """PeerCollectives objects as their constructor lays them out, without a GPU."""
    objs = []
    for r in range(n):
        pc = TP.PeerCollectives.__new__(TP.PeerCollectives)
        pc.n, pc.r, pc.epoch, pc.errors, pc.timeout_ns = n, r, 0, [], int(1e9)
        pc.xn_bytes = xn_elems * 2
        pc.slot_bytes = slot_bytes
        pc.stage_off = (pc.xn_bytes + 255) // 256 * 256
        pc.flag_off = pc.stage_off + n * slot_bytes
        pc.base = dev.alloc(pc.flag_off + 2 * 32 * 4)
        objs.append(pc)
    for pc in objs:
        pc.peer_base = [o.base for o in objs]
    return objs


def _run(objs, fn):
    errs = []

    def body(pc):
        try:
            fn(pc)
        except Exception as e:  # noqa: BLE001
            errs.append(e)

    ts = [threading.Thread(target=body, args=(pc,)) for pc in objs]
    for t in ts:
        t.start()
    for t in ts:
        t.join(30)
    assert not errs, errs


@pytest.mark.parametrize("n", [2, 3])
def test_peer_collectives_protocol(monkeypatch, n):
    dev = FakeDevice(8 << 20)
    monkeypatch.setattr(TP._lib, "call", dev.call)
    count = 64  # elements per rank
    objs = _ranks(dev, n, xn_elems=4 * n * count, slot_bytes=4 * count * 4)

    # direct all-gather (bf16 bytes) into chunk 1 of every rank's gathered rows
    sends = [dev.alloc(2 * count) for _ in range(n)]
    for r, a in enumerate(sends):
        dev.view(a, 2 * count, np.uint16)[:] = np.arange(count, dtype=np.uint16) + 1000 * (r + 1)
    chunk = n * count * 2  # bytes of one gathered chunk
    _run(objs, lambda pc: pc._all_gather(sends[pc.r], pc.base + chunk, count, _lib.OASIS_DTYPE_BF16, 0))
    for pc in objs:
        got = dev.view(pc.base + chunk, chunk, np.uint16).reshape(n, count)
        for r in range(n):
            assert np.array_equal(got[r], np.arange(count, dtype=np.uint16) + 1000 * (r + 1))
        assert not dev.view(pc.base, chunk, np.uint16).any()  # chunk 0 untouched

    # reduce-scatter (fp32), twice in a row (epochs 2 and 3 reuse the same flags)
    for rep in range(2):
        rs_send = [dev.alloc(4 * n * count) for _ in range(n)]
        rs_recv = [dev.alloc(4 * count) for _ in range(n)]
        for r, a in enumerate(rs_send):
            dev.view(a, 4 * n * count, np.float32)[:] = (np.arange(n * count) % 13) * (r + 1) + rep
        _run(objs, lambda pc: pc._reduce_scatter(rs_send[pc.r], rs_recv[pc.r], count, _lib.OASIS_DTYPE_F32, 0))
        for r in range(n):
            exp = sum(((np.arange(n * count) % 13) * (k + 1) + rep)[r * count:(r + 1) * count] for k in range(n))
            assert np.array_equal(dev.view(rs_recv[r], 4 * count, np.float32), exp.astype(np.float32))

    # staged all-gather (fp32) into buffers outside the shared region
    ag_send = [dev.alloc(4 * count) for _ in range(n)]
    ag_recv = [dev.alloc(4 * n * count) for _ in range(n)]
    for r, a in enumerate(ag_send):
        dev.view(a, 4 * count, np.float32)[:] = r + 0.5
    _run(objs, lambda pc: pc._all_gather(ag_send[pc.r], ag_recv[pc.r], count, _lib.OASIS_DTYPE_F32, 0))
    for r in range(n):
        got = dev.view(ag_recv[r], 4 * n * count, np.float32).reshape(n, count)
        assert np.array_equal(got, np.repeat((np.arange(n) + 0.5)[:, None], count, axis=1).astype(np.float32))

    # four collectives: every rank at epoch 4, every flag it received says 4
    for pc in objs:
        assert pc.epoch == 4
        flags = dev.view(pc.base + pc.flag_off, 2 * 32 * 4, np.int32).reshape(2, 32)
        for p in range(n):
            assert flags[0, p] == (0 if p == pc.r else 4) and flags[1, p] == (0 if p == pc.r else 4)


def test_peer_collectives_reject_oversized_staging(monkeypatch):
    dev = FakeDevice(1 << 20)
    monkeypatch.setattr(TP._lib, "call", dev.call)
    (pc,) = _ranks(dev, 1, xn_elems=64, slot_bytes=256)
    with pytest.raises(ValueError):
        pc._reduce_scatter(BASE, BASE, 1024, _lib.OASIS_DTYPE_F32, 0)  # 4 KB > 256-byte slot
    with pytest.raises(ValueError):
        pc._all_gather(BASE, BASE + (1 << 19), 1024, _lib.OASIS_DTYPE_F32, 0)  # staged and too large
