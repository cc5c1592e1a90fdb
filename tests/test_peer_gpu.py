"""The peer-memory collective primitives on one GPU (peer.cu): the handshake
kernels on local flags, the bounded wait giving up on a flag nothing sets, the
rank-ordered reduce of staging slots and the copy entry point. The two-rank
collectives built on them are checked on 2 GPUs in test_tensor_parallel.py."""
from __future__ import annotations

import ctypes as C

import pytest
import torch

from oasis_b200 import _lib

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def _st() -> int:
    return torch.cuda.current_stream().cuda_stream


def test_signal_then_wait_passes_and_leaves_no_error():
    _lib.load().oasis_device_error(1)
    flags = torch.zeros(32, dtype=torch.int32, device=DEV)
    for rank in range(1, 4):  # flags of ranks 1..3 of 4; this rank (0) is skipped
        _lib.call("oasis_peer_signal", C.c_void_p(flags[rank:].data_ptr()), 7, _st())
    _lib.call("oasis_peer_wait", C.c_void_p(flags.data_ptr()), 4, 0, 7, int(2e9), _st())
    torch.cuda.synchronize()
    assert flags[:4].tolist() == [0, 7, 7, 7]
    assert _lib.load().oasis_device_error(1) == 0


def test_wait_times_out_on_a_flag_nothing_sets():
    """A bounded wait: the flag never reaches the epoch, the kernel gives up
    after its limit, records device error 16 and the context stays usable."""
    _lib.load().oasis_device_error(1)
    flags = torch.zeros(2, dtype=torch.int32, device=DEV)
    _lib.call("oasis_peer_wait", C.c_void_p(flags.data_ptr()), 2, 0, 1, int(2e6), _st())  # 2 ms
    torch.cuda.synchronize()
    assert _lib.load().oasis_device_error(1) == 16
    x = torch.ones(4, device=DEV) * 3  # the context still runs work
    assert x.sum().item() == 12.0
    assert _lib.load().oasis_device_error(0) == 0


@pytest.mark.parametrize("dtype,code", [(torch.float32, _lib.OASIS_DTYPE_F32), (torch.bfloat16, _lib.OASIS_DTYPE_BF16)])
@pytest.mark.parametrize("n,own", [(2, 0), (2, 1), (4, 2), (8, 7)])
def test_reduce_slots_sums_in_rank_order(dtype, code, n, own):
    count, stride = 4096 + 8, 4096 + 64
    g = torch.Generator(device="cpu").manual_seed(n * 10 + own)
    staging = torch.randn(n, stride, generator=g).to(DEV, dtype)
    mine = torch.randn(count, generator=g).to(DEV, dtype)
    dst = torch.empty(count, device=DEV, dtype=dtype)
    _lib.call("oasis_reduce_slots", C.c_void_p(dst.data_ptr()), C.c_void_p(staging.data_ptr()), stride,
              C.c_void_p(mine.data_ptr()), own, n, count, code, _st())
    torch.cuda.synchronize()
    acc = torch.zeros(count, device=DEV)
    for k in range(n):  # fp32, rank order, rounded once
        acc += (mine if k == own else staging[k, :count]).float()
    assert torch.equal(dst, acc.to(dtype))


def test_reduce_slots_rejects_bad_arguments():
    t = torch.zeros(64, device=DEV)
    with pytest.raises(_lib.OasisError):
        _lib.call("oasis_reduce_slots", C.c_void_p(t.data_ptr()), C.c_void_p(t.data_ptr()), 8,
                  C.c_void_p(t.data_ptr()), 0, 2, 12, _lib.OASIS_DTYPE_F32, _st())  # count not a multiple of 8
    with pytest.raises(_lib.OasisError):
        _lib.call("oasis_peer_wait", C.c_void_p(t.data_ptr()), 33, 0, 1, 1000, _st())  # more than 32 flags


def test_peer_alloc_copy_and_ipc_handle():
    ptr = C.c_void_p()
    _lib.call("oasis_peer_alloc", 1 << 20, C.byref(ptr))
    try:
        handle = (C.c_char * _lib.OASIS_IPC_HANDLE_BYTES)()
        _lib.call("oasis_ipc_get_handle", ptr, handle)
        assert any(bytes(handle))
        src = torch.arange(1 << 18, device=DEV, dtype=torch.float32)
        _lib.call("oasis_peer_copy", ptr, C.c_void_p(src.data_ptr()), src.numel() * 4, _st())
        back = torch.empty_like(src)
        _lib.call("oasis_peer_copy", C.c_void_p(back.data_ptr()), ptr, src.numel() * 4, _st())
        torch.cuda.synchronize()
        assert torch.equal(back, src)
    finally:
        _lib.call("oasis_peer_free", ptr)
