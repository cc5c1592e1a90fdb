"""n-way tensor parallelism of the DiT forward (the reference's multi-chip
strategy, oasis_inference.py:289-305, 569-626, 1153-1201, re-expressed for
B200 ranks over NCCL).

Rank r of n holds heads [16 r / n, 16 (r + 1) / n):
  QKV   column-parallel: the q, k and v rows of those heads  -> local qkv [M, 3 x 1024 / n]
  attention on the local heads (spatial and temporal attention stay rank-local)
  O     row-parallel: to_out columns of those heads -> fp32 partial [M, 1024]
  FC1   column-parallel (4096 / n hidden units), FC2 row-parallel -> fp32 partial
After each row-parallel projection the partials are summed with an NCCL
all-reduce, then one kernel adds bias, applies the adaLN gate and the residual.
LayerNorm, adaLN, the final layer and the residual stream are replicated.

The whole forward is one C-ABI call, oasis_dit_forward_tp, on the current
stream; the library calls back for each all-reduce, which here is
torch.distributed (NCCL over NVLink) ordered on the same stream.
"""
from __future__ import annotations

import ctypes as C

import torch
import torch.distributed as dist

from . import _lib
from . import host as H
from .weights import DitDeviceWeights, count_blocks

D = H.D_MODEL


def shard_rows(w: torch.Tensor, n: int, r: int) -> torch.Tensor:
    k = w.shape[0] // n
    return w[r * k:(r + 1) * k]


def shard_cols(w: torch.Tensor, n: int, r: int) -> torch.Tensor:
    k = w.shape[1] // n
    return w[:, r * k:(r + 1) * k]


def shard_qkv(w: torch.Tensor, n: int, r: int) -> torch.Tensor:
    """to_qkv.weight [3 x 1024, 1024] -> the q, k, v rows of rank r's heads."""
    return torch.cat([shard_rows(part, n, r) for part in w.split(D, dim=0)], dim=0)


class TPDitWeights:
    """Replicated parts (adaLN, final layer, embed, RoPE) + rank r's shards."""

    def __init__(self, sd: dict, n: int, r: int, device):
        if 16 % n:
            raise ValueError(f"{n}-way tensor parallelism needs n | 16")
        self.n, self.r, self.heads = n, r, 16 // n
        self.full = DitDeviceWeights(sd, device)  # replicated pieces are read from here
        dev = torch.device(device)
        self.n_blocks = count_blocks(sd)

        def bf(t):
            return t.to(dev, torch.bfloat16).contiguous()

        def f32(t):
            return t.to(dev, torch.float32).contiguous()

        self.sub = []
        for i in range(self.n_blocks):
            for s in ("s", "t"):
                p = f"blocks.{i}.{s}"
                self.sub.append(dict(
                    qkv_w=bf(shard_qkv(sd[f"{p}_attn.to_qkv.weight"], n, r)),
                    out_w=bf(shard_cols(sd[f"{p}_attn.to_out.weight"], n, r)),
                    out_b=f32(sd[f"{p}_attn.to_out.bias"]),
                    fc1_w=bf(shard_rows(sd[f"{p}_mlp.fc1.weight"], n, r)),
                    fc1_b=f32(shard_rows(sd[f"{p}_mlp.fc1.bias"], n, r)),
                    fc2_w=bf(shard_cols(sd[f"{p}_mlp.fc2.weight"], n, r)),
                    fc2_b=f32(sd[f"{p}_mlp.fc2.bias"])))
        # the OasisDitWeights of this shard: replicated pointers from `full`,
        # sub-block pointers to the shards
        st = _lib.OasisDitWeights()
        C.pointer(st)[0] = self.full.struct
        for i, blk in enumerate(self.sub):
            for k, v in blk.items():
                setattr(st.sub[i], k, v.data_ptr())
        self.struct = st


def _st() -> int:
    return torch.cuda.current_stream().cuda_stream


class TPScratch:
    """Per-rank buffers of one TP forward for B sessions x T frames: the library
    workspace and the fp32 partial the collective sums."""

    def __init__(self, tpw: TPDitWeights, batch: int, frames: int, device):
        M = batch * frames * 144
        dev = torch.device(device)
        nbytes = int(_lib.load().oasis_tp_workspace_size(batch, frames, tpw.heads))
        self.workspace = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=dev)
        self.part = torch.empty(M, D, device=dev)


def dit_forward_tp(tpw: TPDitWeights, z: torch.Tensor, cond: torch.Tensor, v_out: torch.Tensor, sc: TPScratch,
                   group=None) -> torch.Tensor:
    """TP DiT forward through oasis_dit_forward_tp: z [B, T, 144, 1024] fp32
    (replicated, overwritten), cond [B, T, 1024] -> v_out [B, 144, 64] for the
    last frame (replicated). The library calls back into torch.distributed (NCCL
    over NVLink) for the two all-reduces of every sub-block, on the current
    stream."""
    B, T = z.shape[0], z.shape[1]
    errors = []

    def _allreduce(buf, count, user, stream):
        try:
            dist.all_reduce(sc.part, group=group)
            return 0
        except Exception as e:  # reported as the call's status
            errors.append(e)
            return -2

    cb = _lib.ALLREDUCE_FN(_allreduce)
    a = _lib.OasisTpArgs(B, T, tpw.heads, z.data_ptr(), cond.data_ptr(), v_out.data_ptr(), sc.part.data_ptr(), cb,
                         None, sc.workspace.data_ptr(), sc.workspace.numel())
    try:
        _lib.call("oasis_dit_forward_tp", C.byref(tpw.struct), C.byref(a), _st())
    except _lib.OasisError:
        if errors:
            raise errors[0]
        raise
    return v_out


# --------------------------------------------------------------------------- sequence parallel
class TPSpBuffers:
    """Per-rank buffers of the sequence-parallel TP forward (oasis_dit_forward_tp_sp)
    for B sessions x T frames over `world` ranks: the library workspace and the
    caller-owned communication buffers the collectives read and write."""

    def __init__(self, tpw: TPDitWeights, batch: int, frames: int, device, partial_dtype=torch.bfloat16):
        n = tpw.n
        if batch % n:
            raise ValueError(f"{batch} sessions do not split over {n} ranks")
        if partial_dtype not in (torch.bfloat16, torch.float32):
            raise ValueError("partial_dtype must be bf16 or fp32")
        dev = torch.device(device)
        M = batch * frames * H.N_PATCHES
        Ml = M // n
        self.batch, self.frames, self.world, self.rank = batch, frames, n, tpw.r
        nbytes = int(_lib.load().oasis_tp_sp_workspace_size(batch, frames, tpw.heads, n))
        self.workspace = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=dev)
        self.partial = torch.empty(M, D, dtype=partial_dtype, device=dev)
        self.shard = torch.empty(Ml, D, dtype=partial_dtype, device=dev)
        self.xn_local = torch.empty(Ml, D, dtype=torch.bfloat16, device=dev)
        self.xn = torch.empty(M, D, dtype=torch.bfloat16, device=dev)
        self.v_local = torch.empty(batch // n, H.N_PATCHES, H.OUT_DIM, device=dev)

    def registry(self, v_out: torch.Tensor) -> dict[int, torch.Tensor]:
        """Device pointer -> tensor of every buffer a collective callback may name."""
        return {t.data_ptr(): t for t in (self.partial, self.shard, self.xn_local, self.xn, self.v_local, v_out)}


def _reduce_scatter(recv: torch.Tensor, send: torch.Tensor, group=None) -> None:
    if dist.get_backend(group) == "nccl":
        dist.reduce_scatter_tensor(recv, send, group=group)
    else:  # gloo has no reduce-scatter: all-reduce a copy, keep this rank's slice
        tmp = send.clone()
        dist.all_reduce(tmp, group=group)
        r, n = dist.get_rank(group), dist.get_world_size(group)
        recv.copy_(tmp.view(n, -1)[r].view_as(recv))


def _all_gather(recv: torch.Tensor, send: torch.Tensor, group=None) -> None:
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(recv, send, group=group)
    else:
        dist.all_gather(list(recv.view(dist.get_world_size(group), -1).unbind(0)), send.reshape(-1), group=group)


def buffer_view(registry: dict[int, torch.Tensor], ptr: int, numel: int) -> torch.Tensor:
    """The `numel` elements at device address `ptr` inside one of the registered
    buffers (the library passes chunk offsets into them), as a flat view."""
    for base, t in registry.items():
        es = t.element_size()
        if base <= ptr < base + t.numel() * es:
            off = (ptr - base) // es
            if (ptr - base) % es or off + numel > t.numel():
                raise ValueError(f"collective buffer at +{ptr - base} bytes, {numel} elements, outside its tensor")
            return t.view(-1)[off:off + numel]
    raise KeyError(f"collective buffer {ptr:#x} is not one of the registered tensors")


def dist_collectives(registry: dict[int, torch.Tensor], group=None, errors: list | None = None):
    """The two callbacks of OasisTpSpArgs over torch.distributed (NCCL on GPUs,
    gloo on the CPU): the library names buffers (or chunks of them) by pointer,
    `registry` maps them back to tensors. The collective runs with the stream the
    library passes as the current stream, so it is ordered on it. A raised
    exception becomes a non-zero status (kept in `errors`), which aborts the
    forward."""

    def wrap(fn, send_ranks, recv_ranks):
        def cb(send, recv, count, dtype, user, stream):
            try:
                n = dist.get_world_size(group)
                s = buffer_view(registry, send, count * (n if send_ranks else 1))
                r = buffer_view(registry, recv, count * (n if recv_ranks else 1))
                if stream and torch.cuda.is_available():
                    with torch.cuda.stream(torch.cuda.ExternalStream(stream)):
                        fn(r, s, group)
                else:
                    fn(r, s, group)
                return 0
            except Exception as e:  # noqa: BLE001  (reported through the C status)
                if errors is not None:
                    errors.append(e)
                return -2
        return _lib.COLLECTIVE_FN(cb)

    return wrap(_reduce_scatter, True, False), wrap(_all_gather, False, True)


class _DeviceBytes:
    """A raw device allocation seen by torch (CUDA array interface, uint8)."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 3,
                                         "strides": None}


def _device_bytes(ptr: int, nbytes: int, device) -> torch.Tensor:
    return torch.as_tensor(_DeviceBytes(ptr, nbytes), device=device)


class PeerCollectives:
    """The two collective callbacks of OasisTpSpArgs over peer memory: the bulk
    data crosses NVLink on the copy engines (one copy per peer into its buffer,
    opened through CUDA IPC) and the library's own peer kernels carry the
    handshakes and the reduce-scatter sum, so no collective kernel competes with
    the projections for SMs.

    Every rank shares one device region: the gathered LayerNorm rows (which
    replace `bufs.xn`, so peers write the all-gather straight into the
    projections' input), a staging area of `world` slots for reduce-scatter
    blocks and gathers into other buffers, and two rows of flags. Per collective,
    with the epoch e counted identically on every rank: each rank signals READY=e
    to every peer (its receive region is free: everything before the collective
    on its stream has run), waits for READY=e from every peer, copies its blocks
    into the peers' regions, signals DONE=e, waits for DONE=e from every peer,
    and (reduce-scatter) sums the world's blocks in rank order in fp32.
    Construction and `close` are collective over `group`."""

    READY, DONE = 0, 1

    def __init__(self, bufs: TPSpBuffers, group=None, timeout_s: float = 30.0):
        lib = _lib.load()
        self.lib, self.group = lib, group
        self.n, self.r = bufs.world, bufs.rank
        if dist.get_world_size(group) != self.n or dist.get_rank(group) != self.r:
            raise ValueError("PeerCollectives: the group does not match the buffers' rank / world")
        dev = bufs.xn.device
        self.timeout_ns = int(timeout_s * 1e9)
        es = bufs.partial.element_size()
        self.xn_bytes = bufs.xn.numel() * 2
        slot = max(bufs.shard.numel() * es, bufs.v_local.numel() * 4)
        self.slot_bytes = (slot + 255) // 256 * 256
        self.stage_off = (self.xn_bytes + 255) // 256 * 256
        self.flag_off = self.stage_off + self.n * self.slot_bytes
        total = self.flag_off + 2 * 32 * 4
        base = C.c_void_p()
        _lib.call("oasis_peer_alloc", total, C.byref(base))
        self.base, self.total = base.value, total
        handle = (C.c_char * _lib.OASIS_IPC_HANDLE_BYTES)()
        _lib.call("oasis_ipc_get_handle", C.c_void_p(self.base), handle)
        handles = [None] * self.n
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.peer_base = []
        for p, h in enumerate(handles):
            if p == self.r:
                self.peer_base.append(self.base)
                continue
            ptr = C.c_void_p()
            _lib.call("oasis_ipc_open_handle", C.create_string_buffer(h, len(h)), C.byref(ptr))
            self.peer_base.append(ptr.value)
        # the projections read the gathered rows from the shared region
        bufs.xn = _device_bytes(self.base, self.xn_bytes, dev).view(torch.bfloat16).view(bufs.xn.shape)
        self.bufs = bufs
        self.epoch = 0
        self.errors: list = []
        self._cbs = (_lib.COLLECTIVE_FN(self._guard(self._reduce_scatter)),
                     _lib.COLLECTIVE_FN(self._guard(self._all_gather)))
        torch.cuda.synchronize(dev)
        dist.barrier(group=group)

    @property
    def callbacks(self):
        """(reduce_scatter, all_gather) for dit_forward_tp_sp's `collectives`."""
        return self._cbs

    def _guard(self, fn):
        def cb(send, recv, count, dtype, user, stream):
            try:
                fn(send, recv, count, dtype, stream)
                return 0
            except Exception as e:  # noqa: BLE001  (reported through the C status)
                self.errors.append(e)
                return -2
        return cb

    def _flag(self, p: int, kind: int, src: int) -> int:
        return self.peer_base[p] + self.flag_off + (kind * 32 + src) * 4

    def _handshake(self, kind: int, stream) -> None:
        for p in range(self.n):
            if p != self.r:
                _lib.call("oasis_peer_signal", C.c_void_p(self._flag(p, kind, self.r)), self.epoch, stream)
        _lib.call("oasis_peer_wait", C.c_void_p(self._flag(self.r, kind, 0)), self.n, self.r, self.epoch,
                  self.timeout_ns, stream)

    def _copy(self, dst: int, src: int, nbytes: int, stream) -> None:
        _lib.call("oasis_peer_copy", C.c_void_p(dst), C.c_void_p(src), nbytes, stream)

    def _next_epoch(self) -> None:
        self.epoch = (self.epoch + 1) & 0x7FFFFFFF

    def _all_gather(self, send, recv, count, dtype, stream) -> None:
        nbytes = count * (2 if dtype == _lib.OASIS_DTYPE_BF16 else 4)
        direct = self.base <= recv and recv + self.n * nbytes <= self.base + self.xn_bytes
        if not direct and nbytes > self.slot_bytes:
            raise ValueError(f"all_gather of {nbytes} bytes per rank exceeds the staging slot ({self.slot_bytes})")
        self._next_epoch()
        self._handshake(self.READY, stream)
        for p in range(self.n):
            if p == self.r:
                self._copy(recv + self.r * nbytes, send, nbytes, stream)
            elif direct:  # the same offset in the peer's gathered rows
                self._copy(self.peer_base[p] + (recv - self.base) + self.r * nbytes, send, nbytes, stream)
            else:
                self._copy(self.peer_base[p] + self.stage_off + self.r * self.slot_bytes, send, nbytes, stream)
        self._handshake(self.DONE, stream)
        if not direct:
            for p in range(self.n):
                if p != self.r:
                    self._copy(recv + p * nbytes, self.base + self.stage_off + p * self.slot_bytes, nbytes, stream)

    def _reduce_scatter(self, send, recv, count, dtype, stream) -> None:
        nbytes = count * (2 if dtype == _lib.OASIS_DTYPE_BF16 else 4)
        if nbytes > self.slot_bytes:
            raise ValueError(f"reduce_scatter of {nbytes} bytes per rank exceeds the staging slot ({self.slot_bytes})")
        self._next_epoch()
        self._handshake(self.READY, stream)
        for p in range(self.n):
            if p != self.r:  # my partial of p's rows into p's slot r
                self._copy(self.peer_base[p] + self.stage_off + self.r * self.slot_bytes, send + p * nbytes, nbytes,
                           stream)
        self._handshake(self.DONE, stream)
        es = 2 if dtype == _lib.OASIS_DTYPE_BF16 else 4
        _lib.call("oasis_reduce_slots", C.c_void_p(recv), C.c_void_p(self.base + self.stage_off),
                  self.slot_bytes // es, C.c_void_p(send + self.r * nbytes), self.r, self.n, count, dtype, stream)

    def check(self) -> None:
        """Raises if a callback failed or a peer wait gave up (device error 16)."""
        if self.errors:
            raise self.errors[0]
        err = self.lib.oasis_device_error(1)
        if err:
            raise RuntimeError(f"peer collectives: device error {err} (16: a peer did not signal in time)")

    def close(self) -> None:
        """Collective: every rank finished with the shared region, then unmap and free."""
        if self.base is None:
            return
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        for p, ptr in enumerate(self.peer_base):
            if p != self.r:
                _lib.call("oasis_ipc_close_handle", C.c_void_p(ptr))
        dist.barrier(group=self.group)
        _lib.call("oasis_peer_free", C.c_void_p(self.base))
        self.base = None


def dit_forward_tp_sp(tpw: TPDitWeights, z_local: torch.Tensor, cond_local: torch.Tensor, v_out: torch.Tensor,
                      bufs: TPSpBuffers, collectives=None, group=None, stream=None, comm_stream=None,
                      chunks: int = 1, reserve_sms: int = 0) -> torch.Tensor:
    """Sequence-parallel TP DiT forward through oasis_dit_forward_tp_sp: this
    rank's sessions z_local [B / n, T, 144, 1024] (overwritten) and cond_local
    [B / n, T, 1024] -> v_out [B, 144, 64] for every session's last frame.
    `collectives` = (reduce_scatter, all_gather) callbacks; by default
    torch.distributed on `group`. With `comm_stream` (a torch.cuda.Stream) the
    collectives run there and each rank's sessions go in `chunks` groups, so the
    communication of one group overlaps the projections of the next;
    `reserve_sms` SMs are then kept free of the persistent kernels for the
    collectives' own kernels."""
    errors: list = []
    if collectives is None:
        collectives = dist_collectives(bufs.registry(v_out), group, errors)
    rs, ag = collectives
    dtype = _lib.OASIS_DTYPE_BF16 if bufs.partial.dtype == torch.bfloat16 else _lib.OASIS_DTYPE_F32
    a = _lib.OasisTpSpArgs(bufs.batch, bufs.frames, tpw.heads, bufs.rank, bufs.world, z_local.data_ptr(),
                           cond_local.data_ptr(), v_out.data_ptr(), dtype, bufs.partial.data_ptr(),
                           bufs.shard.data_ptr(), bufs.xn_local.data_ptr(), bufs.xn.data_ptr(),
                           bufs.v_local.data_ptr(), rs, ag, None, bufs.workspace.data_ptr(), bufs.workspace.numel(),
                           None if comm_stream is None else comm_stream.cuda_stream, chunks, reserve_sms)
    st = (stream or torch.cuda.current_stream()).cuda_stream
    try:
        _lib.call("oasis_dit_forward_tp_sp", C.byref(tpw.struct), C.byref(a), st)
    except _lib.OasisError:
        if errors:
            raise errors[0]
        raise
    return v_out
