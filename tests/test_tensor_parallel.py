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
        B, T = 2, 3
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
        torch.cuda.synchronize()
        q.put((rank, rel_l2(v_tp, v_1)))
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp2_matches_single_gpu():
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
    for _, err in res:
        assert err < 5e-3, res  # bf16 operands; partial sums re-associated across ranks
