"""CPU, 2 gloo ranks: the token -> expert EP host logic (splits, orders, the three
collectives each way, the combine order) with a reference backend standing in for the
CUDA kernels.  Each rank's EP output must equal the single-device NVFP4 layer on its
own tokens bit for bit (every output row depends only on its own input row; the combine
order is the global expert order in both)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import ffn_ref, nvfp4_ref as nv, route_ref

S, H, dh, de, E, K = 48, 2, 256, 256, 8, 3


class RefBackend:
    """numpy restatement of the device steps (test infrastructure)."""

    def quant_tokens(self, x_heads):
        x = x_heads.float().numpy().reshape(-1, x_heads.shape[-1])
        codes, sf, g = nv.quantize_rows(x)
        return (torch.from_numpy(nv.pack_codes(codes)), torch.from_numpy(sf), torch.from_numpy(g))

    def pack(self, xq, xsf, xg, H_, E_, E_loc, gather_ids, probs_sorted, expert_offsets):
        offs = expert_offsets.numpy()
        counts = np.diff(offs)
        expert = np.repeat(np.arange(offs.size - 1), counts)
        t = gather_ids.numpy().astype(np.int64) * H_ + expert // E_
        meta = np.zeros((t.size, 4), np.float32)
        meta[:, 0] = xg.numpy()[t]
        meta[:, 1] = (expert % E_loc).astype(np.int32).view(np.float32)
        meta[:, 2] = probs_sorted.numpy()
        return xq[t].clone(), xsf[t].clone(), torch.from_numpy(meta)

    def unpack(self, meta, E_loc):
        m = meta.numpy()
        return (torch.from_numpy(m[:, 0].copy()), torch.from_numpy(m[:, 1].copy().view(np.int32).astype(np.int64)),
                torch.from_numpy(m[:, 2].copy()))

    def sort(self, probs, idx, num_experts):
        p, i = probs.numpy(), idx.numpy()
        g, ps, o = route_ref.flash_mh_moe_global_sort(p, i, num_experts)
        Hh = i.shape[0]
        gidx = (i + np.arange(Hh).reshape(Hh, 1, 1) * num_experts).reshape(-1)
        order = np.argsort(gidx, kind="stable")
        inv = np.empty_like(order)
        inv[order] = np.arange(order.size)
        return (torch.from_numpy(g), torch.from_numpy(ps), torch.from_numpy(o), torch.from_numpy(inv.astype(np.int32)))

    def ffn_rows(self, xq, xsf, xg, gather_ids, probs_sorted, expert_offsets, row_of_flat, gu, dn):
        # rows in sorted order -> outputs in input-row order
        gids = gather_ids.numpy().astype(np.int64)
        offs = expert_offsets.numpy()
        expert = np.repeat(np.arange(offs.size - 1), np.diff(offs))
        codes = nv.unpack_codes(xq.numpy()[gids])
        rows = ffn_ref.nvfp4_expert_rows_ref(codes, xsf.numpy()[gids], xg.numpy()[gids], expert,
                                             probs_sorted.numpy(), gu, dn)
        out = np.zeros((xq.shape[0], rows.shape[1]), np.float32)
        out[gids] = rows
        return torch.from_numpy(out).to(torch.bfloat16)

    def combine(self, rows, S_, H_, row_of_flat, K_):
        r = rows.float().numpy()
        inv = row_of_flat.numpy().reshape(H_ * S_, K_)
        y = np.zeros((H_ * S_, r.shape[1]), np.float32)
        for key in range(H_ * S_):
            for rr in sorted(inv[key]):
                y[key] = y[key] + r[rr]
        y = nv.bf16_round(y).reshape(H_, S_, -1).transpose(1, 0, 2)
        return torch.from_numpy(np.ascontiguousarray(y)).to(torch.bfloat16)


def _problem(rank):
    g = torch.Generator().manual_seed(100 + rank)
    x = torch.randn(S, H, dh, generator=g).to(torch.bfloat16)
    logits = torch.randn(H, S, E, generator=g).numpy()
    probs, idx = route_ref.compute_topk_probs_and_indices(logits, K)
    return x, torch.from_numpy(probs), torch.from_numpy(idx)


def _weights():
    g = torch.Generator().manual_seed(7)
    Wg = (torch.randn(H * E, dh, de, generator=g) * 0.03).to(torch.bfloat16).float().numpy()
    Wu = (torch.randn(H * E, dh, de, generator=g) * 0.03).to(torch.bfloat16).float().numpy()
    Wd = (torch.randn(H * E, de, dh, generator=g) * 0.03).to(torch.bfloat16).float().numpy()
    return nv.pack_gate_up(Wg, Wu), nv.pack_down(Wd)


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import sys
        from pathlib import Path
        root = Path(__file__).resolve().parent.parent
        sys.path[:0] = [str(root), str(root / "magi-2-preview_b200")]
        from flash_mh_moe.ep import ep_moe_layer
        gu, dn = _weights()
        E_loc = H * E // world
        gu_l, dn_l = ffn_ref.slice_packs(gu, dn, rank * E_loc, (rank + 1) * E_loc)
        x, probs, idx = _problem(rank)
        y = ep_moe_layer(x, probs, idx, E, gu_l, dn_l, dist.group.WORLD, backend=RefBackend())
        gg, ps, o = route_ref.flash_mh_moe_global_sort(probs.numpy(), idx.numpy(), E)
        ref = ffn_ref.mh_moe_fwd_nvfp4_ref(x.float().numpy(), gg, ps, o, gu, dn)
        q.put((rank, bool(np.array_equal(y.float().numpy(), ref)), float(np.abs(y.float().numpy() - ref).max())))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_ep_token_to_expert_matches_single_device():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    res = sorted(q.get(timeout=10) for _ in range(world))
    for p in procs:
        assert p.exitcode == 0
    for rank, same, err in res:
        assert same, f"rank {rank}: EP output differs from the single-device layer (max abs {err})"


def test_head_sharded_dispatch_roundtrip_gloo():
    """Reference-compatible head-sharded ep_dispatch / ep_undispatch round trip (gloo)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_roundtrip_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    res = [q.get(timeout=10) for _ in range(2)]
    assert all(ok for _, ok in res)


def _roundtrip_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import sys
        from pathlib import Path
        root = Path(__file__).resolve().parent.parent
        sys.path[:0] = [str(root), str(root / "magi-2-preview_b200")]
        from flash_mh_moe.ep import ep_dispatch, ep_undispatch
        x = torch.randn(6, 4, 8, generator=torch.Generator().manual_seed(rank))
        y = ep_undispatch(ep_dispatch(x, dist.group.WORLD), dist.group.WORLD)
        q.put((rank, bool(torch.equal(x, y))))
    finally:
        dist.destroy_process_group()
