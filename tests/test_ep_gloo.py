"""CPU, 2 gloo ranks: the token -> expert EP host logic (record layout, splits, orders,
the collectives each way, the combine order) with a reference backend standing in for
the CUDA kernels.  Each rank's EP output must match the single-device NVFP4 layer on its
own tokens to bf16 rounding of the per-rank partial sums (rel L2 <= 1e-2; typically
~1e-3), and the expert rows themselves are bit-identical."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import ffn_ref, nvfp4_ref as nv, route_ref

S, H, dh, de, E, K = 48, 2, 256, 256, 8, 3


def _row_bytes(dh_, K_):
    return dh_ // 2 + dh_ // 16 + ((16 + 8 * K_ + 15) // 16) * 16


def _sort_with_inverse(probs, idx, num_experts):
    """route.py's stable global sort, skipping negative ids; inverse map -1 for skipped."""
    Hh, Ss, Kk = idx.shape
    gidx = (idx + np.arange(Hh).reshape(Hh, 1, 1) * num_experts).reshape(-1)
    valid = idx.reshape(-1) >= 0
    flat = np.nonzero(valid)[0]
    order = flat[np.argsort(gidx[flat], kind="stable")]
    tok = np.broadcast_to(np.arange(Ss).reshape(1, Ss, 1), (Hh, Ss, Kk)).reshape(-1)
    counts = np.bincount(gidx[flat], minlength=Hh * num_experts)
    offs = np.zeros(Hh * num_experts + 1, np.int64)
    offs[1:] = np.cumsum(counts)
    inv = np.full(idx.size, -1, np.int64)
    inv[order] = np.arange(order.size)
    n = idx.size
    g = np.zeros(n, np.int32)
    ps = np.zeros(n, np.float32)
    g[:order.size] = tok[order]
    ps[:order.size] = probs.reshape(-1)[order]
    return g, ps, offs, inv.astype(np.int32)


class RefBackend:
    """numpy restatement of the device steps (test infrastructure)."""

    def quant_tokens(self, x_heads):
        x = x_heads.float().numpy().reshape(-1, x_heads.shape[-1])          # row = s*H + h
        codes, sf, g = nv.quantize_rows(x)
        return torch.from_numpy(nv.pack_codes(codes)), torch.from_numpy(sf), torch.from_numpy(g)

    def dest(self, idx, num_experts, n_ranks):
        i = idx.numpy()
        Hh, Ss, Kk = i.shape
        E_loc = Hh * num_experts // n_ranks
        ge = i + np.arange(Hh).reshape(Hh, 1, 1) * num_experts
        d = np.full((Hh * Ss, n_ranks), -1, np.int64)
        r = (ge // E_loc).reshape(Hh * Ss, Kk)
        for k in range(Kk):
            d[np.arange(Hh * Ss), r[:, k]] = r[:, k]
        return torch.from_numpy(d)

    def row_bytes(self, dh_, K_):
        return _row_bytes(dh_, K_)

    def pack(self, xq, xsf, xg, Hh, Ss, idx, probs, num_experts, n_ranks, send_key, send_offsets, R_send):
        dh_ = xq.shape[1] * 2
        Kk = idx.shape[-1]
        E_loc = Hh * num_experts // n_ranks
        rb = _row_bytes(dh_, Kk)
        out = np.zeros((R_send, rb), np.uint8)
        offs = send_offsets.numpy()
        i = idx.numpy().reshape(Hh * Ss, Kk)
        p = probs.numpy().reshape(Hh * Ss, Kk)
        for j in range(R_send):
            d = int(np.searchsorted(offs, j, side="right") - 1)
            t = int(send_key[j])
            h, s_ = divmod(t, Ss)
            q = s_ * Hh + h
            out[j, :dh_ // 2] = xq[q].numpy()
            out[j, dh_ // 2:dh_ // 2 + dh_ // 16] = xsf[q].numpy()
            meta = np.zeros((rb - dh_ // 2 - dh_ // 16) // 4, np.uint32)
            pairs = [(int(h * num_experts + i[t, k]) % E_loc, p[t, k]) for k in range(Kk)
                     if (h * num_experts + i[t, k]) // E_loc == d]
            meta[0] = np.float32(xg[q]).view(np.uint32)
            meta[1] = len(pairs)
            for k in range(Kk):
                e, pr = pairs[k] if k < len(pairs) else (-1, 0.0)
                meta[4 + 2 * k] = np.uint32(e & 0xFFFFFFFF)
                meta[5 + 2 * k] = np.float32(pr).view(np.uint32)
            out[j, dh_ // 2 + dh_ // 16:] = meta.view(np.uint8)
        return torch.from_numpy(out)

    def unpack(self, recv, dh_, Kk, E_loc):
        r = recv.numpy()
        meta = r[:, dh_ // 2 + dh_ // 16:].copy().view(np.uint32)
        c = meta[:, 1].astype(np.int64)
        e = meta[:, 4:4 + 2 * Kk:2].view(np.int32).astype(np.int64)
        pr = meta[:, 5:5 + 2 * Kk:2].view(np.float32).copy()
        e = np.where(np.arange(Kk)[None, :] < c[:, None], e, -1)
        pr = np.where(np.arange(Kk)[None, :] < c[:, None], pr, 0).astype(np.float32)
        return torch.from_numpy(e), torch.from_numpy(pr)

    def sort(self, probs, idx, num_experts):
        return tuple(torch.from_numpy(a) for a in _sort_with_inverse(probs.numpy(), idx.numpy(), num_experts))

    def ffn_records(self, recv, dh_, Kk, gather_ids, probs_sorted, expert_offsets, row_of_flat, gu, dn,
                    stage_events=None):
        r = recv.numpy()
        T = r.shape[0]
        offs = expert_offsets.numpy()
        nvalid = int(offs[-1])
        gids = gather_ids.numpy()[:nvalid].astype(np.int64)
        expert = np.repeat(np.arange(offs.size - 1), np.diff(offs))
        codes = nv.unpack_codes(r[gids, :dh_ // 2])
        sf = r[gids, dh_ // 2:dh_ // 2 + dh_ // 16]
        g = r[gids, dh_ // 2 + dh_ // 16:dh_ // 2 + dh_ // 16 + 4].copy().view(np.float32).reshape(-1)
        rows = ffn_ref.nvfp4_expert_rows_ref(codes, sf, g, expert, probs_sorted.numpy()[:nvalid], gu, dn)
        inv = row_of_flat.numpy().reshape(T, Kk)
        out = np.zeros((T, dh_), np.float32)
        for i in range(T):
            for rr in sorted(x for x in inv[i] if x >= 0):
                out[i] = out[i] + rows[rr]
        return torch.from_numpy(nv.bf16_round(out)).to(torch.bfloat16)

    def combine(self, rows, S_, H_, row_of_flat, K_):
        r = rows.float().numpy()
        inv = row_of_flat.numpy().reshape(H_ * S_, K_)
        y = np.zeros((H_ * S_, r.shape[1]), np.float32)
        for key in range(H_ * S_):
            for rr in sorted(x for x in inv[key] if x >= 0):
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
        err = ffn_ref.rel_l2(y.float().numpy(), ref)
        q.put((rank, bool(err < 1e-2), err))
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
    for rank, ok, err in res:
        assert ok, f"rank {rank}: EP output differs from the single-device layer (rel L2 {err})"


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


def _leave_worker(rank, world, port, q):
    """Both ranks run one EP step; rank 1 then leaves (exits without a further collective,
    as a crashed or departed rank does).  Rank 0's next EP step must fail with an error
    within the process group's timeout instead of waiting for ever."""
    import time
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parent.parent
    sys.path[:0] = [str(root), str(root / "magi-2-preview_b200")]
    from flash_mh_moe.ep import ep_moe_layer
    gu, dn = _weights()
    E_loc = H * E // world
    gu_l, dn_l = ffn_ref.slice_packs(gu, dn, rank * E_loc, (rank + 1) * E_loc)
    x, probs, idx = _problem(rank)
    ep_moe_layer(x, probs, idx, E, gu_l, dn_l, dist.group.WORLD, backend=RefBackend())
    if rank == 1:
        q.put((rank, "left", 0.0))
    else:
        t = time.time()
        try:
            ep_moe_layer(x, probs, idx, E, gu_l, dn_l, dist.group.WORLD, backend=RefBackend())
            q.put((rank, "no error", time.time() - t))
        except Exception as e:   # the collective reports the missing peer
            q.put((rank, "error: " + type(e).__name__, time.time() - t))
    q.close()
    q.join_thread()
    os._exit(0)


def test_ep_peer_leaves_between_steps_raises():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_leave_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict((r, (what, dt)) for r, what, dt in (q.get(timeout=240) for _ in range(world)))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    what, dt = res[0]
    assert what.startswith("error"), f"rank 0's step after rank 1 left: {what}"
    assert dt < 60, f"rank 0 took {dt:.1f} s to notice the missing rank"
