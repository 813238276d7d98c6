"""GPU, 2 ranks (needs >= 2 GPUs; skipped otherwise): the expert-parallel MoE module, with
the exchange fused into the kernels (peer memory; unchunked and as a 2-chunk pipeline) and
over NCCL, against the single-GPU
module on each rank's own tokens.  The EP layer sums each
token's experts per rank (bf16 partial sums) before the source adds the ranks, so the
outputs agree to that rounding: rel L2 <= 1e-2 (typically ~1e-3); EP runs are
run-to-run identical."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

S, H, dh, de, E, K = 512, 1, 512, 256, 16, 4


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q, transport, chunks):
    import sys
    from datetime import timedelta
    from pathlib import Path
    root = Path(__file__).resolve().parent.parent
    sys.path[:0] = [str(root), str(root / "magi-2-preview_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0",
                      MHMOE_EP_TRANSPORT=transport, MHMOE_EP_TIMEOUT_S="5", MHMOE_EP_CHUNKS=str(chunks))
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    try:
        from flash_mh_moe import _lib
        from flash_mh_moe.moe import CoreMultiHeadMoE, CoreMultiHeadMoEConfig, init_moe_params_
        cfg = CoreMultiHeadMoEConfig(hidden_size=H * dh, num_heads=H, num_experts=E, top_k=K,
                                     expert_intermediate_size=de, num_layers=1, params_dtype=torch.bfloat16,
                                     score_func="sigmoid", route_norm=True, route_scale=2.0)
        full = CoreMultiHeadMoE(cfg).to(dev)
        init_moe_params_(full, seed=5, device=dev)
        ep = CoreMultiHeadMoE(cfg, ep_group=dist.group.WORLD).to(dev)
        lo, hi = ep.expert_lo, ep.expert_lo + ep.local_flatten_num_experts
        with torch.no_grad():
            ep.gate.copy_(full.gate)
            ep.W_gate.copy_(full.W_gate[lo:hi])
            ep.W_up.copy_(full.W_up[lo:hi])
            ep.W_down.copy_(full.W_down[lo:hi])
        x = torch.randn(S, H * dh, generator=torch.Generator().manual_seed(40 + rank)).to(torch.bfloat16).to(dev)
        y_ep = ep(x)
        y_ep2 = ep(x)
        y_1 = full(x)
        torch.cuda.synchronize()
        _lib.check_device_status(dev)
        err = float((y_ep.float() - y_1.float()).norm() / y_1.float().norm())
        from flash_mh_moe.ep import LAST_STATS
        q.put((rank, err < 1e-2, bool(torch.equal(y_ep, y_ep2)), err, LAST_STATS.get("transport")))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("transport,chunks", [("peer", 1), ("peer", 2), ("copy", 1), ("copy", 2), ("nccl", 1)])
def test_ep_module_matches_single_gpu(transport, chunks):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, transport, chunks)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    res = sorted(q.get(timeout=30) for _ in range(world))
    for p in procs:
        assert p.exitcode == 0
    for rank, same, repeat, err, used in res:
        assert used == transport
        assert repeat, f"rank {rank}: EP output not deterministic"
        assert same, f"rank {rank}: EP output differs from the single-GPU module (rel L2 {err})"
