#!/usr/bin/env python
"""bench.py — MAGI-2 routed MoE layer (NVFP4) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one forward of the MoE layer (router logits -> top-k -> global sort ->
NVFP4 expert FFN -> combine) over the BASELINE config-1 batch: S=16384 tokens,
d=3072 (H=1), E=128 experts, top-8 softmax routing, SwiGLU7 expert FFN dim 1024.
Synthetic seeded data with the config's distributions (x ~ N(0,1) bf16, router
weight ~ N(0,0.02) bf16-valued fp32, expert weights ~ N(0,0.02) cast to bf16, then
packed to NVFP4 at load).  Inputs are larger than L2 (0.68 GB of NVFP4 weights and
0.1 GB of x are streamed every step), so no explicit flush is needed.

Rank 0 prints one JSON line.  Under torchrun (N>1) the job is BASELINE config 3: the
expert-parallel layer with E=128 experts sharded contiguously over the N GPUs (128/N
each), 8192 tokens per GPU (weak scaling): NVFP4 token records stored straight into the
expert ranks' buffers over NVLink and per-record sums stored back by the receivers'
combine kernel, as a token-chunk pipeline (flash_mh_moe/ep.py; MHMOE_EP_TRANSPORT=nccl
selects the NCCL all-to-all variant).

--no-extras skips the extra timings the 1-GPU line also reports (the other scatter
mode and the 8192-token shape), e.g. for a launch-list capture of the headline step.

`--config prod` runs MAGI-2's production head split instead (12 heads of 256, 256 experts per
head, top-6 sigmoid x4.9, expert FFN dim 1280); `--config 2` the Zipf-skewed routing; `--config
4` the 4-layer 256-token stack (HBM-bound; GB/s).

The line's `roofline` is the gate/up GEMM against 4 x the measured bf16 burst peak
(MEASURED_PEAKS.json; dense FP4 = 4 x bf16) and, in `library_fp4_ceiling`, against a library
NVFP4 GEMM (cuBLASLt through torch._scaled_mm) of the same dense-equivalent shape timed in
the same run.

`cpu_baseline` and `--impl reference` time the reference's own layer path on the host cores
(torch, every host thread): its route.py top-k and global sort and its _scatter_back, run
unchanged from the copy staged under oracle/_ref (oracle/stage_ref.py), around its Triton
expert kernel restated in torch (oracle/ffn_torch_ref.py: bf16 operands, fp32 accumulation),
on the first 4096 tokens of the config-1 batch; on rank 0 only.  The reference arm also tries
the reference's Triton kernel on the GPU at the shapes it is written for and reports what
Triton answers (`triton_reference_gpu`).

`value` is the whole job's tokens/s (all ranks); `tokens_per_s_per_gpu` divides it by N.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
PKG = ROOT / "magi-2-preview_b200"
for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)

CFG1 = dict(name="config1", S=16384, d=3072, H=1, E=128, K=8, de=1024, seed=1, score_func="softmax")
CFG2 = dict(name="config2", S=16384, d=3072, H=1, E=128, K=8, de=1024, seed=2, score_func="softmax", zipf=True)
CFG3 = dict(name="config3", S=8192, d=3072, H=1, E=128, K=8, de=1024, seed=3, score_func="softmax")
CFG4 = dict(name="config4", S=256, d=3072, H=1, E=128, K=8, de=1024, seed=4, score_func="softmax", layers=4)
# MAGI-2's production head split (configs/magi2_preview.json:40-88): 12 heads of 256, 256
# experts per head, top-6 sigmoid, route_scale 4.9, expert FFN dim 1280.
CFGP = dict(name="prod_head_split", S=16384, d=3072, H=12, E=256, K=6, de=1280, seed=5, score_func="sigmoid",
            route_scale=4.9)
CONFIGS = {"1": CFG1, "2": CFG2, "4": CFG4, "prod": CFGP}
METRIC = "MoE-layer tokens/s/GPU; NVFP4 tensor-pipe util %; 1/2/4/8 B200 scaling"
# libmhmoe kernels per step.  1 GPU: fused router, sort x4, tile tables, pad map, fused token
# quantise + row grouping, gate/up GEMM, down GEMM, combine (atomic scatter: output zeroing
# instead).  EP (records arrive quantised): router,
# token quantise, destination mask, send sort x4, pack, unpack, receiver sort x4, tile tables,
# pad map, row grouping, gate/up GEMM, down GEMM, per-record combine, source-side combine.
KERNELS_PER_STEP = 11
KERNELS_PER_STEP_EP = 20
CPU_SAMPLE_TOKENS = 4096


def load_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class ClockSampler:
    """SM clocks and throttle reasons while the timed steps run.

    An NVML polling thread (every 5 ms: the timed region lasts tens of milliseconds) records
    (host time, SM clock, clocks-event reasons); the caller marks the timed region with
    window(start, end) in host time (perf_counter, the timed launches issued after `start`
    and synchronised before `end`) and summary() reports the samples inside it.  nvidia-smi
    sampling (200 ms, the profiling recipe's clocks line) runs beside it as the fallback when
    NVML is unavailable.  Only reads: no clock or other GPU setting is changed."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    PERIOD_S = 0.005
    REASONS = (("hw_slowdown", "HwSlowdown", 0x8), ("hw_thermal_slowdown", "HwThermalSlowdown", 0x40),
               ("sw_thermal_slowdown", "SwThermalSlowdown", 0x20), ("sw_power_cap", "SwPowerCap", 0x4))

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.path = Path(tempfile.mkstemp(prefix="clk", suffix=".csv")[1])
        self.nv: list[tuple[float, float, int]] = []
        self.nv_max = None
        self.win = None
        self._nvml = None
        self._stop = threading.Event()
        self._thread = None
        self.smi_id = str(gpu_index)

    def window(self, t_start: float, t_end: float) -> None:
        self.win = (t_start, t_end)

    def _gpu_uuid(self):
        """"GPU-<uuid>" of CUDA device idx (NVML and nvidia-smi number GPUs in the driver's
        order, not CUDA_VISIBLE_DEVICES's), or None."""
        try:
            import torch
            if not torch.cuda.is_available():
                return None
            u = str(torch.cuda.get_device_properties(self.idx).uuid)
            return u if u.startswith("GPU-") else "GPU-" + u
        except Exception:
            return None

    def _start_nvml(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            h = None
            uuid = self._gpu_uuid()
            if uuid and hasattr(pynvml, "nvmlDeviceGetHandleByUUID"):
                try:
                    h = pynvml.nvmlDeviceGetHandleByUUID(uuid)
                    self.smi_id = uuid             # validated: nvidia-smi can use it too
                except Exception:
                    h = None
            if h is None:
                h = pynvml.nvmlDeviceGetHandleByIndex(self.idx)
            self.nv_max = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
            reasons = (getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None)
                       or pynvml.nvmlDeviceGetCurrentClocksThrottleReasons)
        except Exception:
            return
        self._nvml = pynvml

        def poll():
            while not self._stop.is_set():
                try:
                    t = time.perf_counter()
                    self.nv.append((t, float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)), int(reasons(h))))
                except Exception:
                    return
                self._stop.wait(self.PERIOD_S)

        self._thread = threading.Thread(target=poll, daemon=True)
        self._thread.start()

    def __enter__(self):
        self._start_nvml()
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", self.smi_id], stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2)
        if self._nvml is not None:
            try:
                self._nvml.nvmlShutdown()
            except Exception:
                pass
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.f.close()

    def _summary_nvml(self):
        inside = [x for x in self.nv if self.win and self.win[0] <= x[0] <= self.win[1]]
        use = inside or self.nv
        bits = 0
        for x in use:
            bits |= x[2]
        reasons = []
        for name, const, default in self.REASONS:
            mask = getattr(self._nvml, "nvmlClocksEventReason" + const,
                           getattr(self._nvml, "nvmlClocksThrottleReason" + const, default))
            if bits & int(mask):
                reasons.append(name)
        return {"sm_mhz": statistics.median(x[1] for x in use), "sm_max_mhz": self.nv_max, "reasons": reasons,
                "samples": len(use), "source": "nvml, " + ("inside the timed region" if inside else
                                                            "around the timed region")}

    def summary(self) -> dict:
        if self.nv:
            return self._summary_nvml()
        rows = []
        try:
            for ln in self.path.read_text().splitlines():
                parts = [x.strip() for x in ln.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        except OSError:
            pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(rows), "source": "nvidia-smi, around the timed region"}


def torch_device(world):
    import torch
    return torch.device("cuda", torch.cuda.current_device())


def dist_setup():
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        from datetime import timedelta
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def make_layer(cfg, device, rank, ep_group=None):
    import torch
    from flash_mh_moe.moe import CoreMultiHeadMoE, CoreMultiHeadMoEConfig, init_moe_params_
    mc = CoreMultiHeadMoEConfig(hidden_size=cfg["d"], num_heads=cfg["H"], num_experts=cfg["E"], top_k=cfg["K"],
                                expert_intermediate_size=cfg["de"], num_layers=1, params_dtype=torch.bfloat16,
                                score_func=cfg["score_func"], route_norm=True,
                                route_scale=cfg.get("route_scale", 1.0))
    if ep_group is None:
        m = CoreMultiHeadMoE(mc).to(device)
        init_moe_params_(m, seed=cfg["seed"], device=device)
    else:
        # every rank draws the same full weight set, keeps its contiguous expert slice
        full = CoreMultiHeadMoE(mc).to(device)
        init_moe_params_(full, seed=cfg["seed"], device=device)
        m = CoreMultiHeadMoE(mc, ep_group=ep_group).to(device)
        lo, hi = m.expert_lo, m.expert_lo + m.local_flatten_num_experts
        with torch.no_grad():
            m.gate.copy_(full.gate)
            m.W_gate.copy_(full.W_gate[lo:hi])
            m.W_up.copy_(full.W_up[lo:hi])
            m.W_down.copy_(full.W_down[lo:hi])
        del full
        torch.cuda.empty_cache()
    g = torch.Generator().manual_seed(cfg["seed"] * 1000 + rank)
    x_host = torch.randn(cfg["S"], cfg["d"], generator=g).to(torch.bfloat16)
    return m, x_host


def step_explicit(m, x, ev, deterministic=None):
    """The module forward spelled out, with events between the stages (same kernels)."""
    from flash_mh_moe.fwd import ffn_nvfp4
    from flash_mh_moe.route import flash_mh_moe_global_sort_with_inverse, route_fused
    x_heads = x.view(-1, m.num_heads, m.d_head)
    ev[0].record()
    if getattr(m, "_logit_bias", None) is not None:
        planes, nsplit = m.router_planes()
        probs, idx = route_fused(x_heads, planes, nsplit, m.num_experts, m.topk, m.config.score_func,
                                 logit_bias=m._logit_bias)
    else:
        probs, idx = m._route(x_heads)
    ev[1].record()
    gids, ps, offs, inv = flash_mh_moe_global_sort_with_inverse(probs, idx, m.num_experts)
    gu, dn = m.packed_weights()
    return ffn_nvfp4(x_heads, gids, ps, offs, gu, dn, tok_rows=inv, k_fixed=m.topk, stage_events=ev[2:7],
                     deterministic=deterministic)


def step_ep(m, x, ev):
    """The expert-parallel module forward spelled out, with events between the stages."""
    from flash_mh_moe.ep import ep_chunks, ep_moe_layer, ep_moe_layer_peer_pipelined, ep_transport
    x_heads = x.view(-1, m.num_heads, m.d_head)
    ev[0].record()
    probs, idx = m._route(x_heads)
    ev[1].record()
    gu, dn = m.packed_weights()
    if ep_transport(m) == "copy":
        from flash_mh_moe.ep import ep_moe_layer_copy
        y = ep_moe_layer_copy(x_heads, probs, idx, m.num_experts, gu, dn, m.ep_group, chunks=ep_chunks(2),
                              stage_events=ev[2:7], comm_events=ev[8:12])
    elif ep_transport(m) == "peer":
        y = ep_moe_layer_peer_pipelined(x_heads, probs, idx, m.num_experts, gu, dn, m.ep_group, chunks=ep_chunks(),
                                        stage_events=ev[2:7], comm_events=ev[8:12])
    else:
        y = ep_moe_layer(x_heads, probs, idx, m.num_experts, gu, dn, m.ep_group, stage_events=ev[2:7],
                         comm_events=ev[8:12])
    ev[7].record()
    return y


def run_ours(args, world, rank, local):
    import torch
    import torch.distributed as dist
    from flash_mh_moe import _lib
    cfg = CONFIGS[args.config] if world == 1 else CFG3
    if args.tokens:
        cfg = dict(cfg, S=args.tokens)
    dev = torch.device("cuda", local if world > 1 else 0)
    if cfg.get("layers", 1) > 1:
        return run_stack(args, cfg, dev)
    m, x_host = make_layer(cfg, dev, rank, ep_group=dist.group.WORLD if world > 1 else None)
    if cfg.get("zipf"):
        # config 2: per-expert logit bias b_e = 2 * ln((e+1)^-1.2) -> a few crowded, many empty experts
        e = torch.arange(cfg["E"], dtype=torch.float32, device=dev)
        m._logit_bias = (2.0 * torch.log((e + 1.0) ** -1.2)).repeat(cfg["H"])
    x = x_host.to(dev)
    m.packed_weights()
    if args.release_master:
        m.release_master_weights()
        torch.cuda.empty_cache()
    torch.cuda.synchronize()

    nev = 7 if world == 1 else 12
    step = step_explicit if world == 1 else step_ep
    for _ in range(args.warmup):
        step(m, x, [torch.cuda.Event(enable_timing=True) for _ in range(nev)])
    torch.cuda.synchronize()
    _lib.check_device_status(dev)
    if world > 1:
        dist.barrier()

    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(nev)] for _ in range(args.steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(torch.cuda.current_device() if world == 1 else local) as clk:
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        h0 = time.perf_counter()
        t0.record()
        for k in range(args.steps):
            step(m, x, evs[k])
        t1.record()
        torch.cuda.synchronize()
        clk.window(h0, time.perf_counter())
    if world > 1:
        dist.barrier()
    _lib.check_device_status(dev)
    ms_total = t0.elapsed_time(t1)
    if world > 1:
        t = torch.tensor([ms_total], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_total = float(t.item())
    ms_step = ms_total / args.steps

    def avg(i, j):
        return sum(e[i].elapsed_time(e[j]) for e in evs) / len(evs)

    if world == 1:
        stages = {"route_ms": avg(0, 1), "sort_ms": avg(1, 2), "quant_tables_ms": avg(2, 3),
                  "gemm_gate_up_ms": avg(3, 4), "gemm_down_ms": avg(4, 5), "combine_ms": avg(5, 6)}
    else:
        stages = {"route_ms": avg(0, 1), "dispatch_ms": avg(1, 2), "quant_tables_ms": avg(2, 3),
                  "gemm_gate_up_ms": avg(3, 4), "gemm_down_ms": avg(4, 5), "local_combine_ms": avg(5, 6),
                  "return_combine_ms": avg(6, 7), "a2a_records_ms": avg(8, 9), "a2a_return_ms": avg(10, 11)}

    if world > 1:
        # one untimed extra step that also counts the remote bytes of chunk 0 (peer transport)
        import flash_mh_moe.ep as epmod
        epmod.COLLECT_STATS = True
        step(m, x, [torch.cuda.Event(enable_timing=True) for _ in range(nev)])
        torch.cuda.synchronize()
        epmod.COLLECT_STATS = False

    # end-to-end through the public module API, host buffers, copies inside the timed region
    e2e_ms = (float("nan"), float("nan"))
    if not args.no_e2e:
        e2e_ms = _e2e(args, m, x_host, dev, world)
    out = _report(args, cfg, world, ms_step, stages, e2e_ms, clk, m, x_host)
    if world == 1:
        from flash_mh_moe.fwd import _is_deterministic
        det = _is_deterministic()
        out["config"]["scatter"] = ("combine (deterministic: partial rows + fp32 combine; the default)" if det else
                                    "atomic (MHMOE_SCATTER=atomic: bf16 atomics from the down GEMM, the "
                                    "reference's default scatter)")
        if not args.tokens and not args.no_extras and cfg.get("layers", 1) == 1:
            ms_other = _time_explicit(args, m, x, cfg["S"], deterministic=not det)
            out["other_scatter"] = {"scatter": "atomic" if det else "combine",
                                    "value": round(cfg["S"] / (ms_other * 1e-3), 1), "unit": "tokens/s",
                                    "ms_per_step": round(ms_other, 4)}
        if not args.tokens and not args.no_extras and cfg.get("layers", 1) == 1 and not cfg.get("zipf"):
            # the same layer forward replayed as one CUDA graph (no per-kernel host launches)
            from flash_mh_moe.graph import CapturedForward
            xs = x.contiguous()
            g = CapturedForward(m, xs, warmup=args.warmup)
            for _ in range(args.warmup):
                g(xs)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            e0.record()
            for _ in range(args.steps):
                g(xs)
            e1.record()
            torch.cuda.synchronize()
            msg = e0.elapsed_time(e1) / args.steps
            out["graph_replay"] = {"value": round(cfg["S"] / (msg * 1e-3), 1), "unit": "tokens/s",
                                   "ms_per_step": round(msg, 4),
                                   "note": "module forward captured once (flash_mh_moe.graph.CapturedForward)"}
            del g
        if args.config == "1" and not args.tokens and not args.no_extras:
            S3 = CFG3["S"]
            ms3 = _time_explicit(args, m, x, S3, deterministic=det)
            out["weak_scaling_base"] = {
                "workload": f"config3 per-GPU shape on 1 GPU: {S3} tokens, E=128 local, same scatter as the "
                            "headline",
                "value": round(S3 / (ms3 * 1e-3), 1), "unit": "tokens/s", "ms_per_step": round(ms3, 4)}
    return out


def _time_explicit(args, m, x, S, deterministic):
    """Device time per step of the 1-GPU layer on the first S tokens of x."""
    import torch
    xs = x[:S].contiguous()
    for _ in range(args.warmup):
        step_explicit(m, xs, [torch.cuda.Event(enable_timing=True) for _ in range(7)], deterministic)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(7)] for _ in range(args.steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    t0.record()
    for k in range(args.steps):
        step_explicit(m, xs, evs[k], deterministic)
    t1.record()
    torch.cuda.synchronize()
    return t0.elapsed_time(t1) / args.steps


def _e2e(args, m, x_host, dev, world):
    """End to end through the module forward with host buffers: every step copies its input
    from pinned host memory and its output back.  Returns (overlapped_ms, serial_ms) per
    step: overlapped = the copies on their own streams, double-buffered, so the input copy
    of step k+1 and the output copy of step k-1 run while step k computes (how a serving
    loop feeds the layer); serial = copy in, compute, copy out on one stream."""
    import torch
    import torch.distributed as dist
    from flash_mh_moe.host import near_gpu, pinned_like
    comp = torch.cuda.current_stream(dev)
    # pinned buffers on the GPU's NUMA node, as a serving loop would hold them
    xh = [pinned_like(x_host, dev, copy=True), pinned_like(x_host.clone(), dev, copy=True)]
    yh = [pinned_like(x_host, dev) for _ in range(2)]
    xd = [torch.empty_like(x_host, device=dev) for _ in range(2)]
    s_in, s_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_used = [torch.cuda.Event() for _ in range(2)]
    ev_y = [torch.cuda.Event() for _ in range(2)]

    def overlapped(n):
        for k in range(n):
            b = k & 1
            s_in.wait_event(ev_used[b])            # the step that last read xd[b] is done
            with torch.cuda.stream(s_in):
                xd[b].copy_(xh[b], non_blocking=True)
            ev_in[b].record(s_in)
            comp.wait_event(ev_in[b])
            y = m(xd[b])
            ev_used[b].record(comp)
            ev_y[b].record(comp)
            s_out.wait_event(ev_y[b])
            with torch.cuda.stream(s_out):
                yh[b].copy_(y, non_blocking=True)
            y.record_stream(s_out)
        comp.wait_stream(s_out)

    def serial(n):
        for _ in range(n):
            x = xh[0].to(dev, non_blocking=True)
            yh[0].copy_(m(x), non_blocking=True)

    out = []
    for fn in (overlapped, serial):
        with near_gpu(dev):
            # each step allocates its output, which the copy stream holds until the copy is done:
            # warm up until the caching allocator has grown to its steady state (no device
            # allocation inside the timed steps)
            fn(max(12, args.warmup))
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(comp)
            fn(args.steps)
            e1.record(comp)
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / args.steps
            if world > 1:
                t = torch.tensor([ms], device=dev)
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                ms = float(t.item())
            out.append(ms)
    return out[0], out[1]


def _workload(cfg, world):
    H = cfg["H"]
    head = f"d={cfg['d']} (H=1)" if H == 1 else f"d={cfg['d']} as H={H} heads of {cfg['d'] // H}"
    exp = f"E={cfg['E']}" + ("" if H == 1 else " per head")
    rs = cfg.get("route_scale", 1.0)
    route = f"top-{cfg['K']} {cfg['score_func']}" + (f" x{rs}" if rs != 1.0 else "")
    if world > 1:
        return (f"config3: {cfg['S']} tokens/GPU, {head}, {exp} sharded {cfg['E'] * H // world}/GPU, {route}, "
                f"SwiGLU7 de={cfg['de']}")
    return (f"{cfg['name']}: S={cfg['S']} tokens, {head}, {exp}, {route}, SwiGLU7 de={cfg['de']}"
            + (", Zipf logit bias 2*ln((e+1)^-1.2)" if cfg.get("zipf") else ""))


def fp4_library_ceiling(dev, M, N, K, iters=10):
    """The measured FP4 ceiling: a library NVFP4 GEMM (cuBLASLt through torch._scaled_mm:
    E2M1 operands, E4M3 scales per 16 along K) of the gate/up GEMM's dense-equivalent shape
    M x N x K, median of `iters` launches after warm-up, in TFLOP/s; None when the library
    call is unavailable."""
    import torch
    try:
        g = torch.Generator(device=dev).manual_seed(0)
        a = torch.randint(0, 256, (M, K // 2), dtype=torch.uint8, device=dev, generator=g).view(torch.float4_e2m1fn_x2)
        b = torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, device=dev, generator=g).view(torch.float4_e2m1fn_x2)
        rup = lambda v, m: (v + m - 1) // m * m
        sa = torch.full((rup(M, 128) * rup(K // 16, 4),), 1.0, device=dev).to(torch.float8_e4m3fn)
        sb = torch.full((rup(N, 128) * rup(K // 16, 4),), 1.0, device=dev).to(torch.float8_e4m3fn)
        for _ in range(3):
            torch._scaled_mm(a, b.t(), sa, sb, out_dtype=torch.bfloat16)
        ts = []
        for _ in range(iters):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            torch._scaled_mm(a, b.t(), sa, sb, out_dtype=torch.bfloat16)
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1))
        ms_burst = statistics.median(ts)
        # back to back, as the layer's GEMMs run inside its timed loop (clocks under load)
        loop = 4 * iters
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(loop):
            torch._scaled_mm(a, b.t(), sa, sb, out_dtype=torch.bfloat16)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / loop
        del a, b, sa, sb
        torch.cuda.empty_cache()
        fl = 2.0 * M * N * K
        return {"tflops": round(fl / (ms * 1e-3) / 1e12, 1), "ms": round(ms, 4),
                "tflops_burst": round(fl / (ms_burst * 1e-3) / 1e12, 1), "ms_burst": round(ms_burst, 4),
                "shape_mnk": [M, N, K],
                "what": "cuBLASLt NVFP4 dense GEMM (torch._scaled_mm, e2m1 x e4m3/16 -> bf16) in this run: "
                        f"{loop} launches back to back (tflops; the comparison for a kernel timed inside the "
                        f"layer's loop) and the median of {iters} launches each followed by a synchronize "
                        "(tflops_burst)"}
    except Exception as e:  # pragma: no cover - depends on the installed torch / cuBLASLt
        return {"tflops": None, "unavailable": repr(e)[:200]}


def _report(args, cfg, world, ms_step, stages, e2e_ms, clk, m, x_host):
    S, d, de, K, H = cfg["S"], cfg["d"], cfg["de"], cfg["K"], cfg["H"]
    dh = d // H
    R = S * K * H
    if world > 1:
        from flash_mh_moe.ep import LAST_STATS
        R_gemm = int(LAST_STATS["rows_received"].item()) if "rows_received" in LAST_STATS else R  # expert-GEMM rows
    else:
        R_gemm = R
    flop_gate_up = 2.0 * R_gemm * dh * (2 * de)
    flop_total = 6.0 * R * dh * de
    peaks = load_peaks()
    fp4_peak = 4.0 * peaks["bf16_tflops"]
    achieved = flop_gate_up / (stages["gemm_gate_up_ms"] * 1e-3) / 1e12
    traffic = None
    tf = ROOT / "profiles" / "gemm_gate_up_config1_traffic.json"
    if tf.exists() and cfg["name"] == "config1" and world == 1:
        traffic = json.loads(tf.read_text()).get("bytes_per_launch")
    layer_tflops = flop_total / (ms_step * 1e-3) / 1e12
    value = world * S / (ms_step * 1e-3)
    lib = None
    if not args.no_extras:
        lib = fp4_library_ceiling(torch_device(world), R_gemm, 2 * de, dh)
    roof = {"kernel": "ffn_gemm_nvfp4_kernel<EPI_SWIGLU> (gate/up GEMM)", "bound": "tensor",
            "achieved": round(achieved, 1), "peak": round(fp4_peak, 1), "unit": "TFLOP/s",
            "frac": round(achieved / fp4_peak, 4), "traffic": traffic,
            "peak_note": f"4 x {peaks['source']} bf16 burst {peaks['bf16_tflops']} TFLOP/s (dense FP4 = 4x bf16 "
                         f"on B200; the kernel is timed inside a ~1 ms step); datasheet dense FP4 9000 TFLOP/s -> "
                         f"frac {achieved / 9000.0:.4f}",
            "algorithmic_flop_per_launch": flop_gate_up,
            "traffic_note": "dram__bytes_read.sum + dram__bytes_write.sum of one gate/up launch at config 1 "
                            "(profiles/gemm_gate_up_config1_traffic.json)" if traffic else None}
    if lib is not None:
        roof["library_fp4_ceiling"] = dict(lib, frac=round(achieved / lib["tflops"], 4) if lib.get("tflops") else None)
    out = {
        "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "nvfp4 (e2m1 x ue4m3/16, fp32 accumulate; bf16 in/out)",
        "data": f"synthetic (seeded, {cfg['name']} distributions)",
        "config": {"workload": _workload(cfg, world),
                   "tokens_per_gpu": S, "global_batch": world * S,
                   "parallelism": f"ep{world} (token->expert all-to-all, NCCL)" if world > 1 else "1 GPU",
                   "l2": "inputs larger than L2 (NVFP4 weights of every expert + x streamed every step)"},
        "tokens_per_s_per_gpu": round(value / world, 1),
        "layer_tflops": round(layer_tflops, 1),
        "nvfp4_util_pct": {"vs_4x_measured_bf16_burst": round(100 * layer_tflops / fp4_peak, 2),
                           "vs_datasheet_9pf": round(100 * layer_tflops / 9000.0, 2),
                           "vs_library_fp4_ceiling": (round(100 * layer_tflops / lib["tflops"], 2)
                                                      if lib and lib.get("tflops") else None)},
        "stages_ms": {k: round(v, 4) for k, v in stages.items()},
        "roofline": roof,
        "e2e": None if e2e_ms[0] != e2e_ms[0] else {
            "value": round(world * S / (e2e_ms[0] * 1e-3), 1), "unit": "tokens/s",
            "h2d_bytes_per_step": S * d * 2, "d2h_bytes_per_step": S * d * 2, "ms_per_step": round(e2e_ms[0], 4),
            "api": "CoreMultiHeadMoE.forward (custom op magi2_b200::mh_moe)",
            "copies": "per step: input copied from pinned host memory, output copied back; copies on their own "
                      "streams, double-buffered, overlapping the neighbouring steps' compute",
            "serial": {"value": round(world * S / (e2e_ms[1] * 1e-3), 1), "ms_per_step": round(e2e_ms[1], 4),
                       "note": "copy in, compute, copy out on one stream"}},
        "gpu_launches": (KERNELS_PER_STEP if world == 1 else KERNELS_PER_STEP_EP) * args.steps,   # kernels of libmhmoe inside the device-timed region
        "clocks": clk.summary(),
    }
    if world > 1:
        import torch.distributed as dist
        from flash_mh_moe.ep import LAST_STATS, ep_chunks
        every = [None] * world
        dist.all_gather_object(every, {k: round(v, 4) for k, v in stages.items()})
        out["stages_ms_min_max_over_ranks"] = {k: [min(e[k] for e in every), max(e[k] for e in every)]
                                               for k in stages}
        out["config"]["parallelism"] = (f"ep{world} (token->expert records, "
                                        + (f"fused NVLink peer stores, {ep_chunks()}-chunk pipeline)"
                                           if LAST_STATS.get("transport") == "peer"
                                           else "NCCL all-to-all)"))
        if LAST_STATS.get("transport") == "nccl":
            bd, br = LAST_STATS.get("dispatch_remote_bytes", 0), LAST_STATS.get("return_remote_bytes", 0)
            td, tr = stages["a2a_records_ms"], stages["a2a_return_ms"]
            out["nvlink"] = {"records_remote_bytes": bd, "return_remote_bytes": br,
                             "records_GBps": round(bd / (td * 1e-3) / 1e9, 1) if td > 0 else None,
                             "return_GBps": round(br / (tr * 1e-3) / 1e9, 1) if tr > 0 else None,
                             "peak": 770.0, "unit": "GB/s per direction per GPU",
                             "note": "rank 0: bytes it sends to other ranks / device time of that all-to-all "
                                     "(NCCL; includes waiting for the slowest peer); peak = measured peer copy"}
        else:
            bd = int(LAST_STATS["records_remote_bytes"].item()) if "records_remote_bytes" in LAST_STATS else 0
            br = int(LAST_STATS["return_remote_bytes"].item()) if "return_remote_bytes" in LAST_STATS else 0
            td, tr = stages["a2a_records_ms"], stages["local_combine_ms"]
            out["nvlink"] = {"records_remote_bytes": bd, "return_remote_bytes": br,
                             "records_GBps": round(bd / (td * 1e-3) / 1e9, 1) if td > 0 else None,
                             "return_GBps": round(br / (tr * 1e-3) / 1e9, 1) if tr > 0 else None,
                             "peak": 770.0, "unit": "GB/s per direction per GPU",
                             "note": "rank 0, pipeline chunk 0: remote bytes of the record kernel over its time "
                                     "plus the wait for every source (a2a_records_ms), and remote bytes of the "
                                     "fused combine-and-return kernel over its time (local_combine_ms, which "
                                     "also reads the partial rows); peak = measured peer copy"}
    if world == 1 and not args.no_cpu_baseline and not args.release_master and args.config == "1":
        out["cpu_baseline"] = cpu_baseline(m, x_host, cfg, reps=2)
    return out


def run_stack(args, cfg, dev):
    """Config 4: 4 MoE layers stacked with a bf16 residual add, 256 tokens — dominated by
    streaming each layer's NVFP4 weights from HBM (reported as GB/s)."""
    import torch
    from flash_mh_moe import _lib
    layers = []
    for i in range(cfg["layers"]):
        m, x_host = make_layer(dict(cfg, seed=cfg["seed"] * 10 + i), dev, 0)
        m.release_master_weights()
        layers.append(m)
    torch.cuda.empty_cache()
    x0 = x_host.to(dev)

    def fwd(x):
        for m in layers:
            x = x + m(x)
        return x
    for _ in range(args.warmup):
        fwd(x0)
    torch.cuda.synchronize()
    _lib.check_device_status(dev)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # eager (host launches every step)
    t0.record()
    for _ in range(args.steps):
        fwd(x0)
    t1.record()
    torch.cuda.synchronize()
    ms_eager = t0.elapsed_time(t1) / args.steps
    # the same stack replayed as one CUDA graph (flash_mh_moe.graph): the timed value
    from flash_mh_moe.graph import CapturedForward
    g = CapturedForward(fwd, x0, warmup=args.warmup)
    for _ in range(args.warmup):
        g(x0)
    torch.cuda.synchronize()
    _lib.check_device_status(dev)
    with ClockSampler(0) as clk:
        h0 = time.perf_counter()
        t0.record()
        for _ in range(args.steps):
            g(x0)
        t1.record()
        torch.cuda.synchronize()
        clk.window(h0, time.perf_counter())
    ms = t0.elapsed_time(t1) / args.steps
    gu, dn = layers[0].packed_weights()
    wbytes = sum(t.numel() * t.element_size() for t in (gu.data, gu.sf, gu.gscale, dn.data, dn.sf, dn.gscale))
    act = cfg["S"] * cfg["d"] * 2 * 2
    total_bytes = cfg["layers"] * (wbytes + act)
    peaks = load_peaks()
    gbs = total_bytes / (ms * 1e-3) / 1e9
    return {"metric": METRIC, "value": round(cfg["S"] / (ms * 1e-3), 1), "unit": "tokens/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "nvfp4 (e2m1 x ue4m3/16, fp32 accumulate; bf16 in/out)",
            "data": "synthetic (seeded, config-4 distributions)",
            "config": {"workload": f"config4: {cfg['S']} tokens, {cfg['layers']} stacked MoE layers + bf16 residual, "
                                   "d=3072, E=128, top-8, de=1024", "tokens_per_gpu": cfg["S"],
                       "launch": "the 4-layer stack replayed as one CUDA graph (flash_mh_moe.graph.CapturedForward)"},
            "eager": {"ms_per_step": round(ms_eager, 4), "value": round(cfg["S"] / (ms_eager * 1e-3), 1),
                      "hbm_gbs": round(total_bytes / (ms_eager * 1e-3) / 1e9, 1)},
            "roofline": {"kernel": "whole 4-layer stack (weight streaming)", "bound": "hbm",
                         "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": round(gbs / peaks["hbm_gbs"], 4), "traffic": None,
                         "algorithmic_bytes_per_step": total_bytes,
                         "peak_note": f"{peaks['source']} HBM copy bandwidth; vs 8000 GB/s nominal: {gbs / 8000:.3f}"},
            "gpu_launches": KERNELS_PER_STEP * cfg["layers"] * args.steps, "clocks": clk.summary()}


# ───────────────────────────── CPU reference path ─────────────────────────────
# The reference's own layer path on the host cores: its route.py top-k and global sort and
# its _scatter_back run unchanged from the staged copy under oracle/_ref (oracle/stage_ref.py),
# with the Triton expert kernel restated in torch (oracle/ffn_torch_ref.py; the reference
# has no CPU version of it).  Without the staged copy the oracle's restatement of route.py
# stands in.  torch uses every host thread.

def _cpu_threads() -> int:
    import torch
    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    return torch.get_num_threads()


def _staged_ref():
    try:
        from oracle.stage_ref import import_ref
        return import_ref()
    except ImportError:
        return None


def _host_layer(m, x_host, n_tokens):
    import torch
    with torch.no_grad():
        w = tuple(t.detach().to("cpu", torch.bfloat16) for t in (m.W_gate, m.W_up, m.W_down))
        gate = m.gate.detach().float().cpu()
        bias = m.router.expert_bias.detach().float().cpu()
    x = x_host[:n_tokens].view(n_tokens, m.num_heads, m.d_head).contiguous()
    return x, gate, w, bias


def cpu_layer(m, host, cfg, ref):
    from oracle import ffn_torch_ref
    x, gate, (Wg, Wu, Wd), bias = host
    return ffn_torch_ref.moe_layer_cpu(x, gate, Wg, Wu, Wd, cfg["E"], cfg["K"], cfg["score_func"],
                                       cfg.get("route_scale", 1.0), bias, ref=ref)


def _cpu_sample_note(cfg, n, ref, extra=""):
    return (f"first {n} tokens of the {cfg['name']} batch through the whole layer (router einsum, top-k, sort, all "
            f"{cfg['E'] * cfg['H']} experts' bf16 FFN, scatter)" + extra + "; "
            + ("reference route.py + _scatter_back (staged oracle/_ref) with the expert kernel restated in torch"
               if ref is not None else "oracle restatement of route.py with the expert kernel restated in torch"))


def cpu_baseline(m, x_host, cfg, reps=2):
    cores = _cpu_threads()
    ref = _staged_ref()
    n = min(CPU_SAMPLE_TOKENS, cfg["S"])
    host = _host_layer(m, x_host, n)
    times = []
    for _ in range(reps + 1):
        t = time.perf_counter()
        cpu_layer(m, host, cfg, ref)
        times.append(time.perf_counter() - t)
    best = min(times[1:])
    return {"value": round(n / best, 1), "unit": "tokens/s", "cores": cores, "kind": "reference" if ref else "port",
            "sample": _cpu_sample_note(cfg, n, ref, f", best of {reps} after 1 warm-up")}


def _triton_reference_gpu(ref, dev):
    """The reference's own Triton expert kernel (mh_moe_fwd_func) on this GPU, at the shapes
    it is written for: MAGI-2's production head split and BASELINE config 0.  Triton
    rejects a kernel whose tensor-memory need exceeds the SM's 512 columns before launching
    it; that refusal is reported as is."""
    import torch
    from ref_flash_mh_moe.triton.mh_moe_fwd import mh_moe_fwd_func
    out = {}
    for name, (S, H, dh, E, K, de, score, scale) in {
            "prod_head_split": (16384, 12, 256, 256, 6, 1280, "sigmoid", 4.9),
            "config0": (512, 1, 1024, 8, 2, 2048, "softmax", 1.0)}.items():
        g = torch.Generator(device=dev).manual_seed(0)
        try:
            x = torch.randn(S, H, dh, device=dev, generator=g).to(torch.bfloat16)
            W = [(torch.randn(H * E, a, b, device=dev, generator=g) * 0.02).to(torch.bfloat16)
                 for a, b in ((dh, de), (dh, de), (de, dh))]
            gate = (torch.randn(H, E, dh, device=dev, generator=g) * 0.02).float()

            def layer():
                logits = torch.einsum("shd,hed->hse", x.float(), gate)
                p, i = ref.compute_topk_probs_and_indices(logits, K, score_func=score)
                gi, ps, of = ref.flash_mh_moe_global_sort(p * scale, i, E)
                return mh_moe_fwd_func(x, gi, ps, of, *W, deterministic=False)
            layer()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(5):
                layer()
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / 5
            out[name] = {"ms_per_step": round(ms, 4), "tokens_per_s": round(S / (ms * 1e-3), 1)}
        except Exception as e:
            out[name] = {"unavailable": f"{type(e).__name__}: {str(e).splitlines()[0][:160]}"}
        finally:
            x = W = gate = None
            torch.cuda.empty_cache()
    return out


def run_reference(args, world, rank):
    import torch
    if rank != 0:
        return None
    cfg = CFG1
    dev = torch.device("cuda", 0)
    cores = _cpu_threads()
    ref = _staged_ref()
    m, x_host = make_layer(cfg, dev, 0)
    n = CPU_SAMPLE_TOKENS
    host = _host_layer(m, x_host, n)
    del m
    torch.cuda.empty_cache()
    for _ in range(args.warmup):
        cpu_layer(None, host, cfg, ref)
    t = time.perf_counter()
    for _ in range(args.steps):
        cpu_layer(None, host, cfg, ref)
    dt = (time.perf_counter() - t) / args.steps
    v = n / dt
    out = {"impl": "reference", "metric": METRIC, "value": round(v, 1), "unit": "tokens/s", "n_gpus": world,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3),
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16 (fp32 accumulate)",
           "data": "synthetic (seeded, config1 distributions)",
           "config": {"workload": _workload(cfg, 1), "sample_tokens_per_step": n, "parallelism": "host CPU"},
           "cpu_baseline": {"value": round(v, 1), "unit": "tokens/s", "cores": cores,
                            "kind": "reference" if ref else "port", "sample": _cpu_sample_note(cfg, n, ref)},
           "e2e": {"value": round(v, 1), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
           "gpu_launches": 0}
    if ref is not None and not args.no_extras:
        out["triton_reference_gpu"] = _triton_reference_gpu(ref, dev)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)   # ~0.11 s timed at config 1: ~20 clock samples
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end leg (profiling runs)")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the other-scatter and 8192-token timings (profiling runs)")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="1",
                    help="BASELINE config at N=1 (1: headline; 2: Zipf-skewed routing; 4: 4-layer small batch; "
                         "prod: MAGI-2's production head split)")
    ap.add_argument("--release-master", action="store_true",
                    help="free the bf16 expert weights after NVFP4 packing (profiler captures)")
    ap.add_argument("--tokens", type=int, default=None,
                    help="tokens per GPU (default: config 1's 16384; smaller only for profiler captures)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    world, rank, local = dist_setup()
    try:
        out = run_reference(args, world, rank) if args.impl == "reference" else run_ours(args, world, rank, local)
        if rank == 0 and out is not None:
            print(json.dumps(out), flush=True)
    finally:
        import torch.distributed as dist
        if dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
