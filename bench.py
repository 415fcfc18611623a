#!/usr/bin/env python
"""Benchmark of the Qwen3-VL-2B attention hot path on B200.

Headline (one JSON line on rank 0): config 2 of the baseline — one batched
decode STEP of the text decoder: for each of 28 layers, the new token's q/k
are rotated and k/v appended to that layer's padded cache (fused RoPE + append
kernel), then GQA decode attention runs over each request's valid prefix
(split-KV decode kernel).  B=64 requests per GPU, 16 q heads / 8 KV heads,
head_dim 128, bf16, per-request lengths ~ U[256, 4096] in caches padded to 4096.
The metric is algorithmic HBM bytes moved per second (GB/s), whole job.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 is launched with torchrun, one rank per GPU: every rank runs its own
batch of 64 requests (decode shards by request, no collective; weak scaling).
Secondary numbers in the same line: config 5 (B=4, L=131072) sequence-sharded
across the N ranks with one NCCL all-gather of the (out, LSE) partials, and the
tensor-core prefill (config 4) / ViT varlen (config 3) kernels when built.

``--impl reference`` times the reference's own CPU path (restated in
oracle/reference_cpu.py, as the reference is Python and does not travel) on
the host cores for the same workload and metric.
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

METRIC = "decode-attn HBM GB/s (% peak); prefill/ViT attn TFLOPS; scaling 1/2/4/8 GPU"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
B, L_CAP, LAYERS = 64, 4096, 28


def log(*a):
    print(*a, file=sys.stderr, flush=True)


# ------------------------------------------------------------------ peaks / traffic


def load_peaks() -> tuple[dict, str]:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return {k: float(d[k]) for k in ("hbm_gbs", "bf16_tflops", "bf16_tflops_sustained")}, "measured"
        except Exception:  # noqa: BLE001
            pass
    return dict(FALLBACK_PEAKS), "fallback"


def profiled_traffic(name: str) -> float | None:
    """dram bytes per launch from a committed ncu summary (a line 'dram_bytes_per_launch: N')."""
    p = REPO / "profiles" / name
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.strip().startswith("dram_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].split()[0])
            except ValueError:
                return None
    return None


# ------------------------------------------------------------------ clocks


class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML while running."""

    REASONS = {
        0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
        0x80: "hw_power_brake_slowdown", 0x2: "applications_clocks_setting", 0x10: "sync_boost",
    }

    def __init__(self, device_index: int, period_s: float = 0.02):
        self.samples: list[int] = []
        self.reasons = 0
        self.max_mhz = None
        self.err = None
        self._stop = threading.Event()
        self._period = period_s
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nvml = pynvml
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            phys = int(vis.split(",")[device_index]) if vis else device_index
            self._h = pynvml.nvmlDeviceGetHandleByIndex(phys)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # noqa: BLE001
            self._nvml = None
            self.err = str(e)
        self._t = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self._nvml.nvmlDeviceGetClockInfo(self._h, self._nvml.NVML_CLOCK_SM))
                self.reasons |= int(self._nvml.nvmlDeviceGetCurrentClocksEventReasons(self._h))
            except Exception as e:  # noqa: BLE001
                self.err = str(e)
                return
            time.sleep(self._period)

    def __enter__(self):
        if self._nvml is not None:
            self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._t.is_alive():
            self._t.join()

    def summary(self) -> dict:
        out = {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
               "reasons": [n for bit, n in self.REASONS.items() if self.reasons & bit], "samples": len(self.samples),
               "source": "nvml"}
        if self.err:
            out["error"] = self.err
        return out


# ------------------------------------------------------------------ distributed helpers


def pin_host_cores(local: int, world: int) -> None:
    """One disjoint slice of this process's allowed host cores per local rank,
    so the ranks' Python threads (which issue every launch and copy of the
    end-to-end step) do not compete for the same cores."""
    cores = sorted(os.sched_getaffinity(0))
    per = len(cores) // world
    if per >= 1:
        mine = cores[local * per:(local + 1) * per]
        os.sched_setaffinity(0, mine)
        torch.set_num_threads(len(mine))


def dist_info():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def max_over_ranks(x: float, world: int, device) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int, device):
    if world > 1:
        import torch.distributed as dist

        dist.barrier(device_ids=[device.index])
    torch.cuda.synchronize(device)


# ------------------------------------------------------------------ workload


def step_bytes(lengths: torch.Tensor, layers: int = LAYERS) -> dict:
    """Algorithmic bytes of one config-2 step (padded slots are not counted)."""
    hq, hkv, d, e = 16, 8, 128, 2
    kv = int(sum(2 * hkv * d * e * (int(n) + 1) for n in lengths))  # K and V of the valid prefix incl. the new token
    qo = 2 * B * hq * d * e                                         # decode reads q, writes o
    rope = B * (hq + 2 * hkv) * d * e + 2 * B * d * e + B * hq * d * e + 2 * B * hkv * d * e
    return {"decode_per_layer": kv + qo, "rope_per_layer": rope, "step": layers * (kv + qo + rope)}


def cfg2_config(world: int, layers: int = LAYERS) -> dict:
    """The headline workload's ``config``, printed identically by both arms."""
    from aicas_b200 import workloads as wl

    lengths = wl.cfg2_lengths(0)
    return {"workload": f"cfg2: batched GQA decode step (RoPE + KV append + decode) x {layers} layers",
            "batch_per_gpu": B, "layers": layers, "q_heads": 16, "kv_heads": 8, "head_dim": 128,
            "kv_capacity": L_CAP, "lengths": "U[256,4096] seed 0", "mean_len": round(float(lengths.float().mean()), 2),
            "parallelism": f"dp{world} (requests sharded, no collective)",
            "l2": "inputs larger than L2 (571 MB of valid KV per layer)"}


class DecodeWorkload:
    def __init__(self, device, seed: int, layers: int = LAYERS):
        import aicas_b200 as ab
        from aicas_b200 import workloads as wl

        self.ab, self.wl = ab, wl
        self.device = device
        self.layers = layers
        self.lengths = wl.cfg2_lengths(0)
        self.caches = [wl.cfg2_cache(B, L_CAP, layer, seed=seed, device=device) for layer in range(layers)]
        self.inputs = [wl.cfg2_step_inputs(self.lengths, layer, seed=seed, device=device) for layer in range(layers)]
        self.lens_after = torch.empty(B, dtype=torch.int32, device=device)
        self.q_rot = [torch.empty(B, 1, 16, 128, dtype=torch.bfloat16, device=device).transpose(1, 2)
                      for _ in range(layers)]
        self.bytes = step_bytes(self.lengths, layers)

    def step(self, decode_events=None):
        ab, wl = self.ab, self.wl
        outs = []
        for layer in range(self.layers):
            x = self.inputs[layer]
            kc, vc = self.caches[layer]
            ab.rope_kv_append(x.q, x.k, x.v, x.cos, x.sin, kc, vc, x.positions, q_out=self.q_rot[layer],
                              kv_lens_out=self.lens_after)
            if decode_events is not None:
                decode_events[layer][0].record()
            outs.append(ab.gqa_decode_attention(self.q_rot[layer], kc, vc, sm_scale=wl.SCALE_TEXT,
                                                num_key_value_groups=2, kv_lens=self.lens_after))
            if decode_events is not None:
                decode_events[layer][1].record()
        return outs


def run_decode(args, world, rank, device, peaks, peak_src) -> dict:
    """The headline: config-2 decode steps replayed from one CUDA graph."""
    wk = DecodeWorkload(device, seed=rank, layers=args.layers)
    torch.cuda.synchronize(device)

    # --- capture the 28-layer step (56 launches) in a CUDA graph, with timing
    # events around every decode launch recorded as graph nodes
    cap_stream = torch.cuda.Stream(device)
    cap_stream.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(cap_stream):
        for _ in range(max(args.warmup, 3)):
            wk.step()
    torch.cuda.current_stream(device).wait_stream(cap_stream)
    torch.cuda.synchronize(device)
    def capture(with_events: bool):
        ev = ([[torch.cuda.Event(enable_timing=True, external=True) for _ in range(2)] for _ in range(wk.layers)]
              if with_events else None)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=cap_stream):
            wk.step(decode_events=ev)
        return g, ev

    # two captures of the same step: without events (the timed replays), and
    # with timing events around every decode launch, replayed as the LAST timed
    # step so that the roofline's per-launch times come from the timed region
    # while the events' own cost touches one step of K
    graph, _ = capture(False)
    try:
        graph_ev, ev = capture(True)
        timing_mode = "events recorded as graph nodes around every decode launch of the last timed step"
    except Exception as exc:  # noqa: BLE001  (older drivers: no timing events in graphs)
        log(f"event capture failed ({exc}); timing decode launches eagerly")
        torch.cuda.synchronize(device)
        graph_ev, ev = None, None
        timing_mode = "eager step with events around each decode launch, after the timed replays"
    for _ in range(max(args.warmup, 3)):
        graph.replay()
        if graph_ev is not None:
            graph_ev.replay()
    torch.cuda.synchronize(device)

    # --- timed region: K graph replays (inputs 571 MB of KV per layer > L2)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    last = torch.cuda.Event(enable_timing=True)
    barrier(world, device)
    with ClockSampler(device.index) as clocks:
        start.record()
        for i in range(args.steps):
            if i == args.steps - 1:
                last.record()
            (graph_ev if graph_ev is not None and i == args.steps - 1 else graph).replay()
        end.record()
        torch.cuda.synchronize(device)
    last_step_ms = last.elapsed_time(end)
    elapsed_ms = start.elapsed_time(end)
    barrier(world, device)
    elapsed_ms = max_over_ranks(elapsed_ms, world, device)
    ms_step = elapsed_ms / args.steps
    value = world * wk.bytes["step"] / (ms_step * 1e-3) / 1e9
    if graph_ev is not None:
        # the events hold the launches of the last timed step (28 decode launches)
        dec_ms = [a.elapsed_time(b) for a, b in ev]
    else:
        ev = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(wk.layers)]
        wk.step(decode_events=ev)
        torch.cuda.synchronize(device)
        dec_ms = [a.elapsed_time(b) for a, b in ev]
    dec_avg_ms = statistics.mean(dec_ms)
    achieved = wk.bytes["decode_per_layer"] / (dec_avg_ms * 1e-3) / 1e9
    roofline = {"bound": "hbm", "kernel": "decode_gqa_kernel<bf16,128,2>", "achieved": round(achieved, 1),
                "timing": timing_mode, "launches_timed": len(dec_ms),
                "peak": peaks["hbm_gbs"], "peak_source": f"{peak_src} hbm_gbs", "unit": "GB/s",
                "frac": round(achieved / peaks["hbm_gbs"], 4),
                "traffic": profiled_traffic("decode_gqa_cfg2.txt"),
                "algorithmic_bytes_per_launch": wk.bytes["decode_per_layer"],
                "avg_launch_us": round(dec_avg_ms * 1e3, 2),
                "decode_share_of_step": round(sum(dec_ms) / last_step_ms, 3) if graph_ev is not None
                else round(dec_avg_ms * wk.layers / ms_step, 3)}
    del graph, graph_ev
    e2e = run_e2e(wk, args, world, device) if args.e2e else None
    out = {
        "value": round(value, 1), "ms_per_step": round(ms_step, 4), "config": cfg2_config(world, wk.layers),
        "execution": f"{wk.layers}-layer step captured in one CUDA graph ({2 * wk.layers} launches), replayed",
        "roofline": roofline, "gpu_launches": args.steps * wk.layers * 2, "clocks": clocks.summary(),
    }
    if e2e is not None:
        out["e2e"] = e2e
    del wk
    torch.cuda.empty_cache()
    return out


def _layer_chunks(layers: int) -> list[tuple[int, int]]:
    """Layer ranges [0,1), [1,2), [2,4), [4,8), ... : the inputs of each range
    travel in one host-to-device copy and arrive before the layers ahead of it
    have finished (a layer's inputs cross PCIe ~10x faster than it computes)."""
    bounds, b = [0], 1
    while b < layers:
        bounds.append(b)
        b *= 2
    bounds.append(layers)
    return list(zip(bounds[:-1], bounds[1:]))


def run_e2e(wk: DecodeWorkload, args, world, device) -> dict:
    """Same step through the public HF-facing API, inputs copied from pinned host
    memory every step and the attention outputs read back.  A step's inputs sit
    in one pinned buffer, layer after layer, and go over in a few large copies
    (see _layer_chunks) on a copy stream; one event per chunk orders its layers'
    compute after their inputs, and one per layer orders its read-back after its
    output, so PCIe traffic overlaps the attention of the layers before it."""
    from aicas_b200 import backends
    import aicas_b200 as ab

    class Attn(torch.nn.Module):
        num_key_value_groups, scaling, is_causal = 2, wk.wl.SCALE_TEXT, True

    mod = Attn()
    layout, off, layer_end = [], 0, []
    for x in wk.inputs:
        views = []
        for t in (x.q, x.k, x.v, x.cos, x.sin, x.positions):
            nb = t.numel() * t.element_size()
            views.append((off, nb, t))
            off = (off + nb + 255) // 256 * 256
        layout.append(views)
        layer_end.append(off)
    host_buf = torch.empty(off, dtype=torch.uint8).pin_memory()
    dev_buf = torch.empty(off, dtype=torch.uint8, device=device)
    dev_in = []
    for views in layout:
        ins = []
        for o, nb, t in views:
            host_buf[o:o + nb].copy_(t.detach().cpu().contiguous().view(-1).view(torch.uint8))
            ins.append(dev_buf[o:o + nb].view(t.dtype).view(t.shape))
        dev_in.append(ins)
    chunks = _layer_chunks(wk.layers)
    spans = [(0 if a == 0 else layer_end[a - 1], layer_end[b - 1]) for a, b in chunks]
    host_out = [torch.empty(B, 1, 16, 128, dtype=torch.bfloat16).pin_memory() for _ in range(wk.layers)]
    h2d = off
    d2h = sum(t.numel() * t.element_size() for t in host_out)
    lens_after = torch.empty(B, dtype=torch.int32, device=device)
    main = torch.cuda.current_stream(device)
    copy = torch.cuda.Stream(device)
    ev_in = [torch.cuda.Event() for _ in chunks]
    ev_out = [torch.cuda.Event() for _ in range(wk.layers)]
    chunk_of = [next(i for i, (a, b) in enumerate(chunks) if a <= layer < b) for layer in range(wk.layers)]

    def one_step(main):
        with torch.cuda.stream(copy):
            copy.wait_stream(main)  # the previous step's readers of the input buffer are done
            for i, (lo, hi) in enumerate(spans):
                dev_buf[lo:hi].copy_(host_buf[lo:hi], non_blocking=True)
                ev_in[i].record(copy)
        for layer in range(wk.layers):
            if layer == chunks[chunk_of[layer]][0]:
                main.wait_event(ev_in[chunk_of[layer]])
            q, k, v, cos, sin, pos = dev_in[layer]
            kc, vc = wk.caches[layer]
            q_rot = ab.rope_kv_append(q, k, v, cos, sin, kc, vc, pos, kv_lens_out=lens_after)
            out, _ = backends.text_triton_attention(mod, q_rot, kc, vc, None, kv_lens=lens_after)
            ev_out[layer].record(main)
            with torch.cuda.stream(copy):
                copy.wait_event(ev_out[layer])
                host_out[layer].copy_(out, non_blocking=True)
                keep[layer] = out  # alive until the copy stream has read it
        main.wait_stream(copy)

    keep = [None] * wk.layers
    steps = max(3, min(args.steps, 50))

    def timed_loop(step) -> tuple[float, float]:
        for _ in range(max(args.warmup, 3)):
            step()
        torch.cuda.synchronize(device)
        barrier(world, device)
        t0 = time.perf_counter()
        for _ in range(steps):
            step()
        issued = time.perf_counter()
        torch.cuda.synchronize(device)
        ms = (time.perf_counter() - t0) * 1e3 / steps
        host_ms = (issued - t0) * 1e3 / steps
        return max_over_ranks(ms, world, device), max_over_ranks(host_ms, world, device)

    main = torch.cuda.current_stream(device)
    eager_ms, eager_host_ms = timed_loop(lambda: one_step(main))
    # the same step captured in one CUDA graph, the host copies as graph nodes:
    # the host then issues one launch per step instead of 56 operator calls
    cap = torch.cuda.Stream(device)
    cap.wait_stream(main)
    with torch.cuda.stream(cap):
        one_step(cap)
    main.wait_stream(cap)
    torch.cuda.synchronize(device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=cap):
        one_step(cap)
    ms, host_ms = timed_loop(graph.replay)
    del graph
    gbs = lambda t: round(world * wk.bytes["step"] / (t * 1e-3) / 1e9, 1)  # noqa: E731
    return {"value": gbs(ms), "unit": "GB/s", "ms_per_step": round(ms, 4), "steps": steps,
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "host_issue_ms_per_step": round(host_ms, 4),
            "api": "aicas_b200.rope_kv_append + backends.text_triton_attention (HF attention interface)",
            "timing": "wall clock around the step loop, device synchronised; the step (its pinned-host -> device "
                      "input copies, 56 operator calls and device -> pinned-host output copies, copies on a copy "
                      "stream) captured in one CUDA graph and replayed",
            "h2d_copies_per_step": len(spans), "d2h_copies_per_step": wk.layers,
            "eager": {"value": gbs(eager_ms), "ms_per_step": round(eager_ms, 4),
                      "host_issue_ms_per_step": round(eager_host_ms, 4)},
            "host_cores": len(os.sched_getaffinity(0))}


CFG5_B, CFG5_L, CFG5_CHUNK = 4, 131072, 16384


def cfg5_shard(s0: int, s1: int, device) -> tuple[torch.Tensor, torch.Tensor]:
    """Positions [s0, s1) of config 5's K and V ([4, 8, L, 128] bf16).  The whole
    cache is defined chunk by chunk (16384 positions, chunk c drawn from seed
    5000 + c), so it is the same for every rank count and a rank generates
    only the chunks its shard touches."""
    from aicas_b200 import workloads as wl

    ks, vs = [], []
    for c in range(s0 // CFG5_CHUNK, (s1 + CFG5_CHUNK - 1) // CFG5_CHUNK):
        g = wl.generator(5000 + c, device)
        k = wl.randn((CFG5_B, 8, CFG5_CHUNK, 128), g, torch.bfloat16, device)
        v = wl.randn((CFG5_B, 8, CFG5_CHUNK, 128), g, torch.bfloat16, device)
        lo, hi = max(s0 - c * CFG5_CHUNK, 0), min(s1 - c * CFG5_CHUNK, CFG5_CHUNK)
        ks.append(k[:, :, lo:hi])
        vs.append(v[:, :, lo:hi])
    return torch.cat(ks, 2).contiguous(), torch.cat(vs, 2).contiguous()


def cfg5_reference(q: torch.Tensor, device) -> torch.Tensor:
    """fp32 decode over the whole config-5 cache: softmax(scale q K^T) V per
    (request, query head), [4, 16, 128] fp32, computed one request at a time."""
    from aicas_b200 import workloads as wl

    k, v = cfg5_shard(0, CFG5_L, device)
    out = torch.empty(CFG5_B, 16, 128, dtype=torch.float32, device=device)
    for b in range(CFG5_B):
        kb, vb = k[b].float(), v[b].float()                       # [8, L, 128]
        qb = q[b, :, 0].float().view(8, 2, 128)                   # query heads 2h, 2h+1 read KV head h
        p = torch.softmax(torch.einsum("hgd,hkd->hgk", qb, kb) * wl.SCALE_TEXT, dim=-1)
        out[b] = torch.einsum("hgk,hkd->hgd", p, vb).reshape(16, 128)
    return out


def _parity(out: torch.Tensor, ref: torch.Tensor, world: int, device) -> dict:
    """max-abs / mean-abs of every rank's merged output against the fp32
    reference (max over ranks), held to the north-star bf16 bar."""
    err = (out.float().reshape(ref.shape) - ref).abs()
    stats = torch.tensor([float(err.max()), float(err.mean()), float(torch.isfinite(out.float()).all() == 0)],
                         dtype=torch.float64, device=device)
    if world > 1:
        import torch.distributed as dist

        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
    mx, mean, nonfinite = (float(x) for x in stats.tolist())
    return {"max_abs": round(mx, 6), "mean_abs": round(mean, 7), "tolerance": {"max_abs": 2e-2, "mean_abs": 2e-3},
            "ok": bool(nonfinite == 0 and mx <= 2e-2 and mean <= 2e-3), "against": "fp32 torch over the whole cache"}


def run_split_kv(args, world, rank, device) -> dict:
    """Config 5: B=4, L=131072 sequence-sharded over the ranks (strong scaling).
    At N > 1 the partials are exchanged and merged by the one-kernel NVLink
    peer exchange, or the decode kernel exchanges and merges itself (the fused
    path); the NCCL all-gather + merge path is timed beside them.  All three
    are checked once, outside the timed loops, against an fp32 decode of the
    whole cache; the calls are timed eagerly and replayed from a CUDA graph,
    with the partial decode and exchange kernels timed apart and the host issue
    time."""
    import aicas_b200 as ab
    from aicas_b200 import distributed as adist
    from aicas_b200 import ops
    from aicas_b200 import workloads as wl

    Bq, L = CFG5_B, CFG5_L
    s0, s1 = adist.shard_bounds(L, world, rank)
    q = wl.randn((Bq, 16, 1, 128), wl.generator(5, device), torch.bfloat16, device)
    k, v = cfg5_shard(s0, s1, device)
    exchange = adist.PeerExchange(Bq, 16, 128, device) if world > 1 else None
    iters = max(10, min(200, args.steps))

    def timed(once) -> tuple[float, float]:
        """(device ms per call, max over ranks; host ms to issue one call)"""
        for _ in range(max(args.warmup, 3)):
            once()
        barrier(world, device)
        st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        st.record()
        t0 = time.perf_counter()
        for _ in range(iters):
            once()
        host = (time.perf_counter() - t0) * 1e3 / iters
        en.record()
        torch.cuda.synchronize(device)
        return max_over_ranks(st.elapsed_time(en) / iters, world, device), max_over_ranks(host, world, device)

    def in_graph(once):
        """`once` captured in a CUDA graph (warmed up on the capture stream first,
        so that its workspace exists before the capture)."""
        s = torch.cuda.Stream(device)
        s.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(s):
            for _ in range(3):
                once()
        torch.cuda.current_stream(device).wait_stream(s)
        torch.cuda.synchronize(device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            once()
        return g

    kw = dict(sm_scale=wl.SCALE_TEXT, num_key_value_groups=2)
    ref = cfg5_reference(q, device) if rank == 0 else torch.empty(Bq, 16, 128, device=device)
    if world > 1:
        import torch.distributed as dist

        dist.broadcast(ref, src=0)
    kv_bytes = 2 * Bq * 8 * L * 128 * 2
    base = {"scaling": "strong", "batch": Bq, "kv_len": L, "per_gpu_kv_len": s1 - s0,
            "data": "seeded N(0,1) chunks of 16384 positions, the same whole cache at every rank count"}
    if world == 1:
        decode = lambda: ab.gqa_decode_attention(q, k, v, **kw)  # noqa: E731
        parity = _parity(decode(), ref, world, device)
        ms_eager, host = timed(decode)
        g = in_graph(decode)
        ms, _ = timed(g.replay)
        del g
        best = min(ms, ms_eager)
        return {**base, "value": round(kv_bytes / (best * 1e-3) / 1e9, 1), "unit": "GB/s",
                "ms_per_call": round(best, 4), "graph_ms_per_call": round(ms, 4),
                "eager_ms_per_call": round(ms_eager, 4), "host_ms_per_call": round(host, 4), "collective": "none",
                "timing": "the faster of CUDA-graph replays and eager calls back to back", "parity": parity}

    peer = lambda: adist.sharded_gqa_decode(q, k, v, exchange=exchange, **kw)  # noqa: E731
    fused = lambda: adist.sharded_gqa_decode(q, k, v, exchange=exchange, fused=True, **kw)  # noqa: E731
    nccl = lambda: adist.sharded_gqa_decode(q, k, v, **kw)  # noqa: E731
    parity = {"peer": _parity(peer(), ref, world, device), "fused": _parity(fused(), ref, world, device),
              "nccl": _parity(nccl(), ref, world, device)}
    ms_eager, host = timed(peer)
    ms_fused_eager, host_fused = timed(fused)
    po, lse = ops.gqa_decode_partial(q, k, v, **kw)
    ms_decode, _ = timed(lambda: ops.gqa_decode_partial(q, k, v, **kw))
    ms_exchange, host_exchange = timed(lambda: exchange.merge(po, lse, q.dtype))
    g = in_graph(peer)
    ms, _ = timed(g.replay)
    del g
    g = in_graph(fused)
    ms_fused, _ = timed(g.replay)
    del g
    ms_nccl, _ = timed(nccl)
    torch.cuda.synchronize(device)
    exchange.close()
    # consecutive eager calls overlap each call's decode with the previous call's
    # exchange (programmatic dependent launch) while graph replays serialise at
    # graph boundaries: the fastest form is the call's time, every one is listed
    best, how = min((ms, "CUDA-graph replays of the partial decode + peer exchange kernel"),
                    (ms_eager, "eager calls back to back of the partial decode + peer exchange kernel"),
                    (ms_fused, "CUDA-graph replays of the decode with the exchange fused in"),
                    (ms_fused_eager, "eager calls back to back of the decode with the exchange fused in"))
    return {**base, "value": round(kv_bytes / (best * 1e-3) / 1e9, 1), "unit": "GB/s",
            "ms_per_call": round(best, 4), "graph_ms_per_call": round(min(ms, ms_fused), 4),
            "timing": f"{how}, the fastest of four forms",
            "collective": "NVLink peer memory over CUDA IPC buffers: the exchange fused into the decode kernel "
                          "(per-pair flags), or a separate exchange + merge kernel (one CTA per peer)",
            "breakdown_ms": {"eager_call": round(ms_eager, 4), "host_issue_per_eager_call": round(host, 4),
                             "graph_call": round(ms, 4),
                             "fused_eager_call": round(ms_fused_eager, 4), "fused_graph_call": round(ms_fused, 4),
                             "host_issue_per_fused_call": round(host_fused, 4),
                             "partial_decode": round(ms_decode, 4), "exchange_merge": round(ms_exchange, 4),
                             "host_issue_per_exchange": round(host_exchange, 4)},
            "nccl_all_gather_path": {"value": round(kv_bytes / (ms_nccl * 1e-3) / 1e9, 1),
                                     "ms_per_call": round(ms_nccl, 4), "timing": "eager"},
            "parity": parity}


def run_fmha_secondary(args, world, device, peaks, only=None) -> dict:
    """Configs 3 and 4 on the tensor-core kernels (replicas: each rank its own batch)."""
    from aicas_b200 import _native

    caps = _native.capabilities()
    out = {}
    if only in (None, "prefill"):
        if not caps & _native.CAP_PREFILL_TCGEN05:
            out["prefill_cfg4"] = {"unavailable": "tcgen05 prefill kernel not built in this library"}
        else:
            out["prefill_cfg4"] = time_prefill(args, world, device, peaks)
    if only in (None, "vit"):
        if not caps & _native.CAP_VARLEN_TCGEN05:
            out["vit_cfg3"] = {"unavailable": "tcgen05 varlen kernel not built in this library"}
        else:
            out["vit_cfg3"] = time_varlen(args, world, device, peaks)
        out["vision_rope_cfg3"] = time_vision_rope(args, world, device, peaks)
        if caps & _native.CAP_VISION_QKV:
            out["vision_qkv_cfg3"] = time_vision_qkv(args, world, device, peaks)
    return out


def time_vision_qkv(args, world, device, peaks) -> dict:
    """The vision attention's packed projection + split + RoPE at config 3's
    token count (hidden 1024, 16 heads of 64): one tensor-core kernel
    (aicas_vision_qkv_rope) against HF's path on the same tensors (nn.Linear
    through cuBLAS, then apply_rotary_pos_emb_vision) and against cuBLAS
    followed by the one-kernel RoPE."""
    from transformers.models.qwen3_vl.modeling_qwen3_vl import apply_rotary_pos_emb_vision

    from aicas_b200 import ops
    from aicas_b200 import workloads as wl

    _, _, _, cu, _ = wl.cfg3_varlen(seed=0, device=device)
    T, K, H = int(cu[-1]), 1024, 16
    g = torch.Generator(device=device).manual_seed(0)
    x = torch.randn(T, K, device=device, generator=g).to(torch.bfloat16)
    w = (torch.randn(3 * H * 64, K, device=device, generator=g) / K ** 0.5).to(torch.bfloat16)
    b = (0.1 * torch.randn(3 * H * 64, device=device, generator=g)).to(torch.bfloat16)
    emb = torch.randn(T, 32, device=device, generator=g).repeat(1, 2)
    cos, sin = emb.cos(), emb.sin()

    def hf():
        qkv = torch.nn.functional.linear(x, w, b).view(T, 3, H, 64)
        return apply_rotary_pos_emb_vision(qkv[:, 0], qkv[:, 1], cos, sin)

    def cublas_then_rope():
        qkv = torch.nn.functional.linear(x, w, b).view(T, 3, H, 64)
        return ops.vision_rope(qkv[:, 0], qkv[:, 1], cos, sin)

    st = {}
    ms = _time_calls(lambda: ops.vision_qkv_rope(x, w, b, cos, sin, H), 20, 3, world, device, st)
    gemm_ms = _time_calls(lambda: torch.nn.functional.linear(x, w, b), 20, 3, world, device)
    hf_ms = _time_calls(hf, 10, 3, world, device)
    split_ms = _time_calls(cublas_then_rope, 10, 3, world, device)
    flops = 2 * T * 3 * H * 64 * K
    tf = flops / (ms * 1e-3) / 1e12
    return {"value": round(world * tf, 1), "unit": "TFLOP/s", "ms_per_call": round(ms, 4),
            "median_ms_per_call": round(st["median_ms"], 4), "per_gpu_tflops": round(tf, 1),
            "frac_of_bf16_peak": round(tf / peaks["bf16_tflops"], 4), "flops_per_call": flops,
            "cublas_linear_alone_ms": round(gemm_ms, 4),
            "cublas_linear_tflops": round(flops / (gemm_ms * 1e-3) / 1e12, 1),
            "hf_path_ms": round(hf_ms, 4), "cublas_then_fused_rope_ms": round(split_ms, 4),
            "speedup_vs_hf_path": round(hf_ms / ms, 2),
            "speedup_vs_cublas_then_fused_rope": round(split_ms / ms, 2),
            "config": f"T={T} patches, x [T, 1024] bf16, W [3072, 1024], bias, 16 heads of 64, fp32 cos/sin",
            "scaling": "weak (replicas)"}


def time_vision_rope(args, world, device, peaks) -> dict:
    """The vision attention's RoPE of q and k at config 3's token count
    (views of the packed qkv projection, fp32 cos/sin): the fused kernel
    against Hugging Face's apply_rotary_pos_emb_vision on the same tensors."""
    from transformers.models.qwen3_vl.modeling_qwen3_vl import apply_rotary_pos_emb_vision

    from aicas_b200 import ops
    from aicas_b200 import workloads as wl

    _, _, _, cu, _ = wl.cfg3_varlen(seed=0, device=device)
    T, H, D = int(cu[-1]), 16, 64
    g = torch.Generator(device=device).manual_seed(0)
    qkv = torch.randn(T, 3, H, D, device=device, generator=g).to(torch.bfloat16)
    emb = torch.randn(T, D // 2, device=device, generator=g).repeat(1, 2)
    cos, sin = emb.cos(), emb.sin()
    q, k = qkv[:, 0], qkv[:, 1]
    ms = _time_calls(lambda: ops.vision_rope(q, k, cos, sin), 20, 3, world, device)
    hf_ms = _time_calls(lambda: apply_rotary_pos_emb_vision(q, k, cos, sin), 10, 3, world, device)
    nbytes = 2 * 2 * T * H * D * 2 + 2 * T * D * 4  # q, k read + written (bf16), cos/sin read (fp32)
    gbs = nbytes / (ms * 1e-3) / 1e9
    return {"value": round(world * gbs, 1), "unit": "GB/s", "ms_per_call": round(ms, 4),
            "frac_of_hbm": round(gbs / peaks["hbm_gbs"], 4), "bytes_per_call": nbytes,
            "hf_eager_ms_per_call": round(hf_ms, 4), "speedup_vs_hf": round(hf_ms / ms, 2),
            "config": f"T={T} patches, H16 D64, bf16 q/k views of the packed qkv, fp32 cos/sin",
            "scaling": "weak (replicas)"}


_FLUSH: dict = {}


def _time_calls(fn, iters, warmup, world, device, stats: dict | None = None) -> float:
    """Mean device time of one call (ms), each call timed alone with CUDA events
    after a 256 MiB write that evicts L2 (larger than its 126 MB); max over
    ranks.  ``stats`` receives the median too."""
    flush = _FLUSH.get(device)
    if flush is None:
        flush = _FLUSH[device] = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    for _ in range(warmup):
        fn()
    barrier(world, device)
    times = []
    for _ in range(iters):
        flush.zero_()
        st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        st.record()
        fn()
        en.record()
        en.synchronize()
        times.append(st.elapsed_time(en))
    torch.cuda.synchronize(device)
    times.sort()
    if stats is not None:
        stats["median_ms"] = max_over_ranks(times[len(times) // 2], world, device)
    return max_over_ranks(sum(times) / len(times), world, device)


def time_prefill(args, world, device, peaks) -> dict:
    import aicas_b200 as ab
    from aicas_b200 import workloads as wl

    q, k, v = wl.cfg4_prefill(seed=0, device=device)
    flops = 2 * 8 * 16 * 2048 * 2048 * 128  # causal half of 4*S^2*D per (b, head)
    st = {}
    ms = _time_calls(lambda: ab.gqa_flash_attention(q, k, v, causal=True, sm_scale=wl.SCALE_TEXT,
                                                    num_key_value_groups=2), 20, 3, world, device, st)
    tf = flops / (ms * 1e-3) / 1e12
    return {"value": round(world * tf, 1), "unit": "TFLOP/s", "ms_per_call": round(ms, 4),
            "median_ms_per_call": round(st["median_ms"], 4), "per_gpu_tflops": round(tf, 1),
            "frac_of_bf16_peak": round(tf / peaks["bf16_tflops"], 4), "flops_per_call": flops,
            "config": "B8 S2048 Hq16 Hkv8 D128 causal, MRoPE-rotated q/k", "scaling": "weak (replicas)"}


def time_varlen(args, world, device, peaks) -> dict:
    import aicas_b200 as ab
    from aicas_b200 import workloads as wl

    q, k, v, cu, lens = wl.cfg3_varlen(seed=0, device=device)
    flops = sum(4 * n * n * 64 * 16 for n in lens)
    st = {}
    ms = _time_calls(lambda: ab.varlen_flash_attention(q, k, v, cu_seq_lens_q=cu, cu_seq_lens_k=cu,
                                                       sm_scale=wl.SCALE_VIT), 20, 3, world, device, st)
    tf = flops / (ms * 1e-3) / 1e12
    return {"value": round(world * tf, 1), "unit": "TFLOP/s", "ms_per_call": round(ms, 4),
            "median_ms_per_call": round(st["median_ms"], 4), "per_gpu_tflops": round(tf, 1),
            "frac_of_bf16_peak": round(tf / peaks["bf16_tflops"], 4), "flops_per_call": flops,
            "config": f"32 images, grids U[16,64]^2, T={int(cu[-1])}, H16 D64, non-causal", "scaling": "weak (replicas)"}


def run_products(args, world, device, peaks) -> dict:
    """The weight-streaming side of one batch-8 decode step of Qwen3-VL-2B on
    aicas_decode_linear, captured in one CUDA graph: 28 layers x (RMSNorm +
    q/k/v, o_proj + residual, RMSNorm + gate/up + SiLU*up, down_proj +
    residual) with distinct random weights per layer, then RMSNorm + the LM
    head.  Weights (3.44 GB a step) are far larger than L2, so every step
    streams them from HBM; achieved = weight bytes / step time."""
    from aicas_b200 import ops

    R, H, I, V, L = 8, 2048, 6144, 151936, LAYERS
    g = torch.Generator(device=device).manual_seed(0)

    def w(n, k):
        return (torch.randn(n, k, device=device, generator=g) / k ** 0.5).to(torch.bfloat16)

    layers = [(w(2048, H), w(1024, H), w(1024, H), w(H, 2048), w(I, H), w(I, H), w(H, I)) for _ in range(L)]
    lm = w(V, H)
    nw = (1 + 0.1 * torch.randn(H, device=device, generator=g)).to(torch.bfloat16)
    x0 = torch.randn(R, H, device=device, generator=g).to(torch.bfloat16)
    x, ss = x0.clone(), torch.zeros(R, device=device)
    wbytes = sum(t.numel() * 2 for lw in layers for t in lw) + lm.numel() * 2

    def step():
        x.copy_(x0)
        for i, (wq, wk, wv, wo, wg, wu, wd) in enumerate(layers):
            q, _, _ = ops.decode_linear(x, (wq, wk, wv), norm_weight=nw, x_sumsq=ss if i else None)
            ops.decode_linear(q, wo, residual=x, out=x, sumsq_out=ss)
            h = ops.decode_linear(x, (wg, wu), norm_weight=nw, x_sumsq=ss, swiglu=True)
            ops.decode_linear(h, wd, residual=x, out=x, sumsq_out=ss)
        return ops.decode_linear(x, lm, norm_weight=nw, x_sumsq=ss)

    s = torch.cuda.Stream(device)
    s.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(s):
        step()
    torch.cuda.current_stream(device).wait_stream(s)
    torch.cuda.synchronize(device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        step()
    ms = _time_calls(graph.replay, 10, 3, world, device)
    lm_ms = _time_calls(lambda: ops.decode_linear(x, lm, norm_weight=nw, x_sumsq=ss), 10, 3, world, device)
    del graph
    gbs = wbytes / (ms * 1e-3) / 1e9
    lm_gbs = lm.numel() * 2 / (lm_ms * 1e-3) / 1e9
    return {"value": round(world * gbs, 1), "unit": "GB/s", "ms_per_step": round(ms, 4),
            "per_gpu_gbs": round(gbs, 1), "frac_of_hbm": round(gbs / peaks["hbm_gbs"], 4),
            "weight_bytes_per_step": wbytes, "gpu_launches_per_step": 4 * L + 1,
            "lm_head": {"ms": round(lm_ms, 4), "gbs": round(lm_gbs, 1),
                        "frac_of_hbm": round(lm_gbs / peaks["hbm_gbs"], 4)},
            "config": "batch 8, Qwen3-VL-2B text decoder products (28 layers + LM head), bf16, random weights",
            "scaling": "weak (replicas)"}


# ------------------------------------------------------------------ the reference's own GPU kernels

REF_DIR = REPO / "baseline" / "_ref"


def install_reference(src: Path) -> dict:
    """``--install-reference SRC``: puts the reference's GPU code under
    baseline/_ref (git-ignored; it travels to the GPU box) for the ``refgpu``
    comparison leg.  The reference has no package metadata, so the offline pip
    install is tried first and, when it fails, its ``triton_qwen3vl`` package
    is copied unmodified; its native decode ops are built by its own setup
    script (dujunbaoV1/setup_native_cuda_ops.py) for sm_100a in a scratch copy
    (the source tree may be read-only).  The outcome is written to
    baseline/_ref/INSTALL.json."""
    import shutil
    import subprocess
    import tempfile

    REF_DIR.mkdir(parents=True, exist_ok=True)
    rec: dict = {}
    pip = subprocess.run([sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation",
                          "--find-links", "/opt/wheelhouse", "--target", str(REF_DIR), str(src)],
                         capture_output=True, text=True)
    rec["pip_install"] = {"rc": pip.returncode, "tail": (pip.stdout + pip.stderr).strip().splitlines()[-3:]}
    if not (REF_DIR / "triton_qwen3vl").exists():
        shutil.copytree(src / "triton_qwen3vl", REF_DIR / "triton_qwen3vl",
                        ignore=shutil.ignore_patterns("__pycache__"))
        rec["triton_qwen3vl"] = "copied unmodified (no package metadata for pip)"
    with tempfile.TemporaryDirectory() as tmp:
        work = Path(tmp) / "dujunbaoV1"
        work.mkdir()
        shutil.copy(src / "dujunbaoV1" / "setup_native_cuda_ops.py", work)
        shutil.copytree(src / "dujunbaoV1" / "native_cuda_ops", work / "native_cuda_ops",
                        ignore=shutil.ignore_patterns("__pycache__"))
        env = dict(os.environ, TORCH_CUDA_ARCH_LIST="10.0a", MAX_JOBS="8")
        b = subprocess.run([sys.executable, "setup_native_cuda_ops.py", "build_ext", "--inplace"], cwd=work,
                           capture_output=True, text=True, env=env)
        rec["native_cuda_ops_build"] = {"rc": b.returncode, "arch": "sm_100a (TORCH_CUDA_ARCH_LIST=10.0a)",
                                        "tail": (b.stdout + b.stderr).strip().splitlines()[-3:]}
        if b.returncode == 0:
            dst = REF_DIR / "native_cuda_ops"
            if dst.exists():
                shutil.rmtree(dst)
            shutil.copytree(work / "native_cuda_ops", dst, ignore=shutil.ignore_patterns("__pycache__", "*.o"))
    (REF_DIR / "INSTALL.json").write_text(json.dumps(rec, indent=1))
    return rec


def _load_ref_package(name: str, alias: str):
    """The reference package ``name`` from baseline/_ref under ``alias`` (this
    repository's own drop-in shim already owns the name triton_qwen3vl)."""
    import importlib.util

    root = REF_DIR / name
    if alias in sys.modules:
        return sys.modules[alias]
    spec = importlib.util.spec_from_file_location(alias, root / "__init__.py", submodule_search_locations=[str(root)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[alias] = mod
    spec.loader.exec_module(mod)
    return mod


def run_refgpu(args, world, device, peaks) -> dict:
    """The reference's own GPU kernels on this B200, beside this repository's
    on the same inputs (timing only; each call timed alone after an L2 flush):
    its Triton GQA decode (per-request calls over config 2's ragged valid
    prefixes, and one padded launch at their mean length), its Triton causal
    prefill (config 4) and varlen ViT attention (config 3), and its native fp16
    decode_q1_gqa kernel at the shapes it supports (head_dim 128, <= 1024
    cached tokens)."""
    import aicas_b200 as ab
    from aicas_b200 import workloads as wl

    if not (REF_DIR / "triton_qwen3vl").exists():
        return {"unavailable": "baseline/_ref has no reference install (run bench.py --install-reference SRC)"}
    ref = _load_ref_package("triton_qwen3vl", "ref_triton_qwen3vl")
    import ref_triton_qwen3vl.gqa_decode_attention as rdec  # noqa: F401  (submodules of the alias)
    out: dict = {"source": "baseline/_ref (the reference's triton_qwen3vl, unmodified)"}

    def pair(ref_ms, ours_ms, work, unit):
        return {"reference_ms": round(ref_ms, 4), "ours_ms": round(ours_ms, 4), "speedup": round(ref_ms / ours_ms, 2),
                "reference_" + unit: round(work / (ref_ms * 1e-3) / (1e9 if unit == "gbs" else 1e12), 1),
                "ours_" + unit: round(work / (ours_ms * 1e-3) / (1e9 if unit == "gbs" else 1e12), 1)}

    # ---- decode, config 2, one layer
    lengths = wl.cfg2_lengths(0)
    kc, vc = wl.cfg2_cache(B, L_CAP, 0, seed=0, device=device)
    q = wl.randn((B, 16, 1, 128), wl.generator(3, device), torch.bfloat16, device)
    lens_dev = lengths.to(device)
    layer_bytes = sum(2 * 8 * 128 * 2 * int(n) for n in lengths) + 2 * B * 16 * 128 * 2
    per_req = [(kc[b:b + 1, :, :int(n)].contiguous(), vc[b:b + 1, :, :int(n)].contiguous()) for b, n in enumerate(lengths)]

    def ref_loop():
        for b, (kb, vb) in enumerate(per_req):
            ref.gqa_decode_attention(q[b:b + 1], kb, vb, sm_scale=wl.SCALE_TEXT, num_key_value_groups=2)

    ours = lambda: ab.gqa_decode_attention(q, kc, vc, sm_scale=wl.SCALE_TEXT, num_key_value_groups=2,  # noqa: E731
                                           kv_lens=lens_dev)
    out["decode_cfg2_ragged"] = {**pair(_time_calls(ref_loop, 10, 3, world, device), _time_calls(ours, 20, 3, world, device),
                                        layer_bytes, "gbs"),
                                 "reference_call": "64 gqa_decode_attention calls, one per request over its valid prefix "
                                                   "(the reference has no length vector)",
                                 "ours_call": "one gqa_decode_attention call with kv_lens"}
    del per_req
    mean_len = int(lengths.float().mean())
    ku, vu = kc[:, :, :mean_len].contiguous(), vc[:, :, :mean_len].contiguous()
    uni_bytes = 2 * B * 8 * mean_len * 128 * 2 + 2 * B * 16 * 128 * 2
    out["decode_uniform_mean_len"] = {
        **pair(_time_calls(lambda: ref.gqa_decode_attention(q, ku, vu, sm_scale=wl.SCALE_TEXT, num_key_value_groups=2),
                           20, 3, world, device),
               _time_calls(lambda: ab.gqa_decode_attention(q, ku, vu, sm_scale=wl.SCALE_TEXT, num_key_value_groups=2),
                           20, 3, world, device), uni_bytes, "gbs"),
        "shape": f"B64 Hq16 Hkv8 L{mean_len} D128 bf16 (config 2's mean length, every request)"}
    del ku, vu, kc, vc

    # ---- prefill, config 4, and ViT varlen, config 3
    qp, kp, vp = wl.cfg4_prefill(seed=0, device=device)
    flops = 2 * 8 * 16 * 2048 * 2048 * 128
    out["prefill_cfg4"] = pair(
        _time_calls(lambda: ref.gqa_flash_attention(qp, kp, vp, causal=True, sm_scale=wl.SCALE_TEXT,
                                                    num_key_value_groups=2), 10, 3, world, device),
        _time_calls(lambda: ab.gqa_flash_attention(qp, kp, vp, causal=True, sm_scale=wl.SCALE_TEXT,
                                                   num_key_value_groups=2), 10, 3, world, device), flops, "tflops")
    del qp, kp, vp
    qv, kv_, vv, cu, seg = wl.cfg3_varlen(seed=0, device=device)
    vflops = sum(4 * n * n * 64 * 16 for n in seg)
    cache: dict = {}
    out["vit_cfg3"] = pair(
        _time_calls(lambda: ref.varlen_flash_attention(qv, kv_, vv, cu_seq_lens_q=cu, cu_seq_lens_k=cu,
                                                       sm_scale=wl.SCALE_VIT, max_length_q=max(seg),
                                                       max_length_k=max(seg), metadata_cache=cache), 10, 3, world, device),
        _time_calls(lambda: ab.varlen_flash_attention(qv, kv_, vv, cu_seq_lens_q=cu, cu_seq_lens_k=cu,
                                                      sm_scale=wl.SCALE_VIT), 10, 3, world, device), vflops, "tflops")
    del qv, kv_, vv

    # ---- the native fp16 decode kernel (dujunbaoV1/native_cuda_ops), at the shapes it takes
    if (REF_DIR / "native_cuda_ops").exists():
        try:
            nat_ops = _load_ref_package("native_cuda_ops", "ref_native_cuda_ops")
            avail = nat_ops.is_available()
        except Exception as exc:  # noqa: BLE001
            avail, nat_ops = False, None
            out["native_decode_q1_gqa"] = {"unavailable": f"import failed: {exc}"}
        if avail:
            g = wl.generator(4, device)
            qn = wl.randn((B, 16, 1, 128), g, torch.float16, device)
            kn = wl.randn((B, 8, 1024, 128), g, torch.float16, device)
            vn = wl.randn((B, 8, 1024, 128), g, torch.float16, device)
            q3 = qn[:, :, 0].contiguous()
            nb = 2 * B * 8 * 1024 * 128 * 2 + 2 * B * 16 * 128 * 2
            out["native_decode_q1_gqa"] = {
                **pair(_time_calls(lambda: nat_ops.decode_q1_gqa_forward(q3, kn, vn, 1024, wl.SCALE_TEXT), 10, 3, world,
                                   device),
                       _time_calls(lambda: ab.gqa_decode_attention(qn, kn, vn, sm_scale=wl.SCALE_TEXT,
                                                                   num_key_value_groups=2), 20, 3, world, device),
                       nb, "gbs"),
                "shape": "B64 Hq16 Hkv8 L1024 D128 fp16 (its head_dim and cache-length limits)"}
        elif "native_decode_q1_gqa" not in out:
            out["native_decode_q1_gqa"] = {"unavailable": f"extension did not load: {nat_ops.IMPORT_ERROR}"}
    else:
        out["native_decode_q1_gqa"] = {"unavailable": "not built in baseline/_ref"}
    torch.cuda.empty_cache()
    return out


# ------------------------------------------------------------------ CPU (reference) path


def run_generate(device) -> dict:
    """Configuration 4's end-to-end check: greedy generate of 128 tokens after
    a 2048-token image+text prompt, batch 8, on a random-init model with the
    Qwen3-VL-2B architecture, patched against SDPA on the same weights (host
    timed around device-synchronised generate calls; not a roofline)."""
    from aicas_b200 import integration

    r = integration.run_check(batch=8, seq_len=2048, max_new_tokens=128, grid_hw=(64, 100), device=device,
                              with_control=True)
    r["workload"] = "cfg4-e2e: random-init Qwen3-VL-2B-shaped model, 8 prompts x 2048 tokens (1600 image), greedy 128"
    r["speedup_vs_sdpa"] = r["patched"]["tokens_per_s"] / r["sdpa"]["tokens_per_s"]
    torch.cuda.empty_cache()
    return r


def cpu_decode_sample(target_s: float, max_layers: int = 100000) -> dict:
    """Times the reference's CPU path (oracle/reference_cpu.py) on whole config-2
    layers (all 64 requests) on the host cores, layer after layer of the step
    (each with its own inputs, the distinct layer caches in rotation, as the
    reference arm runs them); returns GB/s of the same metric."""
    from aicas_b200 import workloads as wl
    from oracle import reference_cpu as rc

    torch.set_num_threads(len(os.sched_getaffinity(0)))
    lengths = wl.cfg2_lengths(0)
    per_layer = step_bytes(lengths)["step"] / LAYERS
    caches = [wl.cfg2_cache(B, L_CAP, layer, seed=0) for layer in range(REF_DISTINCT_CACHES)]
    inputs = [wl.cfg2_step_inputs(lengths, layer, seed=0) for layer in range(LAYERS)]

    def layer_call(i):
        x, (kc, vc) = inputs[i % LAYERS], caches[i % REF_DISTINCT_CACHES]
        rc.decode_layer(x.q, x.k, x.v, x.cos, x.sin, kc, vc, x.positions, wl.SCALE_TEXT)

    layer_call(0)  # warm-up
    layers, t0 = 0, time.perf_counter()
    while layers < max_layers and (layers == 0 or time.perf_counter() - t0 < target_s):
        layer_call(layers)
        layers += 1
    dt = time.perf_counter() - t0
    return {"value": round(layers * per_layer / dt / 1e9, 3), "unit": "GB/s", "cores": torch.get_num_threads(),
            "kind": "port", "seconds": round(dt, 2),
            "sample": f"{layers} config-2 layer calls in step order (64 requests each: RoPE + append + per-request "
                      f"SDPA) on CPU, {REF_DISTINCT_CACHES} distinct layer caches in rotation"}


# distinct layer caches the reference arm rotates through: 4 x 1.07 GB of host
# memory (28 would be 30 GB); each layer reads 591 MB of valid K/V, so the
# rotation period (2.4 GB) is far larger than any CPU's last-level cache and
# the CPU gets no reuse from one layer to the next
REF_DISTINCT_CACHES = 4


def run_reference(args, world, rank) -> dict | None:
    """The reference's own CPU path (oracle/reference_cpu.py restates it; the
    reference is Python and cannot travel) on the host cores, on the same
    config-2 step: 28 layers, each with its own step inputs, over distinct
    layer caches.  Imports no native code."""
    if rank != 0:
        return None
    from aicas_b200 import workloads as wl
    from oracle import reference_cpu as rc

    torch.set_num_threads(os.cpu_count() or 1)
    lengths = wl.cfg2_lengths(0)
    per_layer = step_bytes(lengths)["step"] / LAYERS
    caches = [wl.cfg2_cache(B, L_CAP, layer, seed=0) for layer in range(REF_DISTINCT_CACHES)]
    inputs = [wl.cfg2_step_inputs(lengths, layer, seed=0) for layer in range(LAYERS)]

    def one_step():
        for layer, x in enumerate(inputs):
            kc, vc = caches[layer % REF_DISTINCT_CACHES]
            rc.decode_layer(x.q, x.k, x.v, x.cos, x.sin, kc, vc, x.positions, wl.SCALE_TEXT)

    for _ in range(args.warmup):
        one_step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        one_step()
    dt = time.perf_counter() - t0
    value = args.steps * LAYERS * per_layer / dt / 1e9
    sample = (f"one config-2 step per step: 28 layer calls (64 requests each: RoPE + cache append + per-request "
              f"SDPA, bf16) on CPU, each layer with its own inputs, {REF_DISTINCT_CACHES} distinct layer caches "
              "in rotation")
    return {
        "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(dt * 1e3 / args.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "impl": "reference",
        "config": cfg2_config(world),
        "execution": "reference CPU path (torch CPU operators), all host threads",
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": torch.get_num_threads(), "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# ------------------------------------------------------------------ main


class _JsonStdout:
    """Native libraries (NCCL prints its version at communicator set-up) write
    to file descriptor 1 directly; while the benchmark runs, descriptor 1 points
    at stderr, so the one JSON line is all that reaches stdout."""

    def __enter__(self):
        sys.stdout.flush()
        self._saved = os.dup(1)
        os.dup2(2, 1)
        return self

    def emit(self, line: dict) -> None:
        sys.stdout.flush()
        os.write(self._saved, (json.dumps(line) + "\n").encode())

    def __exit__(self, *exc):
        sys.stdout.flush()
        os.dup2(self._saved, 1)
        os.close(self._saved)


def main(argv=None) -> int:
    with _JsonStdout() as out:
        return _main(out, argv)


def _main(out: "_JsonStdout", argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-secondary", dest="secondary", action="store_false",
                    help="skip the tensor-core prefill / ViT measurements")
    ap.add_argument("--no-cpu-baseline", dest="cpu_baseline", action="store_false")
    ap.add_argument("--no-refgpu", dest="refgpu", action="store_false",
                    help="skip timing the reference's own GPU kernels beside ours (N=1 only)")
    ap.add_argument("--no-e2e", dest="e2e", action="store_false", help="skip the end-to-end host-buffer measurement")
    ap.add_argument("--no-generate", dest="generate", action="store_false",
                    help="skip the end-to-end greedy generate on the random-init Qwen3-VL-2B-shaped model")
    ap.add_argument("--only", choices=["decode", "split_kv", "prefill", "vit", "products", "generate", "refgpu"],
                    default=None, help="run one workload (profiling; refgpu: the reference's own GPU kernels beside ours)")
    ap.add_argument("--install-reference", type=Path, default=None, metavar="SRC",
                    help="install the reference checkout at SRC under baseline/_ref for --only refgpu, then exit")
    ap.add_argument("--layers", type=int, default=LAYERS, help="decode layers per step (28 = Qwen3-VL-2B)")
    args = ap.parse_args(argv)
    if args.install_reference is not None:
        out.emit({"install_reference": install_reference(args.install_reference.resolve())})
        return 0
    if args.warmup < 3:
        args.warmup = 3
    world, rank, local = dist_info()
    if world != args.gpus:
        log(f"note: --gpus {args.gpus} but WORLD_SIZE={world}; using WORLD_SIZE")

    if args.impl == "reference":
        line = run_reference(args, world, rank)
        if line is not None:
            out.emit(line)
        return 0

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1 and os.environ.get("AICAS_BENCH_NO_PIN") is None:
        pin_host_cores(local, world)
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=180))
    peaks, src = load_peaks()
    from aicas_b200 import _native

    _native.lib()  # loud failure if the library is missing
    only = args.only
    result = {}
    if only in (None, "decode"):
        result["decode"] = run_decode(args, world, rank, device, peaks, src)
    if only in (None, "split_kv"):
        result["split_kv_cfg5"] = run_split_kv(args, world, rank, device)
    if args.secondary and only in (None, "prefill", "vit"):
        result.update(run_fmha_secondary(args, world, device, peaks, only))
    if args.secondary and only in (None, "products"):
        result["decode_products"] = run_products(args, world, device, peaks)
    if only == "refgpu" or (only is None and world == 1 and args.refgpu):
        result["reference_gpu"] = run_refgpu(args, world, device, peaks)
    if world == 1 and ((args.generate and only is None) or only == "generate"):
        result["generate_cfg4"] = run_generate(device)
    line = None
    if rank == 0:
        line = {"metric": METRIC, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "higher_is_better": True, "vs_baseline": None, "dtype": "bf16", "data": "synthetic"}
        dec = result.pop("decode", None)
        if dec is not None:
            line.update({"value": dec["value"], "unit": "GB/s", "ms_per_step": dec["ms_per_step"], "scaling": "weak",
                         "config": dec["config"], "execution": dec["execution"], "roofline": dec["roofline"],
                         "e2e": dec.get("e2e"),
                         "gpu_launches": dec["gpu_launches"], "clocks": dec["clocks"]})
        else:
            line.update({"value": None, "unit": None, "note": f"--only {only}: headline decode not run"})
        line.update(result)
    if rank == 0 and world == 1 and args.cpu_baseline and only in (None, "decode"):
        line["cpu_baseline"] = cpu_decode_sample(target_s=10.0)
    if world > 1:
        import torch.distributed as dist

        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    if line is not None:
        out.emit(line)
    sk = result.get("split_kv_cfg5", {}).get("parity")
    checks = ([sk] if "ok" in sk else list(sk.values())) if sk else []
    if not all(c["ok"] for c in checks):
        log(f"split-KV parity check FAILED: {sk}")
        return 1
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
