#!/usr/bin/env python3
"""Benchmark: IQ2_XXS matmul weight GB/s at M=1 (decode GEMV) on Llama-3-8B-shaped projections.

Workload (benchmark configuration 1, "batched decode GEMV", at M=1): the 7 projections of a
Llama-3-8B layer (q 4096x4096, k/v 4096x1024, o 4096x4096, gate/up 4096x14336, down 14336x4096;
K x N), IQ2_XXS weights with the benchmark block distribution, f32 N(0,1) activations, repeated
over 32 distinct layers (1.80 GB of packed weights, > 14x the 126 MB L2, so no step reads weights
from L2). Synthetic data.

  value    = packed weight bytes per step / device time per step, the step being all 224
             projections in one batched call (iq2_matmul_grouped; CUDA events on the launch
             stream around K back-to-back replays of a CUDA graph holding one step; inputs resident)
  per_call = the same step as 224 reference-shaped iq2_xxs_matmul calls
  e2e      = the same step through the public API (the one grouped call) with every projection's x
             copied host->device from pinned memory and every output device->host inside the timed
             region, pipelined as a serving loop runs it (copy streams, two buffer sets: step k's
             copies overlap steps k-1 / k+1's compute); e2e.per_call: the same with the 224
             reference-shaped calls
  roofline: the dominant kernel of the timed region (the step's one grouped GEMV launch; its
            duration bounded by the step time) against measured HBM, with ncu DRAM traffic;
            roofline.single_call: the decode GEMV of one 4096x14336 gate/up projection timed alone
            with CUDA events (64 distinct matrices in rotation, > L2).
  cpu_baseline: the reference's own kernels (compiled from source for the host, all threads) on
            a bounded sample of the same workload.

--gpus N > 1 (launched by torchrun, one rank per GPU): every projection is column-sharded over the
N ranks (rank r holds weight rows [r*N/g, (r+1)*N/g), a contiguous slice), and every rank ends
with the full outputs: by default (--exchange fused) the decode GEMV stores each output into
every rank's copy over NVLink (outputs in the communicator's symmetric region; one kernel per
call), or (--exchange nccl) through NCCL all-gathers (one per step in the batched call, one per
projection in the per-call path) -- strong scaling of the same workload; value = whole-job weight
bytes/s, the max over ranks of the device time.

--impl reference: the reference's own kernels on the host cores (see above), same metric.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

METRIC = "IQ2_XXS matmul: weight GB/s at M=1, TFLOPS at M=2048, % of roofline"
LAYERS = 32
# packed weight bytes of the launch captured in profiles/gemv_kernel_grouped_m1.md (8 layers)
GROUPED_PROFILE_BYTES = 8 * 56_229_888


def _peaks():
    try:
        return json.loads((ROOT / "MEASURED_PEAKS.json").read_text()), "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


class ClockSampler:
    """SM clocks and throttle reasons of one GPU, sampled every 10 ms while active: through NVML (the
    device opened before the timed region starts, found by the CUDA device's UUID), else nvidia-smi
    every 100 ms (which takes about a second to produce its first sample)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, device: torch.device):
        self.device = device
        self.proc = self.file = self.thread = None
        self.nvml = None
        self.rows = []  # (sm_mhz, sm_max_mhz, [reason names])
        self.stop = False

    def _open_nvml(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(self.device).uuid)
            h = pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            bits = (pynvml.nvmlClocksEventReasonHwSlowdown, pynvml.nvmlClocksEventReasonHwThermalSlowdown,
                    pynvml.nvmlClocksEventReasonSwThermalSlowdown, pynvml.nvmlClocksEventReasonSwPowerCap)
            smax = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
            return pynvml, h, bits, smax
        except Exception:
            return None

    def _sample_nvml(self):
        pynvml, h, bits, smax = self.nvml
        while not self.stop:
            try:
                sm = float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
                r = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                self.rows.append((sm, smax, [n for n, bit in zip(self.NAMES, bits) if r & bit]))
            except Exception:
                pass
            time.sleep(0.01)

    def __enter__(self):
        import threading
        self.nvml = self._open_nvml()
        if self.nvml is not None:
            self.thread = threading.Thread(target=self._sample_nvml, daemon=True)
            self.thread.start()
            return self
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.device.index}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=self.file, stderr=subprocess.DEVNULL)
        except FileNotFoundError:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.stop = True
        if self.thread is not None:
            self.thread.join(timeout=5)
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if self.nvml is None:
            if self.proc is None:
                return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
            self.file.flush()
            for r in [r.split(",") for r in Path(self.file.name).read_text().strip().splitlines() if r.count(",") >= 8]:
                sm, smax = r[1].strip(), r[2].strip()
                if sm.replace(".", "").isdigit() and smax.replace(".", "").isdigit():
                    self.rows.append((float(sm), float(smax),
                                      [n for i, n in enumerate(self.NAMES) if r[5 + i].strip().lower() == "active"]))
            os.unlink(self.file.name)
        rows = self.rows
        return {"sm_mhz": statistics.median(r[0] for r in rows) if rows else None,
                "sm_max_mhz": max(r[1] for r in rows) if rows else None,
                "reasons": sorted({n for r in rows for n in r[2]}), "samples": len(rows),
                "source": "nvml" if self.nvml is not None else "nvidia-smi"}


# ---------------------------------------------------------------------------------------- ours
class Workload:
    """Device-resident weights, inputs, outputs and workspaces of one step, optionally sharded.
    The x and output buffers come in sets (add_buffer_set): the pipelined end-to-end run alternates
    two, so that one step's copies overlap another step's compute."""

    def __init__(self, m: int, layers: int, rank: int, world: int, device: torch.device, comm=None):
        from candelora_metal_kernels_b200 import grouped_workspace_bytes, synth, workspace_bytes
        from candelora_metal_kernels_b200.sharded import sharded_workspace_bytes
        self.m, self.device, self.rank, self.world, self.comm = m, device, rank, world, comm
        self.weight_bytes = 0        # whole-job packed bytes per step
        x_elems = out_elems = 0
        specs = []
        for layer in range(layers):
            for pi, (name, k, n) in enumerate(synth.LLAMA3_8B_PROJECTIONS):
                specs.append((layer, pi, name, k, n, n // world, x_elems, out_elems))
                x_elems += m * k
                out_elems += m * n  # every rank ends with the full outputs
                self.weight_bytes += synth.packed_bytes(n, k)
        self.x_elems, self.out_elems = x_elems, out_elems
        self.fused = comm is not None and comm.has_symmetric and m <= 16
        self.x_host = torch.empty(x_elems, dtype=torch.float32, pin_memory=True)
        self.out_host = torch.empty(out_elems, dtype=torch.float32, pin_memory=True)
        ws_cache = {}
        self.specs = []  # (qs, sc, n, k, x_off, out_off, ws, name): qs/sc = this rank's row slice
        for (layer, pi, name, k, n, n_loc, xo, oo) in specs:
            seed = layer * 16 + pi
            qs, sc = synth.iq2xxs_weights(n, k, seed, device=device, row_begin=rank * n_loc,
                                          row_end=(rank + 1) * n_loc)
            x = synth.activations(m, k, seed=10_000 + seed)
            self.x_host[xo:xo + m * k].copy_(x.reshape(-1))
            key = (n, k)
            if key not in ws_cache:  # one workspace per shape is enough: calls are stream-ordered
                need = (workspace_bytes(m, n, k, torch.float32) if world == 1
                        else sharded_workspace_bytes(comm, [(torch.empty(m, k, device=device), qs, sc, n, k)]))
                ws_cache[key] = torch.empty(need, dtype=torch.uint8, device=device)
            self.specs.append((qs, sc, n, k, xo, oo, ws_cache[key], name))
        self.sets = []
        self.add_buffer_set()
        self.x_dev, self.out_dev = self.sets[0]["x"], self.sets[0]["out"]
        self.calls, self.problems = self.sets[0]["calls"], self.sets[0]["problems"]
        need = (grouped_workspace_bytes(self.problems) if world == 1
                else sharded_workspace_bytes(comm, self.problems))
        self.grouped_ws = torch.empty(max(need, 1), dtype=torch.uint8, device=device)

    def add_buffer_set(self):
        """Another x buffer and output buffer (outputs in the symmetric region when there is one),
        with the step's calls bound to them; returns its index."""
        comm, m = self.comm, self.m
        x_dev = torch.empty(self.x_elems, dtype=torch.float32, device=self.device)
        out_dev = (comm.symmetric_empty(self.out_elems) if comm is not None and comm.has_symmetric
                   else torch.empty(self.out_elems, dtype=torch.float32, device=self.device))
        x_dev.copy_(self.x_host)
        calls = []  # (x_view, qs, sc, n, k, out_view, ws, name)
        for (qs, sc, n, k, xo, oo, ws, name) in self.specs:
            calls.append((x_dev[xo:xo + m * k].view(m, k), qs, sc, n, k, out_dev[oo:oo + m * n].view(m, n), ws, name))
        problems = [(x, qs, sc, n, k, out) for (x, qs, sc, n, k, out, _, _) in calls]
        self.sets.append({"x": x_dev, "out": out_dev, "calls": calls, "problems": problems})
        return len(self.sets) - 1

    def step(self, grouped: bool = False, b: int = 0):
        """One step on buffer set b: every projection through the per-projection call
        (iq2_xxs_matmul, the reference-shaped call; column-sharded with one all-gather per call on
        N > 1 GPUs), or all of them through one grouped call (one all-gather per step on N > 1 GPUs)."""
        from candelora_metal_kernels_b200 import iq2_matmul_grouped, iq2_xxs_matmul
        from candelora_metal_kernels_b200.sharded import iq2_matmul_grouped_sharded, iq2_matmul_sharded
        calls, problems = self.sets[b]["calls"], self.sets[b]["problems"]
        if self.world == 1:
            if grouped:
                iq2_matmul_grouped(problems, workspace=self.grouped_ws)
            else:
                for (x, qs, sc, n, k, out, ws, _) in calls:
                    iq2_xxs_matmul(x, qs, sc, n, k, out=out, workspace=ws)
        elif grouped:
            iq2_matmul_grouped_sharded(self.comm, problems, workspace=self.grouped_ws)
        else:
            for (x, qs, sc, n, k, out, ws, _) in calls:
                iq2_matmul_sharded(self.comm, x, qs, sc, n, k, out=out, workspace=ws)

    def launches_per_step(self, grouped: bool = False) -> int:
        """This library's kernels per step (NCCL's all-gather kernels not counted): a GEMV launch,
        plus the x-limb prep when the call has a workspace for it (per 256 projections when
        grouped), plus with the NCCL exchange on N > 1 GPUs the scatter kernel (not needed for one
        projection at m = 1). The fused exchange adds no launch."""
        from candelora_metal_kernels_b200 import workspace_bytes
        scatter = self.world > 1 and not self.fused
        if grouped:
            return 2 * ((len(self.calls) + 255) // 256) + (1 if scatter else 0)
        total = 0
        for (_, _, _, n, k, _, _, _) in self.calls:
            total += 1 if workspace_bytes(self.m, n // self.world, k, torch.float32) == 0 else 2
            if scatter and self.m > 1:
                total += 1
        return total


def _time_graph(graph, steps: int, stream) -> float:
    """Device time of `steps` replays, events recorded on the stream the replays run on."""
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        start.record(stream)
        for _ in range(steps):
            graph.replay()
        end.record(stream)
    end.synchronize()
    return start.elapsed_time(end)


def run_ours(args, rank: int, world: int, local_rank: int):
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    import candelora_metal_kernels_b200 as c
    from candelora_metal_kernels_b200 import synth
    c._lib.load()
    dist = world > 1
    comm = None
    if dist:
        from candelora_metal_kernels_b200.sharded import Iq2Comm
        comm = Iq2Comm()  # the library's NCCL communicator; the NCCL process group carries its id
        if args.exchange == "fused":  # outputs here: the GEMV stores them into every rank
            step_out = args.m * args.layers * sum(n for (_, _, n) in synth.LLAMA3_8B_PROJECTIONS) * 4
            # two output sets (the pipelined end-to-end run) + the configuration 3/4 decode outputs
            comm.alloc_symmetric(2 * step_out + (32 << 20))
    wl = Workload(args.m, args.layers, rank, world, device, comm)
    stream = torch.cuda.Stream(device)
    torch.cuda.synchronize()

    # warm-up (eager), then capture one step
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            wl.step()
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        wl.step()
    # the same step through one grouped call
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            wl.step(grouped=True)
    stream.synchronize()
    ggraph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(ggraph, stream=stream):
        wl.step(grouped=True)
    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            ggraph.replay()
    torch.cuda.synchronize()

    def max_over_ranks(ms: float) -> float:
        if not dist:
            return ms
        t = torch.tensor([ms], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())

    # ---- timed region (value): K steps of the batched call, barrier + sync on both sides, max over ranks
    if dist:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    with ClockSampler(device) as clocks:
        ms = _time_graph(ggraph, args.steps, stream)
        # keep sampling a little longer when the timed region is shorter than a sample period
        # (every rank replays the same number of times: the step holds collectives)
        extra = torch.tensor([max(1, int(args.steps * 300 / max(ms, 1e-3))) if ms < 300 else 0], device=device)
        if dist:
            torch.distributed.all_reduce(extra, op=torch.distributed.ReduceOp.MAX)
        if int(extra.item()) > 0:
            _time_graph(ggraph, int(extra.item()), stream)
    torch.cuda.synchronize()
    if dist:
        torch.distributed.barrier()
    ms = max_over_ranks(ms)
    ms_per_step = ms / args.steps
    value = wl.weight_bytes / (ms_per_step * 1e-3) / 1e9

    # ---- the same step as 224 reference-shaped per-projection calls, inputs resident
    with torch.cuda.stream(stream):
        for _ in range(3):
            graph.replay()
    if dist:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    pms = max_over_ranks(_time_graph(graph, args.steps, stream))
    per_call = {"value": round(wl.weight_bytes / (pms / args.steps * 1e-3) / 1e9, 2), "unit": "GB/s",
                "ms_per_step": round(pms / args.steps, 4),
                "path": ("224 iq2_xxs_matmul calls per step" if not dist else
                         "224 column-sharded calls per step, " + _exchange_words(wl, "each")),
                "gpu_launches": wl.launches_per_step(False) * args.steps}

    # ---- end to end: host x -> device, the step through the public API, outputs -> host; the
    # ---- same step as `value` (one grouped call) and, beside it, as 224 reference-shaped calls
    # Pipelined as a serving loop runs it: step k's upload and download go on two copy streams and
    # overlap other steps' compute, with two x and output buffers (graph b = k % 2 is the step on
    # buffer set b). Every step's copies are inside the timed region: the uploads start after the
    # start event and the end event follows the last download.
    wl.add_buffer_set()
    cin, cout = torch.cuda.Stream(device), torch.cuda.Stream(device)

    def capture(grouped: bool, b: int):
        with torch.cuda.stream(stream):
            for _ in range(2):
                wl.step(grouped=grouped, b=b)
        stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            wl.step(grouped=grouped, b=b)
        return g

    ggraph1 = capture(True, 1)
    graph1 = capture(False, 1)

    def e2e_run(graphs) -> float:
        def run(nsteps, start_ev):
            comp, down = [None, None], [None, None]
            for k in range(nsteps):
                b = k % 2
                bs = wl.sets[b]
                with torch.cuda.stream(cin):
                    cin.wait_event(start_ev)
                    if comp[b] is not None:
                        cin.wait_event(comp[b])  # the compute that last read this x buffer
                    bs["x"].copy_(wl.x_host, non_blocking=True)
                    up = torch.cuda.Event()
                    up.record(cin)
                with torch.cuda.stream(stream):
                    stream.wait_event(up)
                    if down[b] is not None:
                        stream.wait_event(down[b])  # the download that last read this output buffer
                    graphs[b].replay()
                    comp[b] = torch.cuda.Event()
                    comp[b].record(stream)
                with torch.cuda.stream(cout):
                    cout.wait_event(comp[b])
                    wl.out_host.copy_(bs["out"], non_blocking=True)
                    down[b] = torch.cuda.Event()
                    down[b].record(cout)
            for ev in down:
                if ev is not None:
                    stream.wait_event(ev)

        with torch.cuda.stream(stream):
            w0 = torch.cuda.Event()
            w0.record(stream)
        run(4, w0)
        stream.synchronize()
        if dist:
            torch.distributed.barrier()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            s0.record(stream)
        run(args.steps, s0)
        with torch.cuda.stream(stream):
            s1.record(stream)
        s1.synchronize()
        torch.cuda.synchronize()
        return max_over_ranks(s0.elapsed_time(s1))

    e2e_ms = e2e_run([ggraph, ggraph1])
    e2e_value = wl.weight_bytes / (e2e_ms / args.steps * 1e-3) / 1e9
    e2e_pc_ms = e2e_run([graph, graph1])
    e2e_per_call = {"value": round(wl.weight_bytes / (e2e_pc_ms / args.steps * 1e-3) / 1e9, 2), "unit": "GB/s",
                    "ms_per_step": round(e2e_pc_ms / args.steps, 4),
                    "path": ("pinned host x -> device, 224 reference-shaped iq2_matmul calls"
                             + (" (column-sharded, " + _exchange_words(wl, "each") + ")" if dist else "")
                             + ", outputs -> pinned host; pipelined: copy streams, two buffer sets")}

    # ---- roofline of the dominant kernel: 4096x14336 decode GEMV alone, 64 matrices in rotation
    peaks, peak_src = _peaks()
    roof = None
    if rank == 0:
        # single-GPU calls on this rank's rows (all of them on one GPU)
        big = [cl for cl in wl.calls if cl[7] in ("gate", "up")]
        n_loc, k = big[0][3] // world, big[0][4]
        out1 = torch.empty(args.m, n_loc, device=device)
        ws1 = torch.empty(c.workspace_bytes(args.m, n_loc, k, torch.float32), dtype=torch.uint8, device=device)
        g2 = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g2, stream=stream):
            for (x, qs, sc, n, k, out, ws, _) in big:
                c.iq2_xxs_matmul(x, qs, sc, n // world, k, out=out1, workspace=ws1)
        with torch.cuda.stream(stream):
            for _ in range(3):
                g2.replay()
        reps = max(3, args.steps // 4)
        ms_big = _time_graph(g2, reps, stream)
        per_launch_ms = ms_big / (reps * len(big))
        bytes_per_launch = synth.packed_bytes(n_loc, k)
        achieved = bytes_per_launch / (per_launch_ms * 1e-3) / 1e9
        single = {"kernel": f"gemv_kernel<1,1,0> (x limbs in-kernel), 4096x{n_loc} m=1, one launch per call",
                  "achieved": round(achieved, 1), "frac": round(achieved / peaks["hbm_gbs"], 4),
                  "us_per_launch": round(per_launch_ms * 1e3, 3), "algorithmic_bytes": bytes_per_launch,
                  "traffic": _ncu_traffic("gemv_kernel_4096x14336_m1.md", bytes_per_launch, bytes_per_launch)}
        # the kernel that dominates the timed region: the step's one grouped GEMV launch (this
        # rank's rows of all 224 projections); its duration is bounded by the step time, which
        # also holds the x-limb prep kernel (a few us)
        step_bytes = sum(synth.packed_bytes(n // world, k) for (_, _, _, n, k, _, _, _) in wl.calls)
        g_achieved = step_bytes / (ms_per_step * 1e-3) / 1e9
        roof = {"bound": "hbm", "kernel": "gemv_kernel<1,256,-1>: the step's projections in one launch (grouped)",
                "achieved": round(g_achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": round(g_achieved / peaks["hbm_gbs"], 4), "peak_source": peak_src,
                "us_per_launch": round(ms_per_step * 1e3, 2), "algorithmic_bytes": step_bytes,
                "traffic": _ncu_traffic("gemv_kernel_grouped_m1.md", step_bytes, GROUPED_PROFILE_BYTES),
                "single_call": single}
        del g2

    del graph, ggraph, graph1, ggraph1
    models = None
    if not args.no_models:
        models = {"forward": forward_bench(args, wl, device, stream, comm, dist),
                  "ffn70b": ffn70b_bench(args, device, stream, comm, rank, world, _peaks()[0])}
    if comm is not None:
        torch.cuda.synchronize()
        comm.close()
    line = None
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32 activations x IQ2_XXS weights (s32/f32 accumulate)",
            "data": "synthetic (seeded IQ2_XXS blocks with the benchmark distribution, N(0,1) f32 x)",
            "config": {"workload": "config1: Llama-3-8B projections q,k,v,o,gate,up,down x 32 layers, M=1",
                       "m": args.m, "layers": args.layers,
                       "weight_bytes_per_step": wl.weight_bytes,
                       "parallelism": (f"column-shard over {world} GPUs, " + _exchange_words(wl, "per call"))
                                      if world > 1 else "1 GPU",
                       "l2": "no flush needed: 1.80 GB of distinct weights per step vs 126 MB L2",
                       "step": ("the 224 projections in one iq2_matmul_grouped call" if world == 1 else
                                "the 224 projections column-sharded in one iq2_matmul_grouped_sharded call ("
                                + _exchange_words(wl, "per step") + ")"),
                       "timing": "CUDA events around K replays of a CUDA graph of one step"},
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": wl.x_host.numel() * 4,
                    "d2h_bytes_per_step": wl.out_host.numel() * 4,
                    "ms_per_step": round(e2e_ms / args.steps, 4),
                    "path": ("pinned host x -> device, the step's 224 projections through one "
                             + ("iq2_matmul_grouped call" if not dist else
                                "iq2_matmul_grouped_sharded call (" + _exchange_words(wl, "per step") + ")")
                             + ", outputs -> pinned host; pipelined: each step's upload and download on "
                               "copy streams overlap the neighbouring steps' compute (two x / output buffer sets)"),
                    "per_call": e2e_per_call},
            "gpu_launches": wl.launches_per_step(True) * args.steps,
            "per_call": per_call,
            "clocks": clocks.summary(),
            "roofline": roof,
        }
        if models is not None:
            line["config4_forward"] = models["forward"]
            line["config3_ffn70b"] = models["ffn70b"]
        if not args.no_gemm:
            line["gemm"] = gemm_bench(args, device, stream, peaks, peak_src)
        if not args.no_next_rows and world == 1:
            line["next_rows"] = next_rows_bench(args, device, stream, peaks, peak_src)
        if not args.no_config01 and world == 1:
            line.update(config01_bench(args, device, stream, peaks, peak_src))
        if not args.no_cpu_baseline and world == 1:
            line["cpu_baseline"] = cpu_baseline(args)
    return line


def _ncu_traffic(summary: str, bytes_per_launch: int, profiled_bytes: int):
    """DRAM bytes per launch from a committed ncu summary (profiles/<summary>), scaled from the
    captured launch (`profiled_bytes` of packed weights) to this one by the weight bytes each
    processes (the traffic is the weights streamed once, so it grows in proportion)."""
    p = ROOT / "profiles" / summary
    try:
        for line in p.read_text().splitlines():
            if line.startswith("dram_bytes_per_launch:"):
                return int(int(line.split(":")[1]) * bytes_per_launch / profiled_bytes)
    except Exception:
        pass
    return None


def _exchange_words(wl, per: str) -> str:
    return ("fused peer-memory all-gather in the GEMV epilogue, no NCCL call" if wl.fused
            else f"one NCCL all-gather {per}")


# ---------------------------------------------------------------------------------------- models
def forward_bench(args, wl, device, stream, comm, dist):
    """Benchmark configuration 4: the 32-layer Llama-3-8B linear stack as one forward pass, with
    a fixed dataflow (q, k, v, gate, up on x in one grouped call; o on q; down on up; the next
    layer's x = RMS-normalised down output), RMS-normalised N(0,1) input rows, M in {1, 32}
    (decode GEMV, tensor-core GEMM). Column-sharded over the ranks when N > 1. Device time per
    forward, max over ranks."""
    import candelora_metal_kernels_b200 as c
    from candelora_metal_kernels_b200 import synth
    from candelora_metal_kernels_b200.sharded import iq2_matmul_grouped_sharded
    layers = [wl.calls[i:i + 7] for i in range(0, len(wl.calls), 7)]
    res = {}
    for m in (1, 32):
        x0 = synth.activations(m, 4096, seed=4242, device=device, rms_normalize=True)
        sym = dist and comm.has_symmetric  # the sharded decode stores into every rank's copy
        outs = {name: (comm.symmetric_empty(m, n) if sym else torch.empty(m, n, device=device))
                for (_, _, _, n, _, _, _, name) in layers[0]}

        def matmuls(probs):
            if dist:
                iq2_matmul_grouped_sharded(comm, probs)
            else:
                c.iq2_matmul_grouped(probs)

        def forward():
            x = x0
            for lay in layers:
                w = {name: (qs, sc, n, k) for (_, qs, sc, n, k, _, _, name) in lay}
                matmuls([(x, *w[nm][:2], w[nm][2], w[nm][3], outs[nm]) for nm in ("q", "k", "v", "gate", "up")])
                matmuls([(outs["q"], *w["o"][:2], w["o"][2], w["o"][3], outs["o"])])
                matmuls([(outs["up"], *w["down"][:2], w["down"][2], w["down"][3], outs["down"])])
                d = outs["down"]
                x = d * torch.rsqrt((d * d).mean(dim=1, keepdim=True) + 1e-6)
            return x

        with torch.cuda.stream(stream):
            for _ in range(2):
                forward()
        stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            y = forward()
        with torch.cuda.stream(stream):
            g.replay()
        if dist:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        reps = max(3, args.steps // 10)
        ms = _time_graph(g, reps, stream) / reps
        if dist:
            t = torch.tensor([ms], device=device)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            ms = float(t.item())
        finite = bool(torch.isfinite(y).all().item())
        del g
        res[f"m{m}"] = {"ms_per_forward": round(ms, 4), "weight_gbs": round(wl.weight_bytes / (ms * 1e-3) / 1e9, 1),
                        "finite": finite}
    return {"workload": "config4: 32-layer Llama-3-8B linear stack, RMS-normalised input rows, "
                        "3 calls per layer (q,k,v,gate,up grouped; o; down) + RMS norm between layers",
            **res}


def ffn70b_bench(args, device, stream, comm, rank, world, peaks):
    """Benchmark configuration 3: Llama-3-70B FFN projections (gate/up 8192x28672, down
    28672x8192) at M=1 (one grouped call, weight GB/s) and M=2048 (bf16 x, TFLOPS),
    column-sharded over the ranks when N > 1. Device time, max over ranks."""
    import candelora_metal_kernels_b200 as c
    from candelora_metal_kernels_b200 import synth
    from candelora_metal_kernels_b200.sharded import iq2_matmul_grouped_sharded
    dist = world > 1
    ws = []
    total_bytes = flops_per_m = 0
    for i, (name, k, n) in enumerate(synth.LLAMA3_70B_FFN):
        n_loc = n // world
        qs, sc = synth.iq2xxs_weights(n, k, seed=700 + i, device=device, row_begin=rank * n_loc,
                                      row_end=(rank + 1) * n_loc)
        ws.append((qs, sc, n, k))
        total_bytes += synth.packed_bytes(n, k)
        flops_per_m += 2 * n * k
    res = {}
    for m, dtype in ((1, torch.float32), (2048, torch.bfloat16)):
        probs = []
        for i, (qs, sc, n, k) in enumerate(ws):
            x = synth.activations(m, k, seed=800 + i, dtype=dtype, device=device)
            sym = dist and m <= 16 and comm.has_symmetric
            probs.append((x, qs, sc, n, k, comm.symmetric_empty(m, n) if sym else torch.empty(m, n, device=device)))

        def run():
            if dist:
                iq2_matmul_grouped_sharded(comm, probs)
            else:
                c.iq2_matmul_grouped(probs)

        with torch.cuda.stream(stream):
            for _ in range(2):
                run()
        stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            run()
        with torch.cuda.stream(stream):
            g.replay()
        if dist:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        reps = 20 if m == 1 else 3
        ms = _time_graph(g, reps, stream) / reps
        if dist:
            t = torch.tensor([ms], device=device)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            ms = float(t.item())
        del g, probs
        if m == 1:
            gbs = total_bytes / (ms * 1e-3) / 1e9
            res["m1"] = {"ms": round(ms, 4), "weight_gbs": round(gbs, 1),
                         "frac_hbm_per_gpu": round(gbs / world / peaks["hbm_gbs"], 4)}
        else:
            tf = flops_per_m * m / (ms * 1e-3) / 1e12
            res["m2048"] = {"ms": round(ms, 3), "tflops": round(tf, 1),
                            "frac_bf16_per_gpu": round(tf / world / peaks["bf16_tflops"], 4)}
    return {"workload": "config3: Llama-3-70B FFN gate/up 8192x28672, down 28672x8192, one grouped call"
                        + (f", column-sharded over {world} GPUs (M=1: "
                           + ("fused peer-memory all-gather" if comm.has_symmetric else "NCCL all-gather")
                           + "; M=2048: NCCL all-gather)" if dist else ""), **res}


# ---------------------------------------------------------------------------------------- configs 0/1
def config01_bench(args, device, stream, peaks, peak_src):
    """Benchmark configurations 0 and 1 on one GPU, every M the configuration names.

    config1: M in {1, 4, 8, 16}, f32 x ~N(0,1), the Llama-3-8B projection shapes. Per M: the step of
    8 layers (56 projections, 450 MB of packed weights) as one grouped call and as 56 reference-shaped
    calls, and per shape one call at a time over enough distinct matrices to exceed 260 MB (> 2x L2).
    config0: M=1, 4096x4096, one call (the GPU line), and the reference's own kernels on the host
    cores for the same matvec (its CPU line). CUDA events around replays of CUDA graphs."""
    import candelora_metal_kernels_b200 as c
    from candelora_metal_kernels_b200 import synth
    hbm = peaks["hbm_gbs"]

    def graph_ms(fn, reps):
        with torch.cuda.stream(stream):
            fn()
        stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            fn()
        with torch.cuda.stream(stream):
            g.replay()
        ms = _time_graph(g, reps, stream) / reps
        del g
        return ms

    def line(nbytes, ms):
        gbs = nbytes / (ms * 1e-3) / 1e9
        return {"us": round(ms * 1e3, 2), "weight_gbs": round(gbs, 1), "frac_hbm": round(gbs / hbm, 4)}

    shapes = [("q/o", 4096, 4096), ("k/v", 4096, 1024), ("gate/up", 4096, 14336), ("down", 14336, 4096)]
    mats = {}
    for (name, k, n) in shapes:
        copies = max(4, int(260e6 // synth.packed_bytes(n, k)) + 1)
        mats[name] = [synth.iq2xxs_weights(n, k, seed=3000 + 97 * i + n, device=device) for i in range(copies)]
    res = {}
    for m in (1, 4, 8, 16):
        r = {}
        for (name, k, n) in shapes:
            x = synth.activations(m, k, seed=31 + m, device=device)
            out = torch.empty(m, n, device=device)
            ws = torch.empty(max(1, c.workspace_bytes(m, n, k, torch.float32)), dtype=torch.uint8, device=device)
            ml = mats[name]

            def calls(ml=ml, x=x, out=out, ws=ws, n=n, k=k):
                for (qs, sc) in ml:
                    c.iq2_xxs_matmul(x, qs, sc, n, k, out=out, workspace=ws)
            ms = graph_ms(calls, 5) / len(ml)
            r[f"single_{k}x{n}"] = line(synth.packed_bytes(n, k), ms)
        probs, wbytes = [], 0
        for layer in range(8):
            for pi, (name, k, n) in enumerate(synth.LLAMA3_8B_PROJECTIONS):
                qs, sc = synth.iq2xxs_weights(n, k, seed=layer * 16 + pi, device=device)
                probs.append((synth.activations(m, k, seed=pi, device=device), qs, sc, n, k,
                              torch.empty(m, n, device=device)))
                wbytes += synth.packed_bytes(n, k)
        gws = torch.empty(max(1, c.grouped_workspace_bytes(probs)), dtype=torch.uint8, device=device)
        r["step_8_layers_grouped"] = line(wbytes, graph_ms(lambda: c.iq2_matmul_grouped(probs, workspace=gws), 10))
        pws = {}
        for (x, qs, sc, n, k, o) in probs:
            pws.setdefault((n, k), torch.empty(max(1, c.workspace_bytes(m, n, k, torch.float32)), dtype=torch.uint8,
                                               device=device))

        def per_call():
            for (x, qs, sc, n, k, o) in probs:
                c.iq2_xxs_matmul(x, qs, sc, n, k, out=o, workspace=pws[(n, k)])
        r["step_8_layers_per_call"] = line(wbytes, graph_ms(per_call, 10))
        res[f"m{m}"] = r
        del probs, gws, pws
    del mats
    torch.cuda.empty_cache()
    cfg0 = dict(res["m1"]["single_4096x4096"])
    if not args.no_cpu_baseline:
        from oracle.oracle import Oracle, RefKernels
        kind = "reference" if RefKernels.available() else "port"
        impl = RefKernels() if kind == "reference" else Oracle()
        qs, sc = synth.iq2xxs_weights(4096, 4096, seed=0)
        x = synth.activations(1, 4096, seed=1).numpy()
        qs, sc = qs.numpy(), sc.numpy()
        threads = os.cpu_count() or 1
        run = ((lambda: impl.matmul(x, qs, sc, 4096, 4096, "f32", threads=threads)) if kind == "reference"
               else (lambda: impl.matmul(x, qs, sc, 4096, 4096, threads=threads)))
        run()
        t0, reps = time.perf_counter(), 0
        while time.perf_counter() - t0 < 2.0:
            run()
            reps += 1
        cms = (time.perf_counter() - t0) / reps * 1e3
        cfg0["cpu"] = {"ms": round(cms, 3), "weight_gbs": round(synth.packed_bytes(4096, 4096) / (cms * 1e-3) / 1e9, 3),
                       "cores": threads, "kind": kind}
    return {"config0": {"workload": "M=1, K=N=4096, f32 x, one call", **cfg0},
            "config1": {"workload": "Llama-3-8B projection shapes, f32 x, M in {1,4,8,16}; single calls over "
                                    "> 260 MB of distinct matrices per shape, and the 8-layer step (450 MB) "
                                    "grouped and per call", "peak_hbm_gbs": hbm, "peak_source": peak_src, **res}}


# ---------------------------------------------------------------------------------------- GEMM
def gemm_bench(args, device, stream, peaks, peak_src):
    """Benchmark configuration 2: prefill GEMM on the tensor-core path, bf16 x ~N(0,1), M in {512,
    2048}, (K, N) in {(4096, 14336), (14336, 4096)}. Each shape rotates over enough distinct (x, W)
    pairs to exceed L2; CUDA events around back-to-back calls captured in a CUDA graph."""
    import candelora_metal_kernels_b200 as c
    from candelora_metal_kernels_b200 import synth
    res = {}
    tot_flop = tot_ms = 0.0
    for m in (2048, 512):
        for (k, n) in ((4096, 14336), (14336, 4096)):
            per = synth.packed_bytes(n, k) + m * k * 2
            copies = max(2, int(260e6 // per) + 1)
            pairs = []
            for i in range(copies):
                qs, sc = synth.iq2xxs_weights(n, k, seed=900 + i, device=device)
                x = synth.activations(m, k, seed=950 + i, dtype=torch.bfloat16, device=device)
                pairs.append((x, qs, sc))
            out = torch.empty(m, n, device=device)
            ws = torch.empty(c.workspace_bytes(m, n, k, torch.bfloat16), dtype=torch.uint8, device=device)
            with torch.cuda.stream(stream):
                for (x, qs, sc) in pairs:
                    c.iq2_xxs_matmul(x, qs, sc, n, k, out=out, workspace=ws)
            stream.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                for (x, qs, sc) in pairs:
                    c.iq2_xxs_matmul(x, qs, sc, n, k, out=out, workspace=ws)
            reps = max(3, args.gemm_reps)
            with torch.cuda.stream(stream):
                g.replay()
            ms = _time_graph(g, reps, stream) / (reps * copies)
            del g
            flop = 2.0 * m * n * k
            tf = flop / (ms * 1e-3) / 1e12
            res[f"m{m}_k{k}_n{n}"] = {"us": round(ms * 1e3, 1), "tflops": round(tf, 1),
                                      "frac": round(tf / peaks["bf16_tflops"], 4)}
            if m == 2048:
                tot_flop += flop
                tot_ms += ms
    tf = tot_flop / (tot_ms * 1e-3) / 1e12
    return {"metric": "TFLOPS at M=2048 (configuration 2: 4096x14336 and 14336x4096, bf16 x)",
            "value": round(tf, 1), "unit": "TFLOP/s",
            "roofline": {"bound": "tensor", "kernel": "gemm_kernel (tcgen05, bf16 x bf16 -> f32)",
                         "achieved": round(tf, 1), "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": round(tf / peaks["bf16_tflops"], 4), "peak_source": f"{peak_src} (burst)"},
            "shapes": res, "l2": "each shape rotates over distinct (x, W) pairs totalling > 260 MB"}


def next_rows_bench(args, device, stream, peaks, peak_src):
    """The rows beside the benchmarked path, each on a Llama-3-8B gate/up shape (K=4096, N=14336),
    one GPU, inputs resident, HBM-bound, against measured HBM:
      w8a8      iq2_matmul_with_activation_quant (IQ2_XXS, W8A8) at M=1 and M=16; packed weight GB/s
      variants  iq2_xs_matmul / iq2_s_matmul / iq3_s_matmul at M=1, f32 x; packed weight GB/s
      variants_prefill_tcgen05  the same at M=2048, bf16 x (the tcgen05 GEMM); TFLOP/s against the
                measured bf16 burst
      dequant   iq2_dequantize to f16 (IQ2_XXS); GB/s of packed bytes read + f16 bytes written
      gguf      split_interleaved of ggml IQ2_XXS blocks; GB/s of block bytes read + written
    Matmuls rotate over distinct weights totalling > 260 MB (CUDA graph of back-to-back calls);
    dequant and repack run on inputs and outputs larger than L2 (CUDA events around eager calls)."""
    import candelora_metal_kernels_b200 as c
    from candelora_metal_kernels_b200 import gguf, synth
    V = c.Iq2MatmulVariant
    hbm = peaks["hbm_gbs"]
    n, k = 14336, 4096
    nb = k // 256
    gen = torch.Generator(device=device)
    gen.manual_seed(7)

    def variant_weights(var):
        bpb, spb = gguf.SPLIT[var]
        wb = torch.randint(0, 256, (n * nb * bpb,), dtype=torch.uint8, device=device, generator=gen)
        ws = torch.randint(0, 256, (n * nb, spb), dtype=torch.uint8, device=device, generator=gen)
        d = (torch.rand(n * nb, device=device, generator=gen) * 9e-3 + 1e-3).to(torch.float16)
        ws[:, :2] = d.view(torch.uint8).view(-1, 2)
        return wb, ws.reshape(-1)

    def matmul_gbs(fn, var, m, xdt=torch.float32):
        bpb, spb = gguf.SPLIT[var]
        wbytes = n * nb * (bpb + spb)
        copies = max(2, int(260e6 // wbytes) + 1)
        ws_list = [synth.iq2xxs_weights(n, k, seed=700 + i, device=device) if var == V.Iq2Xxs
                   else variant_weights(var) for i in range(copies)]
        x = synth.activations(m, k, seed=77, dtype=xdt, device=device)
        out = torch.empty(m, n, device=device)
        wsp = torch.empty(max(1, c.workspace_bytes(m, n, k, xdt, var)), dtype=torch.uint8, device=device)
        with torch.cuda.stream(stream):
            for (wb, sc) in ws_list:
                fn(x, wb, sc, out, wsp)
        stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for (wb, sc) in ws_list:
                fn(x, wb, sc, out, wsp)
        with torch.cuda.stream(stream):
            g.replay()
        reps = 10
        ms = _time_graph(g, reps, stream) / (reps * copies)
        del g
        gbs = wbytes / (ms * 1e-3) / 1e9
        return {"us": round(ms * 1e3, 2), "weight_gbs": round(gbs, 1), "frac_hbm": round(gbs / hbm, 4)}

    def prefill_tflops(var, m=2048):
        """The variant's tcgen05 GEMM at M=m (bf16 x), weights rotated over > 260 MB."""
        bpb, spb = gguf.SPLIT[var]
        wbytes = n * nb * (bpb + spb)
        copies = max(2, int(260e6 // wbytes) + 1)
        ws_list = [variant_weights(var) for _ in range(copies)]
        x = synth.activations(m, k, seed=78, dtype=torch.bfloat16, device=device)
        out = torch.empty(m, n, device=device)
        wsp = torch.empty(max(1, c.workspace_bytes(m, n, k, torch.bfloat16, var)), dtype=torch.uint8, device=device)
        for (wb, sc) in ws_list:
            c.iq2_matmul(x, wb, sc, n, k, var, out=out, workspace=wsp)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 3
        e0.record()
        for _ in range(reps):
            for (wb, sc) in ws_list:
                c.iq2_matmul(x, wb, sc, n, k, var, out=out, workspace=wsp)
        e1.record()
        e1.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / (reps * copies)
        tf = 2.0 * m * n * k / (us * 1e-6) / 1e12
        return {"m": m, "us": round(us, 1), "tflops": round(tf, 1),
                "frac_bf16_burst": round(tf / peaks["bf16_tflops"], 4)}

    aq = c.ActivationQuantConfig(c.ActivationQuantMode.W8A8)
    w8a8 = {f"m{m}": matmul_gbs(lambda x, wb, sc, o, w: c.iq2_matmul_with_activation_quant(
        x, wb, sc, n, k, V.Iq2Xxs, aq, out=o, workspace=w), V.Iq2Xxs, m) for m in (1, 16)}
    variants, variants_prefill = {}, {}
    for name, var in (("iq2_xs", V.Iq2Xs), ("iq2_s", V.Iq2S), ("iq3_s", V.Iq3S)):
        variants[name] = matmul_gbs(lambda x, wb, sc, o, w, var=var: c.iq2_matmul(
            x, wb, sc, n, k, var, out=o, workspace=w), var, 1)
        variants_prefill[name] = prefill_tflops(var)

    def eager_ms(fn, reps=20):
        with torch.cuda.stream(stream):
            fn()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(reps):
                fn()
            e1.record(stream)
        e1.synchronize()
        return e0.elapsed_time(e1) / reps

    # dequant: two 14336x4096 matrices in rotation (2 x 132 MB of traffic per pair of calls)
    mats = [synth.iq2xxs_weights(n, k, seed=710 + i, device=device) for i in range(2)]
    outs = [torch.empty(n, k, dtype=torch.float16, device=device) for _ in range(2)]
    state = [0]

    def deq():
        i = state[0] = state[0] ^ 1
        c.iq2_dequantize(mats[i][0], mats[i][1], n, k, dtype=torch.float16, out=outs[i])
    ms = eager_ms(deq)
    dbytes = synth.packed_bytes(n, k) + n * k * 2
    dq = {"us": round(ms * 1e3, 2), "gbs": round(dbytes / (ms * 1e-3) / 1e9, 1),
          "frac_hbm": round(dbytes / (ms * 1e-3) / 1e9 / hbm, 4), "bytes": dbytes}
    del mats, outs

    # ggml interleaved blocks -> split tensors: 8 x (14336 x 4096) of IQ2_XXS blocks (121 MB each way)
    nblk = 8 * n * nb
    blocks = torch.randint(0, 256, (nblk * 66,), dtype=torch.uint8, device=device, generator=gen)
    ms = eager_ms(lambda: gguf.split_interleaved(blocks, nblk, V.Iq2Xxs), reps=10)
    gbytes = 2 * nblk * 66
    gg = {"us": round(ms * 1e3, 2), "gbs": round(gbytes / (ms * 1e-3) / 1e9, 1),
          "frac_hbm": round(gbytes / (ms * 1e-3) / 1e9 / hbm, 4), "bytes": gbytes}
    del blocks
    return {"shape": "K=4096, N=14336 (Llama-3-8B gate/up)", "peak_hbm_gbs": hbm, "peak_source": peak_src,
            "w8a8": w8a8, "variants": variants, "variants_prefill_tcgen05": variants_prefill,
            "dequant_f16": dq, "gguf_split_interleaved": gg}


# ---------------------------------------------------------------------------------------- CPU
def cpu_baseline(args, seconds: float = 10.0, steps: int | None = None):
    """The reference's own kernels (compiled from source for the host) on a bounded sample of
    the workload: the 7 projections of layer 0 at M=1, repeated for ~`seconds`."""
    from oracle.oracle import Oracle, RefKernels
    from candelora_metal_kernels_b200 import synth
    kind = "reference" if RefKernels.available() else "port"
    impl = RefKernels() if kind == "reference" else Oracle()
    threads = os.cpu_count() or 1
    layer = []
    total = 0
    for pi, (name, k, n) in enumerate(synth.LLAMA3_8B_PROJECTIONS):
        qs, sc = synth.iq2xxs_weights(n, k, pi)
        x = synth.activations(args.m, k, seed=10_000 + pi).numpy()
        layer.append((x, qs.numpy(), sc.numpy(), n, k))
        total += synth.packed_bytes(n, k)

    def one():
        for (x, qs, sc, n, k) in layer:
            if kind == "reference":
                impl.matmul(x, qs, sc, n, k, "f32", threads=threads)
            else:
                impl.matmul(x, qs, sc, n, k, threads=threads)

    one()  # warm
    t0 = time.perf_counter()
    reps = 0
    times = []
    while (steps is None and time.perf_counter() - t0 < seconds) or (steps is not None and reps < steps):
        t1 = time.perf_counter()
        one()
        times.append(time.perf_counter() - t1)
        reps += 1
    el = sum(times)
    return {"value": round(total * reps / el / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": kind,
            "sample": f"layer-0 q,k,v,o,gate,up,down at M=1 ({total} packed bytes) x {reps} passes, {el:.1f} s",
            "ms_per_sample": round(el / reps * 1e3, 2)}


def run_reference(args, rank: int, world: int):
    if rank != 0:
        return None
    cb = cpu_baseline(args, steps=args.steps)
    # warm-up passes are included in cpu_baseline's first untimed call; W extra untimed passes:
    return {"metric": METRIC, "impl": "reference", "value": cb["value"], "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": cb["ms_per_sample"],
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32 activations x IQ2_XXS weights (f32 accumulate)", "data": "synthetic",
            "config": {"workload": "config1: Llama-3-8B projections, M=1 (host cores; bounded sample per step)",
                       "m": args.m},
            "cpu_baseline": {"value": cb["value"], "unit": "GB/s", "cores": cb["cores"], "kind": cb["kind"],
                             "sample": cb["sample"]},
            "e2e": {"value": cb["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


# ---------------------------------------------------------------------------------------- cases
def run_case(args):
    """Only the dominant kernel on its roofline shape, `--steps` times after two warm calls: the
    command the profiler captures. gemv: 4096x14336 (K x N) at M=1, f32 x, two weight copies
    (30 MB) in turn; gemm: M=2048 (or `--m` M > 32) on the same projection, bf16 x; grouped: the
    benchmark step (every projection of `--layers` layers in one iq2_matmul_grouped call, M=1);
    variant: the `--variant` format's matmul on the gemv shape (random blocks, d ~U[1e-3, 1e-2]) at
    `--m` M <= 32 with f32 x (the decode kernel), or M > 32 with bf16 x (the tcgen05 GEMM)."""
    import candelora_metal_kernels_b200 as c
    from candelora_metal_kernels_b200 import gguf, synth
    torch.cuda.set_device(0)
    if args.case == "grouped":
        wl = Workload(1, args.layers, 0, 1, torch.device("cuda", 0))
        for _ in range(2):
            wl.step(grouped=True)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            wl.step(grouped=True)
        e1.record()
        e1.synchronize()
        print(json.dumps({"case": "grouped", "m": 1, "layers": args.layers, "weight_bytes": wl.weight_bytes,
                          "calls": args.steps, "us_per_call": round(e0.elapsed_time(e1) * 1e3 / args.steps, 2)}),
              flush=True)
        return
    k, n = (int(v) for v in args.kn.split(","))
    if args.case == "variant":
        var = {"iq2_xs": c.Iq2MatmulVariant.Iq2Xs, "iq2_s": c.Iq2MatmulVariant.Iq2S,
               "iq3_s": c.Iq2MatmulVariant.Iq3S}[args.variant]
        bpb, spb = gguf.SPLIT[var]
        nb = k // 256
        g = torch.Generator(device="cuda")
        g.manual_seed(1)
        wb = torch.randint(0, 256, (n * nb * bpb,), dtype=torch.uint8, device="cuda", generator=g)
        sc = torch.randint(0, 256, (n * nb, spb), dtype=torch.uint8, device="cuda", generator=g)
        sc[:, :2] = (torch.rand(n * nb, device="cuda", generator=g) * 9e-3 + 1e-3).to(torch.float16).view(
            torch.uint8).view(-1, 2)
        sc = sc.reshape(-1)
        vm = args.m  # (m > 32: the tcgen05 GEMM, bf16 x; else the decode kernel, f32 x)
        x = synth.activations(vm, k, seed=1, dtype=torch.bfloat16 if vm > 32 else torch.float32, device="cuda")
        out = torch.empty(vm, n, device="cuda")
        vws = torch.empty(max(1, c.workspace_bytes(vm, n, k, x.dtype, var)), dtype=torch.uint8, device="cuda")
        for _ in range(2):
            c.iq2_matmul(x, wb, sc, n, k, var, out=out, workspace=vws)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            c.iq2_matmul(x, wb, sc, n, k, var, out=out, workspace=vws)
        e1.record()
        e1.synchronize()
        print(json.dumps({"case": "variant", "variant": args.variant, "m": vm, "k": k, "n": n, "calls": args.steps,
                          "us_per_call": round(e0.elapsed_time(e1) * 1e3 / args.steps, 2)}), flush=True)
        return
    m = 1 if args.case == "gemv" else (args.m if args.m > 32 else 2048)
    dtype = torch.float32 if args.case == "gemv" else torch.bfloat16
    ws_ = [tuple(t.cuda() for t in synth.iq2xxs_weights(n, k, seed=i)) for i in range(2)]
    x = synth.activations(m, k, seed=1, dtype=dtype, device="cuda")
    out = torch.empty(m, n, device="cuda")
    ws = torch.empty(c.workspace_bytes(m, n, k, dtype), dtype=torch.uint8, device="cuda")
    for i in range(2):
        c.iq2_xxs_matmul(x, ws_[i % 2][0], ws_[i % 2][1], n, k, out=out, workspace=ws)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.steps):
        c.iq2_xxs_matmul(x, ws_[i % 2][0], ws_[i % 2][1], n, k, out=out, workspace=ws)
    e1.record()
    e1.synchronize()
    print(json.dumps({"case": args.case, "m": m, "k": k, "n": n, "calls": args.steps,
                      "us_per_call": round(e0.elapsed_time(e1) * 1e3 / args.steps, 2)}), flush=True)


# ---------------------------------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--m", type=int, default=1)
    ap.add_argument("--layers", type=int, default=LAYERS)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-gemm", action="store_true")
    ap.add_argument("--no-next-rows", action="store_true",
                    help="skip the W8A8 / IQ2_XS / IQ2_S / IQ3_S / dequant / ggml-repack measurements")
    ap.add_argument("--no-models", action="store_true", help="skip the configuration 3 and 4 measurements")
    ap.add_argument("--no-config01", action="store_true", help="skip the configuration 0 and 1 sweep (M = 1, 4, 8, 16)")
    ap.add_argument("--exchange", choices=["fused", "nccl"], default="fused",
                    help="N > 1: how the sharded decode's output slices reach every rank")
    ap.add_argument("--gemm-reps", type=int, default=5)
    ap.add_argument("--case", choices=["gemv", "gemm", "grouped", "variant"], default=None,
                    help="run only the dominant kernel's shape (the profiler's small case) and exit")
    ap.add_argument("--kn", default="4096,14336", help="--case gemv/gemm/variant: K,N of the projection")
    ap.add_argument("--variant", choices=["iq2_xs", "iq2_s", "iq3_s"], default="iq2_xs",
                    help="--case variant: the weight format")
    args = ap.parse_args()
    if args.case:
        run_case(args)
        return

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE={world}", file=sys.stderr)

    if args.impl == "reference":
        line = run_reference(args, rank, world)
        if line is not None:
            print(json.dumps(line), flush=True)
        return

    if world > 1:
        import datetime
        torch.cuda.set_device(local_rank)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                             device_id=torch.device("cuda", local_rank))
    try:
        line = run_ours(args, rank, world, local_rank)
        if line is not None:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
