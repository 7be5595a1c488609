"""Model-switch benchmark: BF16 weight GB/s per GPU and switch latency.

One step = one in-place switch of the whole resident model (Teacher2 -> Teacher1
or back, alternating) driven by the encoded delta stream.

  value : kernel-only throughput, the encoded stream already resident in HBM;
          sum over ranks of switched weight bytes / max-over-ranks time.
  e2e   : the same switch through the public API (DeltaWeights.apply) with the
          stream staged every step from the pinned host arena (H2D inside the
          timed region) and the device result read back; on N > 1 ranks each
          switch is confirmed by the NCCL all-reduce of per-rank outcomes.

Workloads (synthetic, generated on the GPU with fixed seeds, see
warpshift_b200/synth.py): llama3-8b (the default on one GPU; one 8B-shaped model
per rank), llama3-70b (the default on N > 1 GPUs: the tensor-parallel shard of
rank r at TP = N), mixtral-8x7b (TP-8 shard, sparse delta; the pinned
full-backup restore is timed beside it), qwen2-0.5b. Inputs are >= 12 GB per
rank, far larger than the 126 MB L2, so no explicit L2 flush is needed.

After the timed regions every tensor of every rank is compared on the device
with a regenerated Teacher (``verified_tensors``).

``--impl reference`` times the reference's switch on the host cores
(oracle/reference_cpu.py: the restore of delta.py:74-92 applied to the
residuals the reference's decode hands it, in the mode its rule chooses),
rank 0 only, with every core, on the same workload; it loads no library of
this repository.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "model-switch latency (ms) and BF16 weight GB/s per GPU, 8B TP1 / 70B TP1-8"
UNIT = "GB/s"


def parse_args() -> argparse.Namespace:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--workload", default=None, choices=["llama3-8b", "llama3-70b", "mixtral-8x7b", "qwen2-0.5b"],
                   help="default: llama3-8b on one GPU, llama3-70b at TP = number of GPUs otherwise")
    p.add_argument("--escapes", type=int, default=0,
                   help="word dictionaries with escape lists: 0 when smaller (default), -1 never, 1 whenever eligible")
    p.add_argument("--split", type=int, default=0,
                   help="split-word dictionaries (low k bits stored raw): 0 the k estimated smallest (default), "
                        "-1 never, 1 / 2 / 4 that k whenever eligible")
    p.add_argument("--policy", default="xor", choices=["auto", "xor", "u16"])
    p.add_argument("--scale", type=float, default=0.01, help="relative perturbation s of Teacher2")
    p.add_argument("--cpu-seconds", type=float, default=15.0, help="CPU baseline time budget")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-reference-gpu", action="store_true",
                   help="skip timing the reference's Triton restore kernel (baseline/_ref) on this GPU")
    p.add_argument("--ref-sample-gb", type=float, default=24.0,
                   help="reference arm: host bytes of the workload switched per step (its leading tensors)")
    p.add_argument("--threads", type=int, default=0, help="host encoder threads (0 = all)")
    p.add_argument("--layers", type=int, default=0, help="truncate the model to N layers (small profiling cases)")
    p.add_argument("--skip-e2e", action="store_true", help="time only the kernel-only switch (profiling cases)")
    p.add_argument("--tp", type=int, default=0, help="tensor-parallel degree of the 70B shard (default: number of ranks)")
    p.add_argument("--compare-full-copy", action="store_true",
                   help="also time the pinned full-backup restore path (on by default for mixtral-8x7b)")
    args = p.parse_args()
    if args.workload is None:
        args.workload = "llama3-8b" if args.gpus == 1 else "llama3-70b"
    if args.workload == "mixtral-8x7b":
        args.compare_full_copy = True
    return args


# --------------------------------------------------------------------------- helpers
def peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        d = json.loads(path.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clock/throttle samples of one GPU while the timed regions run."""

    FIELDS = "clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"

    def __init__(self, gpu_id: str) -> None:
        self.gpu_id = gpu_id
        self.samples: list[list[str]] = []
        self.proc = None
        self.thread = None

    def __enter__(self) -> "ClockSampler":
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.gpu_id, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True,
            )
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self) -> None:
        for line in self.proc.stdout:
            self.samples.append([x.strip() for x in line.split(",")])

    def __exit__(self, *exc) -> None:
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            if self.thread:
                self.thread.join(timeout=5)

    def summary(self) -> dict:
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        sm, mx, reasons = [], [], set()
        for s in self.samples:
            try:
                sm.append(float(s[0]))
                mx.append(float(s[1]))
            except (ValueError, IndexError):
                continue
            for name, flag in zip(names, s[3:7]):
                if flag.strip().lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons), "samples": len(sm)}


def init_distributed(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    group = None
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))
        group = dist.group.WORLD
    return world, rank, local, group


def workload_spec(args, world: int, rank: int):
    import dataclasses

    from warpshift_b200 import synth

    shape = synth.SHAPES[args.workload]
    suffix = ""
    if args.layers:
        shape = dataclasses.replace(shape, layers=min(args.layers, shape.layers))
        suffix = f", truncated to {shape.layers} layers"
    if args.workload == "llama3-70b":
        tp = args.tp or world
        return synth.model_spec(shape, tp=tp, rank=rank % tp), f"llama3-70b tp={tp}, rank r switches shard r{suffix}"
    if args.workload == "mixtral-8x7b":
        return synth.model_spec(shape, tp=8, rank=rank % 8), f"mixtral-8x7b tp=8 shard per rank, sparse delta{suffix}"
    return synth.model_spec(shape), f"{args.workload} tp=1, one model per rank{suffix}"


def workload_config(args, desc: str, nbytes: int) -> dict:
    """The workload's identity: the same object in both arms' lines."""
    return {"workload": desc, "policy": args.policy, "scale": args.scale, "escapes": args.escapes, "split": args.split,
            "l2": f"inputs ({nbytes / 1e9:.2f} GB of weights per rank) larger than the 126 MB L2; no flush"}


def generate_on_device(spec, device, scale):
    """Teacher1 -> one pageable host buffer (cpu_base views); Teacher2 stays resident on the GPU."""
    import torch

    from warpshift_b200 import synth

    total = 0
    offsets = []
    for t in spec.tensors:
        offsets.append(total)
        total += (t.nbytes + 255) // 256 * 256
    host = torch.empty(total, dtype=torch.uint8)
    cpu_base, gpu = {}, {}
    for i, t in enumerate(spec.tensors):
        x = synth.teacher1_tensor(t, i, device)
        view = host[offsets[i] : offsets[i] + t.nbytes].view(t.dtype).view(t.shape)
        view.copy_(x)
        synth.perturb_(x, t, i, scale)
        cpu_base[t.name], gpu[t.name] = view, x
    torch.cuda.synchronize(device)
    torch.cuda.empty_cache()  # the generation temporaries stay cached otherwise (~20 GB at 70B TP=1)
    return cpu_base, gpu


def measure_h2d(device, nbytes: int, group=None) -> tuple[float, float]:
    """The host->device half of a switch alone: this rank copies `nbytes` (its
    stream's size) from pinned host memory, in 1 GiB pieces, with every rank
    starting together as in the end-to-end switch, so ranks that share host
    links share them here too and a rank whose peers finish early speeds up as
    it does in the switch. Returns (GB/s, ms) of this rank's copies."""
    import torch
    import torch.distributed as dist

    if nbytes <= 0:
        return float("nan"), 0.0
    n = min(1 << 30, nbytes)
    src = torch.empty(n, dtype=torch.uint8, pin_memory=True)
    dst = torch.empty(n, dtype=torch.uint8, device=device)
    dst.copy_(src, non_blocking=True)
    torch.cuda.synchronize(device)
    if group is not None:
        dist.barrier(group=group)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for off in range(0, nbytes, n):
        k = min(n, nbytes - off)
        dst[:k].copy_(src[:k], non_blocking=True)
    e.record()
    torch.cuda.synchronize(device)
    ms = s.elapsed_time(e)
    del src, dst
    return nbytes / (ms * 1e-3) / 1e9, ms


def reference_workload(spec, scale: float, policy: str, budget_bytes: int, threads: int):
    """Host tensors holding Teacher2 and the reference's per-packet residuals for the
    leading tensors of ``spec`` up to ``budget_bytes``. Teachers are generated by
    torch (on the GPU when there is one) with the synth conventions; nothing from
    this repository's native library is used."""
    import torch

    from oracle import reference_cpu
    from warpshift_b200 import synth

    device = torch.device("cuda", 0) if torch.cuda.is_available() else torch.device("cpu")
    tensors, packets, total = {}, [], 0
    for i, t in enumerate(spec.tensors):
        if total >= budget_bytes:
            break
        x = synth.teacher1_tensor(t, i, device)
        y = synth.perturb_(x.clone(), t, i, scale)
        a = x.reshape(-1).view(torch.uint8).cpu().numpy()
        b = y.reshape(-1).view(torch.uint8).cpu().numpy()
        del x, y
        tensors[t.name] = b
        packets += reference_cpu.packets_of({t.name: a}, {t.name: b}, {t.name: t.dtype == torch.bfloat16}, policy,
                                            threads)
        total += t.nbytes
    return tensors, packets, total


def reference_cpu_baseline(spec, cpu_base, gpu, policy: str, seconds: float) -> dict:
    """The reference's restore on this host's cores over a bounded sample of the
    workload (~``seconds`` on all cores, then one core), plus this format's own
    entropy stage decoded by the oracle's C decoder, reported separately."""
    import torch

    from oracle import reference_cpu

    cores = len(os.sched_getaffinity(0))
    budget, tensors, packets, total = 2 << 30, {}, [], 0
    for t in spec.tensors:
        if total >= budget:
            break
        a = cpu_base[t.name].reshape(-1).view(torch.uint8).numpy()
        b = gpu[t.name].reshape(-1).view(torch.uint8).cpu().numpy()
        tensors[t.name] = b
        packets += reference_cpu.packets_of({t.name: a}, {t.name: b}, {t.name: t.dtype == torch.bfloat16}, policy, cores)
        total += t.nbytes
    sw = reference_cpu.CpuSwitch(tensors, packets)
    steps, elapsed = 0, 0.0
    while elapsed < seconds or steps < 2:
        elapsed += sw.switch()
        steps += 1
    one_steps, one_elapsed = 0, 0.0
    while one_elapsed < min(5.0, seconds / 2) or one_steps < 1:
        one_elapsed += sw.switch(threads=1)
        one_steps += 1
    out = {
        "value": round(steps * total / elapsed / 1e9, 3), "unit": UNIT, "cores": cores, "kind": "port",
        "sample": (f"{len(tensors)} leading tensor(s) of the workload ({total / 1e9:.2f} GB), {steps} switches: "
                   f"the reference's restore (delta.py:74-92, oracle/reference_cpu.py) over {cores} threads"),
        "seconds": round(elapsed, 2),
        "single_core": {"value": round(one_steps * total / one_elapsed / 1e9, 3), "unit": UNIT, "cores": 1,
                        "switches": one_steps},
    }
    del tensors, packets, sw
    try:
        out["entropy_stage"] = oracle_stream_decode(spec, cpu_base, gpu, policy, min(seconds, 10.0), cores)
    except Exception as exc:  # the entropy leg is informative only
        out["entropy_stage"] = {"error": f"{type(exc).__name__}: {exc}"}
    return out


def oracle_stream_decode(spec, cpu_base, gpu, policy: str, seconds: float, cores: int) -> dict:
    """This format's rANS decode + restore by the oracle's plain-C decoder on the host
    cores (the CPU cost of the entropy stage the GPU kernel fuses)."""
    import ctypes

    import numpy as np

    from oracle import stream as ostream
    from warpshift_b200 import _lib
    from warpshift_b200.delta import _DICT_SLACK_PCT

    a, b, total = {}, {}, 0
    for t in spec.tensors:
        if total >= (1 << 30):
            break
        a[t.name] = cpu_base[t.name]
        b[t.name] = gpu[t.name].cpu()
        total += t.nbytes
    lib = _lib.load()
    descs = (_lib.TensorDesc * len(a))()
    for i, name in enumerate(b):
        descs[i] = _lib.TensorDesc(a[name].data_ptr(), b[name].data_ptr(), b[name].numel() * b[name].element_size(),
                                   int(str(b[name].dtype) == "torch.bfloat16"), 0)
    opts = _lib.BuildOptions(policy=_lib.POLICIES[policy], threads=0, target_on_device=0, device=0,
                             batch_bytes=0, staging_slots=0, pin_arena=0, dict_slack_pct=_DICT_SLACK_PCT)
    plan = ctypes.c_void_p()
    _lib.check(lib.ws_plan_build(descs, len(a), ctypes.byref(opts), None, ctypes.byref(plan)))
    try:
        view, stats = _lib.PlanView(), _lib.PlanStats()
        lib.ws_plan_get_view(plan, ctypes.byref(view))
        lib.ws_plan_get_stats(plan, ctypes.byref(stats))

        def arr(ptr, n, dt):
            return np.ctypeslib.as_array((ctypes.c_uint8 * n).from_address(ptr)).view(dt) if n else np.zeros(0, dt)

        blocks = arr(view.blocks, 32 * view.nblocks, ostream.BLOCK_DTYPE)
        tiles = arr(view.tiles, 16 * view.ntiles, ostream.TILE_DTYPE)
        tables = arr(view.tables, 2048 * view.ntables, np.uint32)
        expected = (int(stats.expected_checksum[0]), int(stats.expected_checksum[1]))
        reverse, steps, elapsed = True, 0, 0.0
        while elapsed < seconds or steps < 2:
            t0 = time.perf_counter()
            err, ck = ostream.apply_plan(blocks, tiles, tables, int(view.arena), 0, reverse, cores)
            elapsed += time.perf_counter() - t0
            if err or ck != expected[1 if reverse else 0]:
                raise RuntimeError("oracle decode produced wrong bytes")
            reverse = not reverse
            steps += 1
    finally:
        lib.ws_plan_destroy(plan)
    return {"value": round(steps * total / elapsed / 1e9, 3), "unit": UNIT, "cores": cores,
            "sample": f"{len(a)} leading tensor(s) ({total / 1e9:.2f} GB), {steps} switches: rANS decode of this "
                      "format + restore in plain C (oracle/stream_oracle.c)"}


def per_direction(ms: list, reverse: list) -> dict:
    """Median step time per switch direction (the reference's validate.py:272-293 reports medians)."""
    out = {}
    for label, flag in (("A->B", False), ("B->A", True)):
        xs = [m for m, r in zip(ms, reverse) if r == flag]
        if xs:
            out[label] = round(statistics.median(xs), 3)
    return out


def verify_all_tensors(spec, gpu, state_is_b: bool, scale: float, device) -> int:
    """Compare every switched tensor with its regenerated Teacher on the device; returns the count."""
    import torch

    from warpshift_b200 import synth

    for i, t in enumerate(spec.tensors):
        ref = synth.teacher1_tensor(t, i, device)
        if state_is_b:
            synth.perturb_(ref, t, i, scale)
        if not torch.equal(ref.reshape(-1).view(torch.uint8), gpu[t.name].reshape(-1).view(torch.uint8)):
            raise RuntimeError(f"final weights differ from the regenerated teacher on {t.name}")
        del ref
    return len(spec.tensors)


def reference_triton_restore(spec, gpu, state_is_b: bool, scale: float, policy: str, device, steps: int,
                             warmup: int) -> dict:
    """The reference's own Triton restore kernel (warpshift/delta.py:60-92, from the
    reference package installed in baseline/_ref) timed on this GPU over the whole
    workload, launched per batch as DeltaWeights.apply does (delta.py:300-324).

    Its input is what the reference's nvCOMP decode would leave in the decoded
    buffer (delta.py:313-316): per 16 MiB packet the XOR regrouped into byte planes
    (mode 1), the zigzag planes (mode 3, U16 policy) or, below 16384 bytes, the raw
    XOR (mode 0), all generated on the device from the Teachers. nvCOMP itself is
    not installed anywhere here, so its decode time is not included: this is the
    reference's switch minus its entropy decode. Returns the mean time of one
    switch of the whole workload and checks that the weights end where they began.
    """
    import torch

    ref = ROOT / "baseline" / "_ref"
    if not (ref / "warpshift" / "delta.py").exists():
        return {"unavailable": "reference package not installed in baseline/_ref"}
    if str(ref) not in sys.path:
        sys.path.insert(0, str(ref))
    from warpshift import delta as refdelta  # the reference's module: imports torch and triton only

    from warpshift_b200 import synth

    chunk, tile = refdelta._CHUNK_BYTES, refdelta._TILE_BYTES
    packets, total = [], 0  # (mode, dst, num_bytes, arena offset)
    for name, t in gpu.items():
        n = t.numel() * t.element_size()
        for off in range(0, n, chunk):
            m = min(chunk, n - off)
            if m < 16384:  # delta.py:185: smaller packets stay raw XOR
                mode = 0
            elif policy == "u16" and t.dtype == torch.bfloat16 and m % 2 == 0:
                mode = 3
            else:
                mode = 1 if m % 2 == 0 else 2
            packets.append((mode, t.data_ptr() + off, m, total, name, off))
            total += (m + 255) // 256 * 256
    free, _ = torch.cuda.mem_get_info(device)
    if total + (2 << 30) > free:
        return {"unavailable": f"the decoded residuals ({total / 1e9:.1f} GB) do not fit next to the workload"}
    arena = torch.empty(total, dtype=torch.uint8, device=device)
    for i, t in enumerate(spec.tensors):
        a = synth.teacher1_tensor(t, i, device)
        b = synth.perturb_(a.clone(), t, i, scale)
        av, bv = a.reshape(-1).view(torch.uint8), b.reshape(-1).view(torch.uint8)
        for mode, _, m, at, name, off in (p for p in packets if p[4] == t.name):
            dst = arena[at : at + m]
            x = torch.bitwise_xor(av[off : off + m], bv[off : off + m])
            if mode == 1:  # delta.py:186
                dst[: m // 2].copy_(x[0::2])
                dst[m // 2 :].copy_(x[1::2])
            elif mode == 3:  # delta.py:26-34 on the device
                d = (bv[off : off + m].view(torch.int16).to(torch.int32) -
                     av[off : off + m].view(torch.int16).to(torch.int32)) & 0xFFFF
                d = torch.where(d >= 32768, d - 65536, d)
                z = ((d << 1) ^ (d >> 15)) & 0xFFFF
                dst[: m // 2].copy_(z & 0xFF)
                dst[m // 2 :].copy_(z >> 8)
            else:
                dst.copy_(x)
        del a, b
    # Batches of at most 64 MiB of residuals, as _batch_layout bounds them (delta.py:37-57).
    layout = refdelta._batch_layout([(m, m) for _, _, m, _, _, _ in packets])
    launches = []
    for batch in layout:
        rows, tiles_of, base = [], [], None
        for row, (index, _, _) in enumerate(batch["packets"]):
            mode, dst, m, at, _, _ = packets[index]
            base = at if base is None else base
            rows.append((mode, dst, m, at - base, len(tiles_of)))
            tiles_of.extend([row] * ((m + tile - 1) // tile))
        launches.append((arena[base:], torch.tensor(rows, dtype=torch.int64, device=device),
                         torch.tensor(tiles_of, dtype=torch.int32, device=device), len(tiles_of)))
    stream = torch.cuda.current_stream(device)

    def switch(reverse: bool) -> None:
        for view, desc, tp, ntiles in launches:
            refdelta._restore_batch[(ntiles,)](view, view, desc, tp, reverse, tile)

    reverse = state_is_b
    for _ in range(max(2, warmup + warmup % 2)):  # an even number: the weights end where they began
        switch(reverse)
        reverse = not reverse
    n = steps + steps % 2
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(n):
        switch(reverse)
        reverse = not reverse
    end.record(stream)
    torch.cuda.synchronize(device)
    ms = start.elapsed_time(end) / n
    del arena, launches
    torch.cuda.empty_cache()
    verify_all_tensors(spec, gpu, state_is_b, scale, device)
    traffic = 2 * spec.nbytes + total  # read + write weights, read the decoded residuals
    return {
        "ms_per_step": round(ms, 3),
        "value": round(spec.nbytes / (ms * 1e-3) / 1e9, 2),
        "unit": UNIT,
        "launches_per_step": len(layout),
        "algorithmic_bytes": traffic,
        "achieved_gbs": round(traffic / (ms * 1e-3) / 1e9, 1),
        "path": ("reference warpshift/delta.py _restore_batch (Triton) over decoded residuals generated on the device, "
                 "one launch per 64 MiB batch; nvCOMP decode not installed, so not included"),
        "modes": sorted({p[0] for p in packets}),
    }


# --------------------------------------------------------------------------- arms
def run_reference(args) -> None:
    """Reference arm: the reference's switch on the host cores, rank 0 only."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if int(os.environ.get("RANK", "0")) != 0:
        return
    from oracle import reference_cpu

    spec, desc = workload_spec(args, world, 0)
    cores = len(os.sched_getaffinity(0))
    budget = int(args.ref_sample_gb * 1e9)
    tensors, packets, total = reference_workload(spec, args.scale, args.policy, budget, cores)
    sw = reference_cpu.CpuSwitch(tensors, packets)
    for _ in range(args.warmup):
        sw.switch()
    times = [sw.switch() for _ in range(args.steps)]
    elapsed = sum(times)
    value = args.steps * total / elapsed / 1e9
    whole = total >= spec.nbytes
    sample = (f"{'the whole workload' if whole else f'{len(tensors)} leading tensors of {len(spec.tensors)}'} "
              f"({total / 1e9:.2f} of {spec.nbytes / 1e9:.2f} GB) per step: the reference's restore "
              f"(delta.py:74-92) of the residuals its decode hands over, in the modes its rule picks "
              f"(oracle/reference_cpu.py), {cores} threads")
    modes: dict[int, int] = {}
    for p in packets:
        modes[p[2]] = modes.get(p[2], 0) + 1
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(value, 3),
        "unit": UNIT,
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(elapsed / args.steps * 1e3 * (spec.nbytes / total), 3),
        "higher_is_better": True,
        "scaling": "weak" if args.workload != "llama3-70b" else "strong",
        "vs_baseline": None,
        "dtype": "u16" if args.policy == "u16" else "u8",
        "data": "synthetic (Teacher1 N(0,0.02) seed 0, Teacher2 relative noise seed 1)",
        "config": workload_config(args, desc, spec.nbytes),
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "detail": {
            "sampled_bytes_per_step": total,
            "workload_bytes": spec.nbytes,
            "ms_per_sample_step": round(elapsed / args.steps * 1e3, 3),
            "step_ms": [round(x * 1e3, 2) for x in times],
            "packets_by_mode": {sem_mode: n for sem_mode, n in sorted(modes.items())},
            "ms_per_step_note": "ms_per_step is the sampled step time scaled to the whole workload",
            "native_code": "none of this repository's (NumPy on host threads)",
        },
    }
    print(json.dumps(line), flush=True)


def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    from warpshift_b200.delta import DeltaWeights

    world, rank, local, group = init_distributed(args)
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    spec, desc = workload_spec(args, world, rank)
    # Ranks generate and prepare one at a time: each holds its Teacher1 copy in
    # host memory only during its own turn, so peak host memory is one shard
    # plus the compressed arenas, whatever the number of ranks on the node.
    delta, gpu, prepare_s, cpu_base_line = None, None, 0.0, None
    for turn in range(world):
        if turn == rank:
            cpu_base, gpu = generate_on_device(spec, device, args.scale)
            if rank == 0 and world == 1 and not args.no_cpu_baseline:
                cpu_base_line = reference_cpu_baseline(spec, cpu_base, gpu, args.policy, args.cpu_seconds)
            t0 = time.perf_counter()
            delta = DeltaWeights(cpu_base, gpu, policy=args.policy, threads=args.threads, escapes=args.escapes,
                                 split=args.split)
            prepare_s = time.perf_counter() - t0
            del cpu_base
        if group is not None:
            dist.barrier(group=group)
    stats = delta.stats
    native = delta.native_stats()
    W = stats["runtime_bytes"]
    C = int(native.arena_bytes)
    touched = int(native.touched_bytes)
    meta = int(native.metadata_bytes)
    h2d_gbs, h2d_ms = measure_h2d(device, C, group) if not args.skip_e2e else (float("nan"), 0.0)
    stream = delta.compute_stream

    def barrier():
        if group is not None:
            dist.barrier(group=group)
        torch.cuda.synchronize(device)

    def max_over_ranks(x: float) -> float:
        if group is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
        return float(t.item())

    def sum_over_ranks(x: float) -> float:
        if group is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=device)
        dist.all_reduce(t, group=group)
        return float(t.item())

    def per_rank(values: list[float]) -> list[list[float]]:
        """Every rank's `values`, in rank order (one all-gather)."""
        mine = torch.tensor(values, dtype=torch.float64, device=device)
        if group is None:
            return [mine.tolist()]
        everyone = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(everyone, mine, group=group)
        return [t.tolist() for t in everyone]

    props = torch.cuda.get_device_properties(device)
    gpu_id = f"GPU-{props.uuid}" if getattr(props, "uuid", None) else str(local)
    sampler = ClockSampler(gpu_id)
    # The resident model is Teacher2; each step switches to the other teacher.
    state_is_b = True

    # ---- kernel-only: stream resident in HBM
    delta.set_resident(True)
    for _ in range(args.warmup):
        delta.apply_async(reverse=state_is_b)
        delta.finish()
        state_is_b = not state_is_b
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    launches_k = 0
    k_reverse: list[bool] = []  # direction of each timed step (True: B -> A)
    e_reverse: list[bool] = []
    e_step_ms: list[float] = []
    with sampler:
        barrier()
        t_begin = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        t_begin.record(stream)
        for k in range(args.steps):
            starts[k].record(stream)
            delta.apply_async(reverse=state_is_b)
            ends[k].record(stream)
            k_reverse.append(state_is_b)
            state_is_b = not state_is_b
            launches_k += 1
        t_end.record(stream)
        torch.cuda.synchronize(device)
        delta.finish()
        barrier()
        kernel_ms = t_begin.elapsed_time(t_end)
        step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
        delta.set_resident(False)

        # ---- end to end through DeltaWeights.apply: H2D staging + result read-back each step
        e2e_ms, launches_e = None, 0
        if not args.skip_e2e:
            for _ in range(args.warmup):
                delta.apply(reverse=state_is_b)
                if group is not None:
                    delta.confirm(group)
                state_is_b = not state_is_b
            barrier()
            caller = torch.cuda.current_stream(device)
            e_begin, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e_marks = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
            e_begin.record(caller)
            e_marks[0].record(caller)
            for k in range(args.steps):
                delta.apply(reverse=state_is_b)
                if group is not None:
                    delta.confirm(group)
                e_marks[k + 1].record(caller)
                launches_e += delta.last_apply["launches"]
                e_reverse.append(state_is_b)
                state_is_b = not state_is_b
            e_end.record(caller)
            torch.cuda.synchronize(device)
            barrier()
            e2e_ms = e_begin.elapsed_time(e_end)
            e_step_ms = [a.elapsed_time(b) for a, b in zip(e_marks, e_marks[1:])]
    clocks = sampler.summary()

    full_copy = None
    if args.compare_full_copy:
        # weights.py:65-70 pinned backup, then 77-82 restore: copy_ every tensor, sync.
        backup = {}
        for name, t in gpu.items():
            backup[name] = torch.empty_like(t, device="cpu", pin_memory=True)
            backup[name].copy_(t)
        torch.cuda.synchronize(device)
        caller = torch.cuda.current_stream(device)
        for _ in range(max(1, args.warmup)):
            for name, t in gpu.items():
                t.copy_(backup[name], non_blocking=True)
            torch.cuda.synchronize(device)
        barrier()
        f_begin, f_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f_begin.record(caller)
        for _ in range(args.steps):
            for name, t in gpu.items():
                t.copy_(backup[name], non_blocking=True)
            torch.cuda.synchronize(device)
        f_end.record(caller)
        torch.cuda.synchronize(device)
        barrier()
        f_ms = max_over_ranks(f_begin.elapsed_time(f_end))
        full_copy = {
            "value": round(sum_over_ranks(W) * args.steps / (f_ms * 1e-3) / 1e9, 2),
            "unit": UNIT,
            "ms_per_step": round(f_ms / args.steps, 3),
            "h2d_bytes_per_step": W,
            "path": "pinned full-backup restore (weights.py:65-82): torch copy_ per tensor from pinned host memory",
        }
        del backup

    kernel_ms_max = max_over_ranks(kernel_ms)
    e2e_ms_max = max_over_ranks(e2e_ms) if e2e_ms is not None else None
    W_total = sum_over_ranks(W)
    value = W_total * args.steps / (kernel_ms_max * 1e-3) / 1e9
    e2e_value = W_total * args.steps / (e2e_ms_max * 1e-3) / 1e9 if e2e_ms_max else None
    avg_step_ms = statistics.mean(step_ms)
    algo_bytes = 2 * touched + C + meta
    achieved = algo_bytes / (avg_step_ms * 1e-3) / 1e9
    pk = peaks()
    traffic = None
    traffic_file = ROOT / "profiles" / "ws_apply_kernel_dram_traffic.json"
    if traffic_file.exists() and not args.layers:
        entry = json.loads(traffic_file.read_text()).get(f"{args.workload}/{args.policy}/{args.scale}")
        if entry:
            traffic = entry["dram_bytes_per_launch"]
    # Each rank's end-to-end bound is the time its own stream's copy took with
    # every rank copying at once (or its kernel's HBM bound, when longer); the
    # switch ends with its slowest rank, so the group's bound is their maximum.
    rank_roof_ms = max(h2d_ms, algo_bytes / (pk["hbm_gbs"] * 1e9) * 1e3)
    rank_e2e_ms = e2e_ms / args.steps if e2e_ms is not None else None
    t_roof_ms = max_over_ranks(rank_roof_ms)
    # Per-rank fraction of its own roofline; the minimum over ranks is reported.
    min_rank_frac = -max_over_ranks(-(rank_roof_ms / rank_e2e_ms)) if rank_e2e_ms else None
    h2d_slowest = -max_over_ranks(-h2d_gbs) if h2d_gbs == h2d_gbs else h2d_gbs
    ranks_h2d_e2e_kernel = per_rank([h2d_gbs, rank_e2e_ms if rank_e2e_ms else float("nan"),
                                     kernel_ms / args.steps])
    # On-device per-tensor hashes of the switched weights (the replacement for the
    # acceptance check's D2H sha256), timed over every tensor of this rank.
    from warpshift_b200.verify import tensor_hashes

    tensor_hashes(gpu)
    hs, he = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    hs.record()
    final_hashes = tensor_hashes(gpu)
    he.record()
    torch.cuda.synchronize(device)
    hash_ms = hs.elapsed_time(he)
    # Exactness of the final state: every tensor against its regenerated Teacher,
    # plus the device hashes of the first and last tensor.
    from warpshift_b200 import synth

    verified = verify_all_tensors(spec, gpu, state_is_b, args.scale, device)
    for i in (0, len(spec.tensors) - 1):
        t = spec.tensors[i]
        ref = synth.teacher1_tensor(t, i, device)
        if state_is_b:
            synth.perturb_(ref, t, i, args.scale)
        if tensor_hashes({t.name: ref})[t.name] != final_hashes[t.name]:
            raise RuntimeError(f"device hash of {t.name} differs from the regenerated teacher's")
    verified_total = int(sum_over_ranks(verified))
    ref_gpu = None
    if world == 1 and not args.no_reference_gpu:
        try:
            ref_gpu = reference_triton_restore(spec, gpu, state_is_b, args.scale, args.policy, device, args.steps,
                                               args.warmup)
        except Exception as exc:  # informative leg: report, never fail the bench
            ref_gpu = {"unavailable": f"{type(exc).__name__}: {exc}"[:300]}
    if rank != 0:
        return
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(kernel_ms_max / args.steps, 3),
        "higher_is_better": True,
        "scaling": "weak" if args.workload != "llama3-70b" else "strong",
        "vs_baseline": None,
        "dtype": "u16" if args.policy == "u16" else "u8",
        "data": "synthetic (Teacher1 N(0,0.02) seed 0, Teacher2 relative noise seed 1, generated on the GPU)",
        "config": workload_config(args, desc, spec.nbytes),
        "e2e": None if e2e_value is None else {
            "value": round(e2e_value, 2),
            "unit": UNIT,
            "ms_per_step": round(e2e_ms_max / args.steps, 3),
            "h2d_bytes_per_step": C,
            "d2h_bytes_per_step": 16,
            "h2d_gbs_measured": round(h2d_slowest, 2),
            "h2d_measurement": "each rank copies its stream's size from pinned memory (1 GiB pieces), all ranks "
                               "starting together; slowest rank's rate",
            "roofline_ms": round(t_roof_ms, 3),
            "roofline_frac": round(t_roof_ms / (e2e_ms_max / args.steps), 3),
            "min_rank_roofline_frac": round(min_rank_frac, 3) if min_rank_frac else None,
            "launches": launches_e,
            "median_ms": per_direction(e_step_ms, e_reverse),
        },
        "roofline": {
            "bound": "hbm",
            "achieved": round(achieved, 1),
            "peak": pk["hbm_gbs"],
            "unit": "GB/s",
            "frac": round(achieved / pk["hbm_gbs"], 3),
            "traffic": traffic,
            "algorithmic_bytes_per_launch": algo_bytes,
            "peak_source": pk["source"] + " (MEASURED_PEAKS.json hbm_gbs, burst copy)",
            "kernel": "ws_apply_kernel (fused rANS decode + in-place apply)",
        },
        "verified_tensors": verified_total,
        "reference_gpu_restore": ref_gpu,
        "full_copy": full_copy,
        "tensor_hash": {
            "ms": round(hash_ms, 3),
            "gbs": round(W / (hash_ms * 1e-3) / 1e9, 1),
            "frac_of_hbm_peak": round(W / (hash_ms * 1e-3) / 1e9 / pk["hbm_gbs"], 3),
            "tensors": len(final_hashes),
            "path": "warpshift_b200.verify.tensor_hashes (ws_tensor_hashes), all tensors of the rank, one call",
        },
        "gpu_launches": launches_k + launches_e,
        "clocks": clocks,
        "detail": {
            "parallelism": (f"{world} ranks, each switching its own shard; NCCL all-reduce of per-rank outcomes per "
                            "end-to-end switch") if world > 1 else "1 GPU",
            "weight_bytes_per_rank": W,
            "compressed_bytes_per_rank": C,
            "compression_ratio": round(touched / C, 3) if C else None,
            "touched_bytes_per_rank": touched,
            "prepare_seconds": round(prepare_s, 2),
            "encode_seconds": round(stats["encode_seconds"], 2),
            "encoder": stats.get("encoder"),
            "kernel_step_ms": [round(x, 3) for x in step_ms],
            "kernel_median_ms": per_direction(step_ms, k_reverse),
            "e2e_step_ms": [round(x, 3) for x in e_step_ms],
            "per_rank": [{"h2d_gbs": None if h != h else round(h, 2), "e2e_ms": None if e != e else round(e, 3),
                          "kernel_ms": round(k, 3)} for h, e, k in ranks_h2d_e2e_kernel],
        },
    }
    if cpu_base_line is not None:
        line["cpu_baseline"] = cpu_base_line
    print(json.dumps(line), flush=True)
    delta.close()


def main() -> None:
    args = parse_args()
    if args.warmup < 0 or args.steps < 1:
        raise SystemExit("need --steps >= 1")
    try:
        if args.impl == "reference":
            run_reference(args)
        else:
            run_ours(args)
    finally:
        import torch.distributed as dist

        if dist.is_available() and dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
