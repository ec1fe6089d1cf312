"""SBDA attention fwd+bwd benchmark on B200 (BASELINE.json metric, config 4).

Workload: one 1,048,576-position sequence per GPU, 20 SBDA layers (offsets
(0,1), (0,2), (0,1,2,4) ... (0,1,2,2^19)), 4 heads x 64, bf16, q/k/v/dO ~ N(0,1)
from a seed, in the reference's memory layout ([B,L,H,D] projections viewed
as [B,H,L,D]).  A step is the forward of all 20 layers followed by the
backward of all 20 layers.  Metric: Mpositions/s = positions per GPU x GPUs /
step time.  Each tensor is 512 MiB (> 126 MB L2), so no L2 flush is needed.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Under torchrun each rank runs an independent sequence (batch sharding, no
data-path collective; weak scaling); the timed region is bracketed by a
barrier and synchronize on every rank and the slowest rank's time is used.
The same JSON line carries the other configurations as blocks: ``cfg2`` (one
layer at B 4 x 8 heads x 32,768, one GPU), ``cfg3_batch_head`` (15 layers at
B 8 x 8 heads x 32,768 with the (batch, head) sequences split across the
ranks: strong scaling) and ``cfg5_seqshard`` (one 4,194,304-position sequence
x 22 layers in contiguous shards across the ranks, halos over NVLink: strong
scaling).  ``--impl reference`` times the reference's algorithm (the CPU
oracle port of ``BiAttn/left_v2.py``'s exact path) on the host cores instead.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

METRIC = "SBDA attn fwd+bwd Mpositions/s at 1M×20L; % of B200 HBM roofline"
UNIT = "Mpositions/s"
FALLBACK_HBM_GBS = 6650.0
PEER_LINK_GBS = 770.0  # measured peer copy per direction on this pool (nominal 900)
# CPU sample length of both CPU legs (the cpu_baseline object and --impl reference): 65,536
# positions with every layer's offsets; the gather path is O(L) per layer, so positions/s carries
# over to 1M.  At 65,536 positions every layer up to 2^15 has live far sources.
CPU_SAMPLE_POSITIONS = 65536


def parse_args():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=30)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=("b200", "reference"), default="b200")
    p.add_argument("--workload", choices=("cfg4", "cfg5", "block", "normed", "backbone", "gqa"), default="cfg4",
                   help="cfg4 (default, the metric): one 1M-position sequence per GPU; cfg5: one "
                        "4M-position, 22-layer sequence split into contiguous shards across the GPUs")
    p.add_argument("--length", type=int, default=1 << 20)
    p.add_argument("--layers", type=int, default=20)
    p.add_argument("--layer-list", type=str, default="",
                   help="comma-separated subset of layers to run (profiling cases); default all")
    p.add_argument("--heads", type=int, default=4)
    p.add_argument("--head-dim", type=int, default=64)
    p.add_argument("--e2e-steps", type=int, default=3)
    p.add_argument("--e2e-copy-streams", type=int, default=1,
                   help="copy streams per direction in the e2e leg (a layer's tensors alternate between them); "
                        "1, 2 and 3 measured alike, 40-43 GB/s host-to-device: the host link is the bound")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-blocks", action="store_true",
                   help="skip the config-2, config-3 and config-5 blocks of the default line")
    p.add_argument("--cpu-sample-length", type=int, default=CPU_SAMPLE_POSITIONS)
    return p.parse_args()


def workload_config(args, world: int) -> dict:
    return {
        "workload": (f"cfg4: SBDA attention stack fwd+bwd, {args.length} positions x {args.layers} layers, "
                     f"{args.heads} heads x {args.head_dim}, batch 1 per GPU"),
        "global_batch": world,
        "seq_len": args.length,
        "layers": args.layers,
        "heads": args.heads,
        "head_dim": args.head_dim,
        "parallelism": f"batch-sharded x{world} (independent sequences, no collectives)",
        "l2": "every tensor 512 MiB > 126 MB L2; no flush needed",
        "cpu_sample_positions": args.cpu_sample_length,
    }


def measured_peak_gbs() -> tuple[float, str]:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as handle:
            return float(json.load(handle)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


# DRAM bytes per (batch, head, position) row of one windowed backward launch (dram__bytes_read.sum
# + dram__bytes_write.sum), measured by ncu on a small case of the same kernel: 262,144 positions
# x 4 heads x 64, bf16, layers 4, 10 and 17 (local and chain walks), averaged over the three
# launches.  Traffic grows in proportion to the rows, so a full launch's traffic is this figure
# times its rows.  The capture command and the per-launch figures are in
# profiles/sbda_bwd_kernel_small_case.md.
BWD_DRAM_BYTES_PER_ROW: float | None = 884.2


def backward_traffic(rows: int) -> float | None:
    """Per-launch DRAM traffic of the windowed backward for ``rows`` rows (see above)."""
    return None if BWD_DRAM_BYTES_PER_ROW is None else BWD_DRAM_BYTES_PER_ROW * rows


def shard_link_model(total: int, world: int, heads: int, head_dim: int, elem: int, offsets_per_layer,
                     hbm_gbs: float, link_gbs: float = PEER_LINK_GBS) -> dict:
    """Bytes that must cross NVLink in one fwd+bwd step of contiguous sequence shards, and the
    step time they allow.

    Per layer with far offset d, rank r (shard [a, a + S)) reads from other ranks:
      * forward and backward: K and V of the far sources of its rows i with 0 <= i - d < a
        (2 * D * e bytes per row and head, once in each pass);
      * backward: for its keys j whose far consumer j + d lies past its shard (and inside the
        sequence), that consumer's Q, dO, K, V and LSE (4 * D * e + 4 bytes), because the far
        consumers of a rank's keys are recomputed on the key's rank.
    The 1- and 2-row near halos at shard ends are left out (under 0.01 % of the bytes).  A layer
    takes at least max(local algorithmic bytes / HBM peak, remote bytes / link bandwidth) on each
    rank; the step target is the sum over layers of the slowest rank's bound.
    """
    shard = total // world
    local = shard * heads * (11 * head_dim * elem + 8)
    worst_remote, target_s = 0, 0.0
    for offsets in offsets_per_layer:
        d = max(offsets)
        if d < 3:
            target_s += local / (hbm_gbs * 1e9)
            continue
        layer_bound = 0.0
        for rank in range(world):
            a = rank * shard
            far_rows = max(0, min(a + shard, a + d) - max(a, d))
            consumer_rows = max(0, min(a + shard, total - d) - max(a, a + shard - d))
            remote = heads * (2 * far_rows * 2 * head_dim * elem + consumer_rows * (4 * head_dim * elem + 4))
            worst_remote = max(worst_remote, remote)
            layer_bound = max(layer_bound, local / (hbm_gbs * 1e9), remote / (link_gbs * 1e9))
        target_s += layer_bound
    return {"link_gbs": link_gbs, "max_remote_bytes_one_layer": worst_remote, "target_ms": target_s * 1e3}


class ClockSampler:
    """Samples nvidia-smi clocks / throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int) -> None:
        self.proc = None
        try:
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            ident = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", ident, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, RuntimeError):
            self.proc = None

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, smax, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in out.splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for name, value in zip(names, parts[5:9]):
                if value.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax), "reasons": sorted(reasons),
                "samples": len(sm)}


def cpu_baseline(args, *, sample_length: int, threads: int | None = None) -> dict:
    """Oracle port of the reference's exact path (fp32, CPU) over all layers at a bounded length."""
    from oracle import sbda_oracle as orc

    if threads:
        torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(7)
    shape = (1, args.heads, sample_length, args.head_dim)
    q, k, v, do = (torch.randn(shape, generator=g) for _ in range(4))
    orc.exact_attention_grads(q[:, :, :256], k[:, :, :256], v[:, :, :256], (0, 1, 2, 4), do[:, :, :256])
    start = time.perf_counter()
    for layer in range(1, args.layers + 1):
        offsets = orc.schedule_offsets(layer, "sbda", args.layers)
        orc.exact_attention_grads(q, k, v, offsets, do)
    elapsed = time.perf_counter() - start
    return {"value": sample_length / elapsed / 1e6, "unit": UNIT, "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": (f"oracle port of left_v2 exact path (torch CPU fp32), fwd+bwd of all {args.layers} "
                       f"layers at {sample_length} positions x {args.heads} heads x {args.head_dim}; "
                       "O(N) per layer, so positions/s carries to 1M"),
            "seconds": elapsed}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    from oracle import sbda_oracle as orc

    torch.set_num_threads(os.cpu_count() or 1)
    sample = args.cpu_sample_length
    g = torch.Generator().manual_seed(7)
    shape = (1, args.heads, sample, args.head_dim)
    q, k, v, do = (torch.randn(shape, generator=g) for _ in range(4))
    layer_offsets = [orc.schedule_offsets(layer, "sbda", args.layers) for layer in range(1, args.layers + 1)]

    def step():
        for offsets in layer_offsets:
            orc.exact_attention_grads(q, k, v, offsets, do)

    for _ in range(args.warmup):
        step()
    start = time.perf_counter()
    for _ in range(args.steps):
        step()
    elapsed = (time.perf_counter() - start) / max(1, args.steps)
    value = sample / elapsed / 1e6
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": elapsed * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic N(0,1), seeded",
        "config": workload_config(args, world),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
                         "sample": (f"each step: oracle port of left_v2 exact path (torch CPU fp32), fwd+bwd of "
                                    f"all {args.layers} layers at {sample} positions x {args.heads} heads x "
                                    f"{args.head_dim}; the reference ships no native CPU code")},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_b200(args) -> None:
    import torch.distributed as dist

    import sbda_b200
    from sbda_b200 import ops

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime

        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(value: float) -> float:
        if world == 1:
            return value
        t = torch.tensor([value], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    L, H, D, layers = args.length, args.heads, args.head_dim, args.layers
    dtype = torch.bfloat16
    offsets = sbda_b200.sbda_layer_offsets(layers)
    if args.layer_list:
        offsets = [offsets[int(x) - 1] for x in args.layer_list.split(",")]
        layers = len(offsets)
    gen = torch.Generator(device=device).manual_seed(1234 + rank)

    def blhd():
        return torch.randn((1, L, H, D), device=device, dtype=dtype, generator=gen).permute(0, 2, 1, 3)

    qs = [blhd() for _ in range(layers)]
    ks = [blhd() for _ in range(layers)]
    vs = [blhd() for _ in range(layers)]
    dos = [blhd() for _ in range(layers)]
    lses = [torch.empty((1, H, L), device=device, dtype=torch.float32) for _ in range(layers)]
    out = torch.empty_like(qs[0])
    grads = (torch.empty_like(qs[0]), torch.empty_like(qs[0]), torch.empty_like(qs[0]))
    fwd_events, bwd_events = [], []

    def step(record: bool = False):
        for layer in range(layers):
            if record:
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record()
            ops.sbda_forward(qs[layer], ks[layer], vs[layer], offsets[layer], out=out, lse=lses[layer])
            if record:
                e.record()
                fwd_events.append((s, e))
        for layer in reversed(range(layers)):
            if record:
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record()
            ops.sbda_backward(qs[layer], ks[layer], vs[layer], dos[layer], lses[layer], offsets[layer],
                              grads=grads)
            if record:
                e.record()
                bwd_events.append((s, e))

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    if sbda_b200.device_status(reset=True):
        raise RuntimeError("device fault reported during warm-up")

    # Timed region: steps back to back, bracketed by barrier + synchronize.
    barrier()
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    time.sleep(0.3)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.steps):
        step()
    end.record()
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop()
    step_ms = max_over_ranks(start.elapsed_time(end) / args.steps)

    # Per-kernel durations (separate pass with an event pair around every launch).
    for _ in range(2):
        step(record=True)
    torch.cuda.synchronize()
    fwd_ms = statistics.mean(s.elapsed_time(e) for s, e in fwd_events)
    bwd_ms = statistics.mean(s.elapsed_time(e) for s, e in bwd_events)
    # per-layer launch times (forward in layer order; backward recorded in reverse)
    n_rec = len(fwd_events) // layers
    fwd_layer_ms = [statistics.mean(fwd_events[k * layers + j][0].elapsed_time(fwd_events[k * layers + j][1])
                                    for k in range(n_rec)) for j in range(layers)]
    bwd_layer_ms = [statistics.mean(bwd_events[k * layers + (layers - 1 - j)][0].elapsed_time(
        bwd_events[k * layers + (layers - 1 - j)][1]) for k in range(n_rec)) for j in range(layers)]

    # Host time to issue one step's 40 launches (no synchronisation inside), median of 3.
    host_ms = []
    for _ in range(3):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        step()
        host_ms.append((time.perf_counter() - t0) * 1e3)
    torch.cuda.synchronize()
    host_ms = statistics.median(host_ms)

    # The same step captured once as a CUDA graph and replayed: the same 40 kernels on the same
    # buffers, without the per-launch host work (planning, tensor-map encoding, ctypes calls).
    graph_info = None
    try:
        side = torch.cuda.Stream(device)
        side.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(side):
            step()
        torch.cuda.current_stream(device).wait_stream(side)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        for _ in range(max(3, args.warmup)):
            graph.replay()
        barrier()
        torch.cuda.synchronize()
        gs, ge = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        gs.record()
        for _ in range(args.steps):
            graph.replay()
        ge.record()
        torch.cuda.synchronize()
        barrier()
        graph_ms = max_over_ranks(gs.elapsed_time(ge) / args.steps)
        graph_info = {"ms_per_step": graph_ms, "value": L * world / (graph_ms * 1e-3) / 1e6, "unit": UNIT}
        del graph
    except RuntimeError as err:  # reported, not fatal for the bench line
        graph_info = {"error": str(err).splitlines()[0][:200]}

    rows = H * L
    e = 2
    fwd_bytes = rows * (4 * D * e + 4)
    bwd_bytes = rows * (7 * D * e + 4)
    peak, peak_kind = measured_peak_gbs()
    positions = L * world
    value = positions / (step_ms * 1e-3) / 1e6
    dominant = ("sbda_bwd_kernel", bwd_bytes, bwd_ms) if bwd_ms >= fwd_ms else ("sbda_fwd_kernel", fwd_bytes, fwd_ms)
    achieved = dominant[1] / (dominant[2] * 1e-3) / 1e9
    traffic = backward_traffic(rows) if dominant[0] == "sbda_bwd_kernel" else None
    step_bytes = layers * (fwd_bytes + bwd_bytes)
    step_gbs = step_bytes / (step_ms * 1e-3) / 1e9

    e2e = None
    if not args.no_e2e:
        e2e = measure_e2e(args, device, offsets, barrier, max_over_ranks, world)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(args, sample_length=args.cpu_sample_length, threads=os.cpu_count())
        cpu.pop("seconds", None)

    # The other configurations, as blocks of the same line (the headline stays config 4).
    blocks = {}
    if not args.no_blocks:
        del qs, ks, vs, dos, lses, out, grads
        torch.cuda.empty_cache()
        block_steps = max(5, min(args.steps, 20))
        if world == 1:
            blocks["cfg2"] = cfg2_block(device, block_steps, args.warmup, peak)
            torch.cuda.empty_cache()
            blocks["cfg4_norm_rope_attention"] = norm_rope_attention_block(device, max(3, min(args.steps, 10)),
                                                                           args.warmup, peak)
            torch.cuda.empty_cache()
            blocks["cfg4_backbone_vs_dense"] = backbone_block(device, 3, args.warmup)
            torch.cuda.empty_cache()
            blocks["gqa"] = gqa_block(device, max(3, min(args.steps, 10)), args.warmup, peak)
            torch.cuda.empty_cache()
        blocks["cfg3_batch_head"] = cfg3_block(device, world, rank, block_steps, args.warmup, peak, barrier,
                                               max_over_ranks)
        torch.cuda.empty_cache()
        blocks["cfg5_seqshard"] = seqshard_block(device, world, rank, max(3, min(args.steps, 10)), args.warmup,
                                                 peak)
        torch.cuda.empty_cache()

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": max(3, args.warmup), "ms_per_step": step_ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic N(0,1), seeded, resident in HBM",
            "config": workload_config(args, world),
            "roofline": {"bound": "hbm", "kernel": dominant[0], "achieved": achieved, "peak": peak,
                         "unit": "GB/s", "frac": achieved / peak, "peak_kind": peak_kind,
                         "traffic": traffic, "algorithmic_bytes_per_launch": dominant[1],
                         "launch_ms": dominant[2]},
            "step_roofline": {"achieved": step_gbs, "peak": peak, "unit": "GB/s", "frac": step_gbs / peak,
                              "algorithmic_bytes_per_step": step_bytes, "fwd_launch_ms": fwd_ms,
                              "bwd_launch_ms": bwd_ms,
                              "fwd_layer_ms": [round(x, 4) for x in fwd_layer_ms],
                              "bwd_layer_ms": [round(x, 4) for x in bwd_layer_ms],
                              "sum_launch_ms": layers * (fwd_ms + bwd_ms),
                              "gap_ms": step_ms - layers * (fwd_ms + bwd_ms),
                              "gap_note": ("step time minus the per-launch event times; an event pair around "
                                           "every launch serialises the kernels, so the sum can exceed the "
                                           "back-to-back step and the gap be negative"),
                              "host_enqueue_ms_per_step": host_ms},
            "graph_replay": graph_info,
            "clocks": clocks,
            "e2e": e2e,
            "cpu_baseline": cpu,
            "gpu_launches": 2 * layers * args.steps,
        }
        line.update(blocks)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def measure_e2e(args, device, offsets, barrier, max_over_ranks, world) -> dict:
    """Public API (fused_sbda_key_backward + autograd) with pinned host buffers.

    Every layer of every step copies q, k, v, dO host->device and dQ, dK, dV
    device->host inside the timed region.  The copies run on side streams
    (PCIe is full duplex; ``--e2e-copy-streams`` per direction, a layer's
    tensors alternating between them): layer l+1's inputs land in the second
    of two device buffer sets while layer l computes, and layer l's gradients
    drain while layer l+1 computes; events order every buffer reuse.
    """
    import sbda_b200

    L, H, D, layers = args.length, args.heads, args.head_dim, len(offsets)
    g = torch.Generator().manual_seed(99)
    host_in = [torch.randn((1, L, H, D), generator=g).to(torch.bfloat16).pin_memory() for _ in range(4)]
    host_out = [torch.empty((1, L, H, D), dtype=torch.bfloat16).pin_memory() for _ in range(3)]
    dev_sets = [[torch.empty((1, L, H, D), device=device, dtype=torch.bfloat16) for _ in range(4)]
                for _ in range(2)]
    off_tensors = [torch.tensor(o, dtype=torch.int32, device=device) for o in offsets]
    compute = torch.cuda.current_stream(device)
    n_copy = max(1, args.e2e_copy_streams)
    h2d = [torch.cuda.Stream(device) for _ in range(n_copy)]
    d2h = [torch.cuda.Stream(device) for _ in range(n_copy)]

    def step():
        # per buffer set: inputs landed (one event per copy stream), compute done with it
        ready = [[torch.cuda.Event() for _ in h2d] for _ in range(2)]
        freed = [torch.cuda.Event(), torch.cuda.Event()]
        for st in h2d + d2h:
            st.wait_stream(compute)

        def load(layer):
            s = layer % 2
            for i, st in enumerate(h2d):
                with torch.cuda.stream(st):
                    if layer >= 2:
                        st.wait_event(freed[s])
                    for j in range(i, len(host_in), n_copy):
                        dev_sets[s][j].copy_(host_in[j], non_blocking=True)
                    ready[s][i].record(st)

        load(0)
        for layer in range(layers):
            s = layer % 2
            if layer + 1 < layers:
                load(layer + 1)
            for ev in ready[s]:
                compute.wait_event(ev)
            q, k, v = (t.permute(0, 2, 1, 3).requires_grad_() for t in dev_sets[s][:3])
            out = sbda_b200.fused_sbda_key_backward(q, k, v, off_tensors[layer])
            out.backward(dev_sets[s][3].permute(0, 2, 1, 3))
            freed[s].record(compute)
            grads = (q.grad, k.grad, v.grad)
            for i, st in enumerate(d2h):
                st.wait_stream(compute)
                with torch.cuda.stream(st):
                    for j in range(i, len(grads), n_copy):
                        host_out[j].copy_(grads[j].permute(0, 2, 1, 3), non_blocking=True)
                for j in range(i, len(grads), n_copy):
                    grads[j].record_stream(st)
        for st in h2d + d2h:
            compute.wait_stream(st)

    step()
    torch.cuda.synchronize()
    steps = max(1, args.e2e_steps)
    barrier()
    torch.cuda.synchronize()
    marks = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    marks[0].record()
    for i in range(steps):
        step()
        marks[i + 1].record()
    torch.cuda.synchronize()
    barrier()
    per_step = [marks[i].elapsed_time(marks[i + 1]) for i in range(steps)]
    ms = max_over_ranks(marks[0].elapsed_time(marks[-1]) / steps)
    tensor_bytes = L * H * D * 2
    return {"value": L * world / (ms * 1e-3) / 1e6, "unit": UNIT, "h2d_bytes_per_step": 4 * tensor_bytes * layers,
            "d2h_bytes_per_step": 3 * tensor_bytes * layers, "ms_per_step": ms, "steps": steps,
            "ms_per_step_min_max": [min(per_step), max(per_step)],
            "api": "sbda_b200.fused_sbda_key_backward + autograd backward, pinned host buffers; "
                   f"copies on {n_copy} side stream(s) per direction, overlapped with compute"}


class L2Flush:
    """Writes a 256 MiB buffer (more than the 126 MB L2) so the next step starts from DRAM."""

    def __init__(self, device) -> None:
        self.buf = torch.empty(256 << 20, dtype=torch.uint8, device=device)
        self.n = 0

    def __call__(self) -> None:
        self.n += 1
        self.buf.fill_(self.n & 0xFF)


def timed_steps(step, steps: int, warmup: int, flush: L2Flush | None) -> float:
    """Mean CUDA-event time (ms) of ``step`` over ``steps`` runs after ``warmup`` untimed ones;
    with ``flush``, L2 is flushed before every run, outside the event pair."""
    for _ in range(max(3, warmup)):
        step()
    events = []
    for _ in range(steps):
        if flush is not None:
            flush()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        step()
        e.record()
        events.append((s, e))
    torch.cuda.synchronize()
    return statistics.mean(s.elapsed_time(e) for s, e in events)


def _blhd(shape_blhd, device, gen, dtype=torch.bfloat16):
    """q/k/v-like [B, H, L, D] view of a [B, L, H, D] tensor (the projections' layout)."""
    return torch.randn(shape_blhd, device=device, dtype=dtype, generator=gen).permute(0, 2, 1, 3)


def cfg2_block(device, steps: int, warmup: int, peak: float) -> dict:
    """Config 2: one SBDA layer (l = 10: offsets 0, 1, 2, 512), B 4 x 8 heads x 64, L 32,768, bf16,
    forward + backward; L2 flushed between steps (every tensor is ~134 MB, about the L2 size)."""
    import sbda_b200
    from sbda_b200 import ops

    B, H, L, D = 4, 8, 32768, 64
    offsets = sbda_b200.topology_offsets(10, topology="sbda")
    gen = torch.Generator(device=device).manual_seed(10)
    q, k, v, do = (_blhd((B, L, H, D), device, gen) for _ in range(4))
    out, lse = torch.empty_like(q), torch.empty((B, H, L), device=device, dtype=torch.float32)
    grads = (torch.empty_like(q), torch.empty_like(k), torch.empty_like(v))
    flush = L2Flush(device)
    fwd = lambda: ops.sbda_forward(q, k, v, offsets, out=out, lse=lse)  # noqa: E731
    bwd = lambda: ops.sbda_backward(q, k, v, do, lse, offsets, grads=grads)  # noqa: E731
    fwd_ms = timed_steps(fwd, steps, warmup, flush)
    bwd_ms = timed_steps(bwd, steps, warmup, flush)
    step_ms = timed_steps(lambda: (fwd(), bwd()), steps, warmup, flush)
    rows = B * H * L
    fb, bb = rows * (4 * D * 2 + 4), rows * (7 * D * 2 + 4)
    return {
        "workload": "cfg2: SBDA layer 10 (offsets 0,1,2,512), B 4 x 8 heads x 64, L 32768, bf16, fwd+bwd",
        "value": B * L / (step_ms * 1e-3) / 1e6, "unit": UNIT, "ms_per_step": step_ms,
        "l2": "256 MiB buffer written before every timed step",
        "roofline": {"bound": "hbm", "peak": peak, "unit": "GB/s",
                     "fwd": {"ms": fwd_ms, "achieved": fb / (fwd_ms * 1e-3) / 1e9,
                             "frac": fb / (fwd_ms * 1e-3) / 1e9 / peak, "algorithmic_bytes": fb},
                     "bwd": {"ms": bwd_ms, "achieved": bb / (bwd_ms * 1e-3) / 1e9,
                             "frac": bb / (bwd_ms * 1e-3) / 1e9 / peak, "algorithmic_bytes": bb},
                     "step": {"achieved": (fb + bb) / (step_ms * 1e-3) / 1e9,
                              "frac": (fb + bb) / (step_ms * 1e-3) / 1e9 / peak}},
        "gpu_launches": 2 * steps,
    }


def gqa_block(device, steps: int, warmup: int, peak: float, length: int = 1 << 20, layers: int = 20, heads: int = 4,
              kv_heads: int = 2) -> dict:
    """Grouped-query attention at the config-4 shape: 4 query heads sharing 2 kv heads, 64 wide,
    bf16, fwd+bwd of all 20 SBDA layers (``fused_sbda_gqa_key_backward``'s op through the C
    ABI).  Both directions run on the windowed kernels with K/V rows from kv head h / G; the
    backward writes fp32 per-query-head dK/dV partials to a workspace and sums each group in a
    fixed order (``sbda_b200_backward_grouped``).  Algorithmic bytes per (position, query head)
    row: Q, dO, O, dQ at 2 * 64 B each plus K, V, dK, dV once per kv head, and the fp32 LSE written
    and read; the partials' round trip (2 x 4 x 64 B written and read per query row) is not
    algorithmic and counts against the fraction."""
    import sbda_b200
    from sbda_b200 import ops

    D = 64
    offsets = sbda_b200.sbda_layer_offsets(layers)
    gen = torch.Generator(device=device).manual_seed(9)
    qs = [_blhd((1, length, heads, D), device, gen) for _ in range(layers)]
    dos = [_blhd((1, length, heads, D), device, gen) for _ in range(layers)]
    ks = [_blhd((1, length, kv_heads, D), device, gen) for _ in range(layers)]
    vs = [_blhd((1, length, kv_heads, D), device, gen) for _ in range(layers)]
    lses = [torch.empty((1, heads, length), device=device, dtype=torch.float32) for _ in range(layers)]
    out = torch.empty_like(qs[0])
    grads = (torch.empty_like(qs[0]), torch.empty_like(ks[0]), torch.empty_like(vs[0]))

    def fwd():
        for layer in range(layers):
            ops.sbda_forward(qs[layer], ks[layer], vs[layer], offsets[layer], out=out, lse=lses[layer])

    def bwd():
        for layer in reversed(range(layers)):
            ops.sbda_backward(qs[layer], ks[layer], vs[layer], dos[layer], lses[layer], offsets[layer], grads=grads)

    fwd_ms = timed_steps(fwd, steps, warmup, None)
    bwd_ms = timed_steps(bwd, steps, warmup, None)
    e = 2
    q_rows, kv_rows = length * heads * layers, length * kv_heads * layers
    fwd_bytes = q_rows * (2 * D * e + 4) + kv_rows * 2 * D * e
    bwd_bytes = q_rows * (4 * D * e + 4) + kv_rows * 4 * D * e
    return {
        "workload": (f"GQA: {length} positions x {layers} layers, {heads} query heads / {kv_heads} kv heads x {D}, "
                     "bf16, fwd+bwd"),
        "value": length / ((fwd_ms + bwd_ms) * 1e-3) / 1e6, "unit": UNIT, "ms_per_step": fwd_ms + bwd_ms,
        "fwd_ms": fwd_ms, "bwd_ms": bwd_ms,
        "kernels": ("windowed kernels both ways (K/V from kv head h / G); backward: fp32 per-query-head dK/dV "
                    "partials, then a fixed-order group sum"),
        "l2": "every q/dO tensor 512 MiB, k/v 256 MiB > 126 MB L2",
        "roofline": {"bound": "hbm", "peak": peak, "unit": "GB/s",
                     "fwd_frac": fwd_bytes / (fwd_ms * 1e-3) / 1e9 / peak,
                     "bwd_frac": bwd_bytes / (bwd_ms * 1e-3) / 1e9 / peak},
        "gpu_launches": 2 * layers * steps,
    }


def backbone_block(device, steps: int, warmup: int, length: int = 1 << 20, layers: int = 20, dim: int = 256,
                   heads: int = 4, ffn: int = 1024) -> dict:
    """Config 4's forward comparison, as the reference's protocol runs it
    (``BinaryDiffusionAttention/bench_gemm_breakdown.py:120-209``: ``forward_hidden`` of a
    ``BiAttnLM``, no vocabulary head, bf16, batch 1).  The shape is config 4's: 1,048,576 positions,
    20 layers, d_model 256, 4 heads x 64, FFN 1024.  Timed on the same GPU:

    * the whole backbone forward (``sbda_b200.BiAttnLM`` in bf16: norms, projections, SBDA
      attention, SwiGLU FFN);
    * the 20 SBDA attention forwards alone (the C-ABI op on q/k/v of this shape);
    * dense causal attention: torch's scaled_dot_product_attention(is_causal=True) on the same
      q/k/v.  It is timed on one layer, since its cost does not depend on the layer, and counted
      20 times.  The dense backbone is the SBDA backbone with the SBDA attention time replaced by
      the dense one.
    """
    import torch.nn.functional as F

    import sbda_b200
    from sbda_b200 import ops

    torch.manual_seed(1)
    cfg = sbda_b200.BiAttnConfig(vocab_size=6400, dim=dim, layers=layers, heads=heads, ff_hidden=ffn,
                                 attention_backend="sbda")
    model = sbda_b200.BiAttnLM(cfg).to(device=device, dtype=torch.bfloat16).eval()
    gen = torch.Generator(device=device).manual_seed(5)
    ids = torch.randint(6400, (1, length), device=device, generator=gen)
    head_dim = dim // heads
    q, k, v = (_blhd((1, length, heads, head_dim), device, gen) for _ in range(3))
    out, lse = torch.empty_like(q), torch.empty((1, heads, length), device=device, dtype=torch.float32)
    offsets = sbda_b200.sbda_layer_offsets(layers)
    result = {"workload": (f"cfg4 forward: BiAttnLM.forward_hidden, {length} positions x {layers} layers, d_model {dim}, "
                           f"{heads} heads x {head_dim}, FFN {ffn}, bf16, batch 1 (no vocabulary head)"),
              "unit": "ms"}
    with torch.inference_mode():
        result["backbone_fwd_ms"] = timed_steps(lambda: model.forward_hidden(ids), steps, warmup, None)
        result["sbda_attention_fwd_ms"] = timed_steps(
            lambda: [ops.sbda_forward(q, k, v, offsets[layer], out=out, lse=lse) for layer in range(layers)],
            steps, warmup, None)
        del model
        torch.cuda.empty_cache()
        try:
            dense_layer = timed_steps(lambda: F.scaled_dot_product_attention(q, k, v, is_causal=True), 2, 1, None)
            result["dense_attention_fwd_ms"] = dense_layer * layers
            result["dense_attention_fwd_ms_one_layer"] = dense_layer
            result["dense_backbone_fwd_ms"] = (result["backbone_fwd_ms"] - result["sbda_attention_fwd_ms"]
                                               + result["dense_attention_fwd_ms"])
            result["attention_speedup_vs_dense"] = result["dense_attention_fwd_ms"] / result["sbda_attention_fwd_ms"]
            result["backbone_speedup_vs_dense"] = result["dense_backbone_fwd_ms"] / result["backbone_fwd_ms"]
        except (RuntimeError, torch.OutOfMemoryError) as err:  # reported, not fatal for the bench line
            result["dense_attention_error"] = str(err).splitlines()[0][:200]
    result["value"] = length / (result["backbone_fwd_ms"] * 1e-3) / 1e6
    result["value_unit"] = "Mpositions/s (backbone forward)"
    return result


def norm_rope_attention_block(device, steps: int, warmup: int, peak: float, length: int = 1 << 20, heads: int = 4,
                              layers: int = 20) -> dict:
    """Config 4 with the q/k per-head RMSNorm + RoPE in the step (what ``SBDAttention`` runs
    between its projections and its output projection), forward + backward of all 20 layers, two
    routes on the same seeded inputs through the public API:

    * fused: ``normed_attention`` -- one kernel each way, norm + RoPE inside the attention kernels;
    * separate: ``norm_rope`` on q and on k, then ``fused_sbda_key_backward`` -- five kernels each
      way, the normalised q / k written to and read back from HBM.

    Algorithmic bytes per (position, head) row: fused 1,416 (the attention's; q/k arrive raw and
    dq/dk leave raw); separate adds norm + RoPE forward (read and write q and k: 4 x 128 B) and
    backward (read x and dy, write dx for q and k: 6 x 128 B) for 2,696."""
    import sbda_b200

    D = 64
    offsets = sbda_b200.sbda_layer_offsets(layers)
    gen = torch.Generator(device=device).manual_seed(400)
    qs, ks, vs, dos = ([_blhd((1, length, heads, D), device, gen) for _ in range(layers)] for _ in range(4))
    wq = torch.rand(D, device=device, generator=gen) + 0.5
    wk = torch.rand(D, device=device, generator=gen) + 0.5
    for layer in range(layers):
        if not sbda_b200.normed_supported(qs[layer], ks[layer], vs[layer], offsets[layer]):
            raise RuntimeError(f"layer {layer + 1} is not served by the fused kernels")

    def fused():
        for layer in range(layers):
            q, k, v = (t.detach().requires_grad_() for t in (qs[layer], ks[layer], vs[layer]))
            w1, w2 = wq.detach().requires_grad_(), wk.detach().requires_grad_()
            sbda_b200.normed_attention(q, k, v, w1, w2, offsets[layer]).backward(dos[layer])

    def separate():
        for layer in range(layers):
            q, k, v = (t.detach().requires_grad_() for t in (qs[layer], ks[layer], vs[layer]))
            w1, w2 = wq.detach().requires_grad_(), wk.detach().requires_grad_()
            qn = sbda_b200.norm_rope(q.permute(0, 2, 1, 3), w1).permute(0, 2, 1, 3)
            kn = sbda_b200.norm_rope(k.permute(0, 2, 1, 3), w2).permute(0, 2, 1, 3)
            sbda_b200.fused_sbda_key_backward(qn, kn, v, offsets[layer]).backward(dos[layer])

    fused_ms = timed_steps(fused, steps, warmup, None)
    separate_ms = timed_steps(separate, steps, warmup, None)
    rows = length * heads * layers
    fused_bytes, separate_bytes = rows * (11 * D * 2 + 8), rows * (21 * D * 2 + 8)
    return {
        "workload": (f"cfg4 + per-head RMSNorm + RoPE of q and k: {length} positions x {layers} layers, {heads} "
                     f"heads x {D}, bf16, fwd+bwd through the public API"),
        "value": length / (separate_ms * 1e-3) / 1e6, "unit": UNIT,
        "value_route": "separate (SBDAttention's default route)",
        "fused_ms_per_step": fused_ms, "separate_ms_per_step": separate_ms,
        "speedup_fused_vs_separate": separate_ms / fused_ms,
        "fused_Mpositions_s": length / (fused_ms * 1e-3) / 1e6,
        "separate_Mpositions_s": length / (separate_ms * 1e-3) / 1e6,
        "l2": "every tensor 512 MiB > 126 MB L2",
        "roofline": {"bound": "hbm", "peak": peak, "unit": "GB/s",
                     "fused": {"algorithmic_bytes_per_step": fused_bytes,
                               "achieved": fused_bytes / (fused_ms * 1e-3) / 1e9,
                               "frac": fused_bytes / (fused_ms * 1e-3) / 1e9 / peak},
                     "separate": {"algorithmic_bytes_per_step": separate_bytes,
                                  "achieved": separate_bytes / (separate_ms * 1e-3) / 1e9,
                                  "frac": separate_bytes / (separate_ms * 1e-3) / 1e9 / peak}},
        "gpu_launches": {"fused": (2 + 2) * layers * steps, "separate": (2 + 2 + 2 + 2 * 2) * layers * steps},
    }


def cfg3_block(device, world: int, rank: int, steps: int, warmup: int, peak: float, barrier, max_over_ranks) -> dict:
    """Config 3: the paper's training shape, B 8 x 8 heads x 64, L 32,768, 15 SBDA layers, bf16,
    forward + backward of every attention layer, with the B x H (batch, head) sequences split into
    contiguous ranges across the ranks (``sbda_b200.partition``; no data-path collective).  Total
    work is fixed: strong scaling.  L2 flushed before every timed step."""
    import sbda_b200
    from sbda_b200.partition import partitioned_backward, partitioned_forward, unit_range

    B, H, L, D, layers = 8, 8, 32768, 64, 15
    offsets = [sbda_b200.topology_offsets(layer, topology="sbda", total_layers=layers)
               for layer in range(1, layers + 1)]
    gen = torch.Generator(device=device).manual_seed(300)
    qs, ks, vs, dos = ([_blhd((B, L, H, D), device, gen) for _ in range(layers)] for _ in range(4))
    lses = [torch.empty((B, H, L), device=device, dtype=torch.float32) for _ in range(layers)]
    out = torch.empty_like(qs[0])
    grads = (torch.empty_like(qs[0]), torch.empty_like(qs[0]), torch.empty_like(qs[0]))

    def step():
        for layer in range(layers):
            partitioned_forward(qs[layer], ks[layer], vs[layer], offsets[layer], world, rank, out=out, lse=lses[layer])
        for layer in reversed(range(layers)):
            partitioned_backward(qs[layer], ks[layer], vs[layer], dos[layer], lses[layer], offsets[layer], world,
                                 rank, grads=grads)

    barrier()
    ms = max_over_ranks(timed_steps(step, steps, warmup, L2Flush(device)))
    lo, hi = unit_range(B, H, world, rank)
    rank_bytes = (hi - lo) * L * layers * (11 * D * 2 + 8)
    return {
        "workload": (f"cfg3: 15 SBDA layers, B {B} x {H} heads x {D}, L {L}, bf16, fwd+bwd; (batch, head) "
                     f"sequences split into {world} contiguous ranges"),
        "value": B * L / (ms * 1e-3) / 1e6, "unit": UNIT, "ms_per_step": ms, "scaling": "strong",
        "units_per_rank": [unit_range(B, H, world, r)[1] - unit_range(B, H, world, r)[0] for r in range(world)],
        "l2": "256 MiB buffer written before every timed step",
        "roofline": {"bound": "hbm", "achieved_per_gpu": rank_bytes / (ms * 1e-3) / 1e9, "peak": peak,
                     "unit": "GB/s", "frac": rank_bytes / (ms * 1e-3) / 1e9 / peak},
        "gpu_launches": 2 * layers * steps,
    }


def seqshard_block(device, world: int, rank: int, steps: int, warmup: int, peak: float, total: int = 1 << 22,
                   heads: int = 4, head_dim: int = 64) -> dict:
    """Config 5: one sequence of ``total`` positions x 22 SBDA layers in ``world`` contiguous shards
    (strong scaling); the i - 2^(l-1) halos come from the owning GPU over NVLink inside the kernels.
    One GPU runs the unsharded kernels on the whole sequence."""
    import torch.distributed as dist

    import sbda_b200
    from sbda_b200.sharded import ShardGroup, sharded_backward, sharded_forward

    layers, H, D = 22, heads, head_dim
    shard = total // world
    shards = ShardGroup()
    offsets = sbda_b200.sbda_layer_offsets(layers)
    gen = torch.Generator(device=device).manual_seed(77 + rank)
    bufs = []
    for _ in range(4):  # q, k, v, dO of this rank's shard (one set, reused by every layer)
        t = shards.empty(1, shard, H, D, dtype=torch.bfloat16, device=device)
        t.copy_(torch.randn(t.shape, device=device, generator=gen).to(torch.bfloat16))
        bufs.append(t.permute(0, 2, 1, 3))
    q, k, v, do = bufs
    lses = [shards.empty(1, H, shard, dtype=torch.float32, device=device) for _ in range(layers)]
    out = torch.empty_like(q)

    def step():
        for layer in range(layers):
            sharded_forward(q, k, v, offsets[layer], shards, out=out, lse=lses[layer])
        for layer in reversed(range(layers)):
            sharded_backward(q, k, v, do, lses[layer], offsets[layer], shards)

    for _ in range(max(3, warmup)):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        step()
    end.record()
    torch.cuda.synchronize()
    ms = start.elapsed_time(end) / steps
    if world > 1:
        t = torch.tensor([ms], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        shards.barrier()
        torch.cuda.synchronize()
    step_bytes = total * H * layers * (11 * D * 2 + 8)
    link = shard_link_model(total, world, H, D, 2, offsets, peak)
    link["frac_of_target"] = link["target_ms"] / ms
    return {
        "workload": f"cfg5: {total} positions x {layers} layers, {H} heads x {D}, {world} contiguous shards of {shard}",
        "value": total / (ms * 1e-3) / 1e6, "unit": UNIT, "ms_per_step": ms, "scaling": "strong",
        "kernels": ("windowed (sbda_v2) kernels; 1 GPU: unsharded calls; N > 1: sharded calls whose K/V tiles and "
                    "halos past the shard are staged from the owning GPU over NVLink with non-multicast TMA"),
        "shard_link_model": link,
        "step_roofline": {"achieved": step_bytes / (ms * 1e-3) / 1e9, "peak": peak * world, "unit": "GB/s",
                          "frac": step_bytes / (ms * 1e-3) / 1e9 / (peak * world),
                          "algorithmic_bytes_per_step": step_bytes},
        "gpu_launches": 2 * layers * steps,
    }


def run_seqshard(args) -> None:
    """``--workload cfg5``: the config-5 line on its own (strong scaling over the torchrun ranks)."""
    import datetime

    import torch.distributed as dist

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    peak, peak_kind = measured_peak_gbs()
    total = 1 << 22 if args.length == 1 << 20 else args.length
    sampler = ClockSampler(local)
    block = seqshard_block(device, world, rank, args.steps, args.warmup, peak, total=total, heads=args.heads,
                           head_dim=args.head_dim)
    clocks = sampler.stop()
    if rank == 0:
        line = {"metric": "SBDA attn fwd+bwd Mpositions/s, one 4M-position sequence x 22 layers in contiguous shards",
                "n_gpus": world, "steps": args.steps, "warmup": max(3, args.warmup), "higher_is_better": True,
                "vs_baseline": None, "dtype": "bf16", "data": "synthetic N(0,1), seeded, resident in HBM",
                "clocks": clocks, "peak_kind": peak_kind}
        line.update(block)
        line["config"] = {"workload": line.pop("workload"), "kernels": line.pop("kernels")}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_block(args) -> None:
    """Block parts around the attention op (BiAttn/model.py:299-335) at the config-4 width.

    Times, per layer, the forward and backward of everything in the block that is neither a GEMM
    nor the attention op: the pre-attention RMSNorm, the attention's padding-row multiply, the
    residual add, the pre-FFN RMSNorm, the SwiGLU gate and the final masked residual.  Two arms on
    the same seeded inputs: the reference's eager ops and this package's fused kernels.  One
    JSON line; the fused arm's algorithmic bytes give its HBM roofline.
    """
    import torch.nn.functional as F

    from sbda_b200 import block as blk

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    L, dim, hidden = args.length, args.heads * args.head_dim, 4 * args.heads * args.head_dim
    dtype = torch.bfloat16
    g = torch.Generator(device=dev).manual_seed(77)
    mk = lambda *s: torch.randn(*s, device=dev, generator=g).to(dtype)  # noqa: E731
    x, attn_out, ff = mk(1, L, dim), mk(1, L, dim), mk(1, L, dim)
    gate, up = mk(1, L, hidden), mk(1, L, hidden)
    mask = torch.rand(1, L, device=dev, generator=g) > 0.01
    w1, w2 = (torch.rand(dim, device=dev, generator=g) + 0.5 for _ in range(2))
    dys = [mk(1, L, dim), mk(1, L, dim), mk(1, L, hidden)]  # gradients reaching n1, y, h

    def eager():
        xs, a, gt, u, f = (t.detach().requires_grad_() for t in (x, attn_out, gate, up, ff))
        n1 = F.rms_norm(xs, (dim,), w1.to(dtype), 1e-6)
        x1 = xs + a * mask[:, :, None].to(dtype)
        n2 = F.rms_norm(x1, (dim,), w2.to(dtype), 1e-6)
        h = F.silu(gt) * u
        y = x1 + f * mask[:, :, None].to(dtype)
        torch.autograd.backward((n1, y, h, n2), (dys[0], dys[1], dys[2], dys[0]))

    def fused():
        xs, a, gt, u, f = (t.detach().requires_grad_() for t in (x, attn_out, gate, up, ff))
        n1 = blk.rms_norm(xs, w1)
        x1, n2 = blk.add_rms_norm(xs, a, w2, 1e-6, mask)
        h = blk.silu_mul(gt, u)
        y = torch.addcmul(x1, f, mask[:, :, None].to(dtype))
        torch.autograd.backward((n1, y, h, n2), (dys[0], dys[1], dys[2], dys[0]))

    def timed(fn):
        for _ in range(max(3, args.warmup)):
            fn()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(args.steps):
            fn()
        end.record()
        torch.cuda.synchronize()
        return start.elapsed_time(end) / args.steps

    eager_ms, fused_ms = timed(eager), timed(fused)
    e, r = 2, L
    # Fused arm, algorithmic bytes (each tensor read or written once per kernel):
    # fwd norm1 x->n1 (2), add+norm x,a->x1,n2 (4), gate g,u->h (3h), residual x1,f->y (3);
    # bwd norm1 x,dn1->dx (3), add+norm x1,dn2,dy->dx,da (5), gate g,u,dh->dg,du (5h), residual dy->df (2).
    units = (2 + 4 + 3 + 3 + 5 + 2) * dim + (3 + 5) * hidden
    algo = r * e * units + r * (4 * 4 + 1 * 2)  # + rstd rows, mask bytes
    achieved = algo / (fused_ms * 1e-3) / 1e9
    peak, _ = measured_peak_gbs()
    print(json.dumps({
        "metric": "SBDA block elementwise parts (norms, residuals, masks, SwiGLU gate) fwd+bwd ms per layer",
        "value": fused_ms, "unit": "ms", "n_gpus": 1, "steps": args.steps, "warmup": max(3, args.warmup),
        "higher_is_better": False, "eager_ms": eager_ms, "speedup_vs_eager": eager_ms / fused_ms,
        "dtype": "bf16", "data": "synthetic N(0,1), seeded",
        "config": {"workload": "block parts at config 4 width", "positions": L, "dim": dim, "ffn_hidden": hidden},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "algorithmic_bytes": algo},
    }), flush=True)


def main() -> None:
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "cfg5":
        run_seqshard(args)
    elif args.workload == "block":
        run_block(args)
    elif args.workload == "gqa":
        torch.cuda.set_device(0)
        peak, _ = measured_peak_gbs()
        print(json.dumps(gqa_block(torch.device("cuda", 0), args.steps, args.warmup, peak, length=args.length,
                                   layers=args.layers)), flush=True)
    elif args.workload == "backbone":
        torch.cuda.set_device(0)
        print(json.dumps(backbone_block(torch.device("cuda", 0), args.steps, args.warmup, length=args.length,
                                        layers=args.layers)), flush=True)
    elif args.workload == "normed":
        torch.cuda.set_device(0)
        peak, _ = measured_peak_gbs()
        block = norm_rope_attention_block(torch.device("cuda", 0), args.steps, args.warmup, peak, length=args.length,
                                          heads=args.heads, layers=args.layers)
        print(json.dumps(block), flush=True)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
