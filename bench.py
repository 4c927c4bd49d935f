"""Benchmark of the paged verify-attention hot path (driver contract: one JSON line).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload target_verify_8b|draft_decode_0p6b|long_verify_8b_k4|long_verify_8b_k8|hostkv_copy|kv_migrate]
                    [--kernel auto|decode|verify]

Metric: paged verify-attention achieved HBM TB/s at the
Qwen3-8B shape.  A *step* is the attention of one Target verify forward: one
``paged_attention`` call per layer (36 calls), each over the layer's own slice
of a 24,576-block paged KV pool (58 GB of fp16 K+V), for 16 requests verified
at depth 4 with prefix lengths U[256, 4096].  Every step therefore streams
5.1 GB of distinct KV (inputs larger than the 126 MB L2, no flush needed).

``value``  = algorithmic bytes (unique K+V + q + o + block-table entries) of
             all ranks / max-over-ranks device time, with inputs in HBM.
``e2e``    = the same bytes / device time of the user-facing call
             (``nebulasd_b200.kernels.paged_attention`` with an ``infer_state``),
             with every step's q rows, lengths, seq ids and block table copied
             from pinned host memory and every step's o copied back inside the
             timed region.
Multi-GPU runs (torchrun) are weak scaling: each rank owns its own 16
requests and pool, no collective on the path.  ``--impl reference`` times the
reference semantics (the fp32 PyTorch-eager oracle) on the host cores.

``--workload hostkv_copy`` measures the HostKV path instead: a step is one
restore plan (host arena -> GPU cache, both planes) and one writeback plan
(GPU -> host) of four requests' block runs, Qwen3-8B block size (36 layers,
1,179,648 B per block and plane), through ``NativeCopyBackend`` in its kernel
mode and in its copy-engine mode (one ``cudaMemcpyAsync`` per run and plane,
the reference's transfer engine); ``value`` is its default (``auto``) mode; the
roofline is a single large pinned copy measured in the same run.

``--workload kv_migrate`` (two visible GPUs, one process) measures same-role
migration: ``migrate_blocks`` copying four requests' block runs of Qwen3-8B
blocks (both planes) from GPU 0's cache into GPU 1's over NVLink, in kernel
mode (peer loads) and copy-engine mode, against a single large peer copy.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
import types
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "paged verify-attn achieved HBM TB/s (% peak), Qwen3-8B shape, 1/2/4/8 B200"
UNIT = "TB/s"


def _args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=("ours", "reference"))
    ap.add_argument("--workload", default="target_verify_8b")
    ap.add_argument("--kernel", default="auto", choices=("auto", "decode", "verify", "verify_long"))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=None)
    ap.add_argument("--layers", type=int, default=None,
                    help="override the workload's layer count (profiling: a small pool, same per-call shape)")
    ap.add_argument("--requests", type=int, default=None,
                    help="override the workload's request count (profiling: a smaller pool, same per-request shape)")
    ap.add_argument("--no-soak", action="store_true", help="skip the 1 s clock-sampling soak (profiling runs)")
    ap.add_argument("--no-secondary", action="store_true",
                    help="skip the secondary figures (reference kernels on this GPU, configs 2, 2b and 4)")
    return ap.parse_args()


def _dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def max_over_ranks(ms: float, device, world: int) -> float:
    """The job's time: the slowest rank's (each rank times its own stream)."""
    if world <= 1:
        return ms
    t = torch.tensor([ms], dtype=torch.float64, device=device)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def _traffic(workload: str, kernel: str):
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary, if any."""
    f = ROOT / "profiles" / f"{kernel}_attn_{workload}.md"
    if not f.exists():
        return None
    for line in f.read_text().splitlines():
        if line.strip().startswith("traffic_bytes_per_launch:"):
            try:
                return int(float(line.split(":", 1)[1].strip()))
            except ValueError:
                return None
    return None


class Clocks:
    """nvidia-smi sampling during the timed region (median SM MHz, throttle reasons)."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.out = out
        return False

    def summary(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        busy = [s for s in sm if mx and s > 0.3 * mx] or sm
        return {"sm_mhz": statistics.median(busy) if busy else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def build_workload(name: str, seed: int, device, layers_override=None, requests_override=None):
    from nebulasd_b200.workloads import CONFIGS, make_paged_batch
    cfg = dict(CONFIGS[name])
    layers = cfg.pop("num_layers", 1)
    if layers_override:
        layers = layers_override
    if requests_override:  # profiling: fewer requests, a pool scaled to match
        cfg["pool_blocks"] = -(-cfg["pool_blocks"] * requests_override // cfg["num_requests"])
        cfg["num_requests"] = requests_override
    b = make_paged_batch(seed, num_layers=layers, cur_layer=0, device=device, **cfg)
    return b, layers, cfg


def step_bytes(b, layers: int) -> int:
    """Algorithmic bytes of one step: per layer unique K+V, q and o rows, block-table entries."""
    kv = b.kv_bytes()
    qo = 2 * b.q.numel() * b.q.element_size()
    tables = 4 * sum(math.ceil((c + d + 1) / 16) for c, d in zip(b.ctx, b.depths))
    return layers * (kv + qo + tables)


def run_ours(args):
    world, rank, local = _dist()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    from nebulasd_b200 import _lib
    from nebulasd_b200.kernels import paged_attention, paged_attention_raw
    from nebulasd_b200.kernels.paged_attn import choose_kernel, set_kernel
    set_kernel(args.kernel)

    b, layers, cfg = build_workload(args.workload, 1234 + 7919 * rank, dev, args.layers, args.requests)
    kernel = choose_kernel(b.num_q_heads, b.num_kv_heads, int(b.q.shape[0]), max(b.seq_lens_list))
    kname = {_lib.NEB_ATTN_DECODE: "decode", _lib.NEB_ATTN_VERIFY: "verify",
             _lib.NEB_ATTN_VERIFY_LONG: "verify_long"}[kernel]
    o = torch.empty_like(b.q)
    stream = torch.cuda.current_stream(dev)
    scale = b.q.shape[-1] ** -0.5

    # The timed step calls the C ABI with each layer's arguments built once, as
    # a C or C++ host would, so that host work stays far below the kernels'
    # time even with one process per GPU on a shared host; the e2e figure below
    # goes through the Python drop-in.  Arguments as paged_attention_raw passes them.
    from nebulasd_b200.kernels.paged_attn import _entry, _last_workspace
    paged_attention_raw(b.q, b.k_cache, b.v_cache, b.block_table, b.seq_lens, b.seq_ids, 0, scale, o,
                        kernel=kernel, stream=stream)  # checks the tensors once
    entry = _entry(kernel)
    ws = _last_workspace(kernel, b.q, stream, stream.cuda_stream, b.q.shape[0], b.q.shape[1], b.k_cache.shape[2])
    nblk, nlay, hkv, bsz, hdim = b.k_cache.shape
    argsets = [(b.q.data_ptr(), b.k_cache.data_ptr(), b.v_cache.data_ptr(), b.block_table.data_ptr(),
                b.block_table.shape[0], b.block_table.shape[1], b.seq_lens.data_ptr(), b.seq_ids.data_ptr(),
                b.q.shape[0], b.q.shape[1], hkv, hdim, bsz, nblk, nlay, layer, float(scale), o.data_ptr(),
                ws.data_ptr(), ws.numel(), stream.cuda_stream) for layer in range(layers)]

    def step():
        for a in argsets:
            rc = entry(*a)
            if rc:
                _lib.check(rc, "paged_attention")

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    with Clocks(local) as clk:
        t_soak = time.time()
        while not args.no_soak and time.time() - t_soak < 1.0:   # let the sampler see the kernel under load
            step()
            torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
    ms = e0.elapsed_time(e1)
    ms_max = max_over_ranks(ms, dev, world)
    per_step = step_bytes(b, layers)
    total_bytes = per_step * args.steps * world
    value = total_bytes / (ms_max * 1e-3) / 1e12
    launch_ms = ms / (args.steps * layers)
    achieved_gbs = per_step / layers / (launch_ms * 1e-3) / 1e9
    peak, peak_kind = _peaks()

    # ---- e2e through the drop-in API with host buffers, copies overlapped
    e2e_steps = args.e2e_steps or max(3, min(args.steps, 50))
    e2e_value, h2d, d2h = measure_e2e(b, layers, dev, world, e2e_steps, scale, barrier)

    # ---- requests/s, and strong scaling (16 requests in total over the ranks)
    requests_per_s = world * cfg["num_requests"] * args.steps / (ms_max * 1e-3)
    strong = measure_strong(b, layers, cfg, dev, world, rank, kernel, scale, barrier, ms_max / args.steps)

    # ---- secondary figures on one GPU: the reference's own kernels on this
    # B200, the other configs' kernels (single-GPU runs only)
    secondary = {}
    if world == 1 and not args.no_secondary:
        secondary["reference_gpu"] = _guard(lambda: reference_gpu_bar(b, layers, scale, launch_ms))
        k_cache_free(b)  # the headline pool, before the other configs' pools
        torch.cuda.empty_cache()
        secondary["draft_decode_0p6b"] = _guard(lambda: secondary_attention("draft_decode_0p6b", dev, 5))
        secondary["fused_qk_norm_rope_store_0p6b"] = _guard(lambda: fused_bar(dev))
        secondary["long_verify_8b_k4"] = _guard(lambda: secondary_attention("long_verify_8b_k4", dev, 3))
        secondary["long_verify_8b_k8"] = _guard(lambda: secondary_attention("long_verify_8b_k8", dev, 3))
        secondary["long_verify_8b_k4_hostkv"] = _guard(lambda: long_hostkv_line("long_verify_8b_k4", dev, 10))
        secondary["prefill_8b"] = _guard(lambda: prefill_line(dev, 10, 3))
        secondary["greedy_accept_8b"] = _guard(lambda: accept_line(dev, 50, 3))

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(args.workload, budget_s=10.0)

    if world > 1:
        torch.distributed.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16 (fp32 accumulate)", "data": "synthetic",
        "config": {"workload": args.workload, "kernel": kname, "requests_per_gpu": cfg["num_requests"],
                   "depth": cfg["depth"], "ctx": [cfg["ctx_lo"], cfg["ctx_hi"]], "num_q_heads": cfg["num_q_heads"],
                   "num_kv_heads": cfg["num_kv_heads"], "head_dim": 128, "block_size": 16, "num_layers": layers,
                   "pool_blocks": cfg["pool_blocks"], "calls_per_step": layers,
                   "l2": f"inputs larger than L2: each step streams {per_step / 1e9:.2f} GB of distinct KV",
                   "parallelism": f"{world} independent request shards (no collective)"},
        "roofline": {"bound": "hbm", "achieved": round(achieved_gbs, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved_gbs / peak, 4), "peak_kind": peak_kind,
                     "traffic": _traffic(args.workload, kname),
                     "bytes_per_launch": per_step // layers, "launch_us": round(launch_ms * 1e3, 3)},
        "e2e": {"value": round(e2e_value, 4), "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "steps": e2e_steps, "api": "nebulasd_b200.kernels.paged_attention",
                "copies": "each step's q rows, lengths and table H2D and its o rows D2H on two side streams, "
                          "double-buffered so they overlap the neighbouring steps"},
        "requests_per_s": round(requests_per_s, 1),
        "strong_scaling": strong,
        "gpu_launches": args.steps * layers,
        "clocks": clk.summary(),
        "cpu_baseline": cpu,
    }
    line.update(secondary)
    print(json.dumps(line), flush=True)


def _guard(fn):
    """A secondary measurement, or why it is unavailable (it never costs the headline line)."""
    try:
        return fn()
    except Exception as e:  # noqa: BLE001 - reported in the JSON line
        return {"unavailable": f"{type(e).__name__}: {e}"[:300]}


def k_cache_free(b):
    b.k_cache = b.v_cache = None


def measure_e2e(b, layers, dev, world, steps, scale, barrier):
    """Same metric through ``nebulasd_b200.kernels.paged_attention`` with HOST buffers.

    Every step copies its inputs from pinned host memory (the block table,
    lengths and seq ids, and all layers' q rows) on an H2D stream and reads
    every layer's o rows back on a D2H stream, both inside the timed region.
    The device buffers are doubled: step s + 1's inputs go up while step s
    computes, and step s's outputs come down while step s + 1 computes (the
    pipelined host interface of a serving loop); the timed region ends when
    the last step's outputs are on the host.
    """
    from nebulasd_b200.kernels import paged_attention
    from nebulasd_b200.workloads import decode_infer_state
    R, H, D = b.q.shape
    q_host = torch.empty((layers, R, H, D), dtype=torch.float16, pin_memory=True)
    q_host.copy_(b.q.cpu().unsqueeze(0).expand(layers, R, H, D))
    o_host = torch.empty((layers, R, H * D), dtype=torch.float16, pin_memory=True)
    lens_host = b.seq_lens.cpu().pin_memory()
    ids_host = b.seq_ids.cpu().pin_memory()
    bt_host = b.block_table.cpu().pin_memory()
    bufs = []
    for _ in range(2):
        buf = types.SimpleNamespace(
            q=torch.empty((layers, R, H, D), dtype=torch.float16, device=dev),
            o=torch.empty((layers, R, H * D), dtype=torch.float16, device=dev),
            lens=torch.empty_like(b.seq_lens), ids=torch.empty_like(b.seq_ids), bt=torch.empty_like(b.block_table),
            ready=torch.cuda.Event(), used=torch.cuda.Event(), done=torch.cuda.Event(), drained=torch.cuda.Event())
        buf.st = decode_infer_state(buf.lens, buf.ids, b.seq_lens_list, b.num_kv_heads, scale)
        bufs.append(buf)
    mc = types.SimpleNamespace(num_q_heads=H, num_kv_heads=b.num_kv_heads, head_dim=D, num_layers=layers)
    ec = types.SimpleNamespace(block_size=16, max_blocks_per_seq=b.block_table.shape[1])
    comp = torch.cuda.current_stream(dev)
    h2d_s, d2h_s = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    def upload(buf):
        with torch.cuda.stream(h2d_s):
            h2d_s.wait_event(buf.used)  # the step that last read this buffer is done with it
            buf.lens.copy_(lens_host, non_blocking=True)
            buf.ids.copy_(ids_host, non_blocking=True)
            buf.bt.copy_(bt_host, non_blocking=True)
            buf.q.copy_(q_host, non_blocking=True)
            buf.ready.record(h2d_s)

    def compute(buf):
        comp.wait_event(buf.ready)
        comp.wait_event(buf.drained)  # the previous read-back of this buffer's outputs
        for layer in range(layers):
            paged_attention(buf.q[layer], b.k_cache, b.v_cache, buf.bt, mc, ec, buf.st, layer, buf.o[layer])
        buf.used.record(comp)
        buf.done.record(comp)
        with torch.cuda.stream(d2h_s):
            d2h_s.wait_event(buf.done)
            o_host.copy_(buf.o, non_blocking=True)
            buf.drained.record(d2h_s)

    def run(n):
        upload(bufs[0])
        for i in range(n):
            if i + 1 < n:
                upload(bufs[(i + 1) % 2])
            compute(bufs[i % 2])

    run(2)
    torch.cuda.synchronize()
    barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(comp)
    h2d_s.wait_event(f0)
    run(steps)
    comp.wait_event(bufs[(steps - 1) % 2].drained)
    f1.record(comp)
    torch.cuda.synchronize()
    barrier()
    ems = max_over_ranks(f0.elapsed_time(f1), dev, world)
    value = step_bytes(b, layers) * steps * world / (ems * 1e-3) / 1e12
    h2d = q_host.numel() * 2 + lens_host.numel() * 4 + ids_host.numel() * 4 + bt_host.numel() * 4
    d2h = o_host.numel() * 2
    return value, h2d, d2h


def measure_strong(b, layers, cfg, dev, world, rank, kernel, scale, barrier, headline_ms_per_step):
    """Strong scaling: the headline's 16 requests in total, split evenly over the ranks."""
    total = cfg["num_requests"]
    if world == 1:
        return {"requests_total": total, "requests_per_gpu": total, "ms_per_step": round(headline_ms_per_step, 4),
                "requests_per_s": round(total / (headline_ms_per_step * 1e-3), 1)}
    from nebulasd_b200.kernels import paged_attention_raw
    from nebulasd_b200.workloads import make_paged_batch
    per = max(1, total // world)
    sub = dict(cfg)
    sub["num_requests"] = per
    sb = make_paged_batch(4321 + 7919 * rank, num_layers=layers, cur_layer=0, device=dev,
                          cache=(b.k_cache, b.v_cache), **sub)
    o = torch.empty_like(sb.q)
    stream = torch.cuda.current_stream(dev)

    def step():
        for layer in range(layers):
            paged_attention_raw(sb.q, sb.k_cache, sb.v_cache, sb.block_table, sb.seq_lens, sb.seq_ids, layer, scale,
                                o, kernel=kernel, stream=stream)

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    barrier()
    steps = 20
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1), dev, world) / steps
    return {"requests_total": per * world, "requests_per_gpu": per, "ms_per_step": round(ms, 4),
            "requests_per_s": round(per * world / (ms * 1e-3), 1)}


def _time_steps(fn, steps, warmup=2):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def _time_queued(fn, steps, warmup=3):
    """Device time per call of a launch-bound op: the stream is held behind a
    GPU sleep while the calls are queued, so host launch overhead cannot
    leave the GPU idle between them."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda._sleep(int(2e8))  # about 0.1 s at the B200's clock: room to queue every call
    e0.record()
    for _ in range(steps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def reference_gpu_bar(b, layers, scale, our_launch_ms):
    """The reference's own Triton ``paged_attention`` (phase 1 + phase 2,
    ``swiftLLM/swiftllm/worker/kernels/paged_attn.py:152-222``), JIT-compiled by
    Triton for this GPU, on the headline batch and pool (one call per layer, its
    own split-K choice ``worker/model.py:380-384``), timed with CUDA events."""
    from baseline import reference as R
    if not R.available():
        return {"unavailable": "reference not installed under baseline/_ref"}
    pa = R.swiftllm("worker.kernels.paged_attn")
    from nebulasd_b200.workloads import decode_infer_state
    R_, H, D = b.q.shape
    st = decode_infer_state(b.seq_lens, b.seq_ids, b.seq_lens_list, b.num_kv_heads, scale)
    mc = types.SimpleNamespace(num_q_heads=H, num_kv_heads=b.num_kv_heads, head_dim=D, num_layers=layers)
    ec = types.SimpleNamespace(block_size=16, max_blocks_per_seq=b.block_table.shape[1])
    o = torch.empty((R_, H * D), dtype=torch.float16, device=b.q.device)

    def step():
        for layer in range(layers):
            pa.paged_attention(b.q, b.k_cache, b.v_cache, b.block_table, mc, ec, st, layer, o)

    t0 = time.perf_counter()
    step()  # JIT compile on first use
    torch.cuda.synchronize()
    compile_s = time.perf_counter() - t0
    ms = _time_steps(step, 3, warmup=1)
    per_launch = ms / layers
    bytes_per_launch = step_bytes(b, 1)
    return {"impl": "reference Triton paged_attention (phase 1 + phase 2), same batch and pool",
            "value": round(bytes_per_launch / (per_launch * 1e-3) / 1e12, 4), "unit": UNIT,
            "launch_us": round(per_launch * 1e3, 2), "ours_speedup": round(per_launch / our_launch_ms, 2),
            "seq_block_size": st.seq_block_size, "first_call_s": round(compile_s, 1)}


def secondary_attention(workload, dev, steps):
    """Another config's attention through the same drop-in op (auto kernel choice)."""
    from nebulasd_b200 import _lib
    from nebulasd_b200.kernels import paged_attention_raw
    from nebulasd_b200.kernels.paged_attn import choose_kernel
    b, layers, cfg = build_workload(workload, 1234, dev)
    kernel = choose_kernel(b.num_q_heads, b.num_kv_heads, int(b.q.shape[0]), max(b.seq_lens_list))
    o = torch.empty_like(b.q)
    scale = b.q.shape[-1] ** -0.5
    reps = max(1, 36 // layers)

    def step():
        for _ in range(reps):
            for layer in range(layers):
                paged_attention_raw(b.q, b.k_cache, b.v_cache, b.block_table, b.seq_lens, b.seq_ids, layer, scale,
                                    o, kernel=kernel)

    ms = _time_steps(step, steps)
    launch_ms = ms / (reps * layers)
    per_launch = step_bytes(b, 1)
    peak, _ = _peaks()
    tbps = per_launch / (launch_ms * 1e-3) / 1e12
    out = {"value": round(tbps, 4), "unit": UNIT, "frac_of_measured_peak": round(tbps * 1e3 / peak, 4),
           "launch_us": round(launch_ms * 1e3, 2), "bytes_per_launch": per_launch,
           "kernel": {_lib.NEB_ATTN_DECODE: "decode", _lib.NEB_ATTN_VERIFY: "verify",
                      _lib.NEB_ATTN_VERIFY_LONG: "verify_long"}[kernel],
           "requests": cfg["num_requests"], "depth": cfg["depth"], "ctx": [cfg["ctx_lo"], cfg["ctx_hi"]],
           "num_layers": layers}
    out["traffic_profile"] = _traffic(workload, out["kernel"])
    k_cache_free(b)
    torch.cuda.empty_cache()
    return out


def fused_bar(dev, layers_override=None):
    """Config 2b: QK-RMSNorm + RoPE + KV store of the Draft's 64 decode tokens
    (Qwen3-0.6B: 16 q / 8 kv heads, 28-layer pool), our single launch against
    the reference's four Triton launches (``transformer_layer.py:114-143``) on
    the same inputs."""
    from nebulasd_b200.kernels import qk_norm_rope_store
    from nebulasd_b200.workloads import CONFIGS, decode_infer_state, make_paged_batch
    from baseline import reference as R
    cfg = dict(CONFIGS["draft_decode_0p6b"])
    layers = cfg.pop("num_layers")
    if layers_override:  # profiling: a smaller pool, same per-call work
        layers = layers_override
    cfg["pool_blocks"] = 8192  # holds the batch's blocks; smaller than config 2's pool, so the set-up is short
    b = make_paged_batch(77, num_layers=layers, cur_layer=0, device=dev, **cfg)
    T, H, D = b.q.shape
    hk = b.num_kv_heads
    g = torch.Generator(device=dev).manual_seed(78)
    k = torch.randn((T, hk, D), generator=g, device=dev, dtype=torch.float16)
    v = torch.randn((T, hk, D), generator=g, device=dev, dtype=torch.float16)
    wq = (1 + 0.02 * torch.randn(D, generator=g, device=dev)).half()
    wk = (1 + 0.02 * torch.randn(D, generator=g, device=dev)).half()
    pos = (b.seq_lens - 1).long()
    inv = 1.0 / (1e6 ** (torch.arange(0, D, 2, device=dev, dtype=torch.float32) / D))
    freqs = torch.outer(pos.float(), inv)
    st = decode_infer_state(b.seq_lens, b.seq_ids, b.seq_lens_list, hk, D ** -0.5)
    st.position_cos, st.position_sin = torch.cos(freqs).half(), torch.sin(freqs).half()
    st.num_prefill_seqs, st.num_prefill_tokens = 0, 0
    mc = types.SimpleNamespace(num_q_heads=H, num_kv_heads=hk, head_dim=D, num_layers=layers, rms_norm_eps=1e-6)
    ec = types.SimpleNamespace(block_size=16, max_blocks_per_seq=b.block_table.shape[1])
    q0 = b.q.clone()
    k0 = k.clone()
    layer = layers // 2

    def ours():
        qk_norm_rope_store(q0, k0, v, wq, wk, 1e-6, b.k_cache, b.v_cache, b.block_table, mc, ec, st, layer)

    out = {"tokens": T, "ours_launches": 1, "ours_us": round(_time_steps(ours, 200, 5) * 1e3, 2)}
    # moved bytes: q and k read and written, v read, k and v written to the cache
    out["bytes"] = (2 * q0.numel() + 2 * k0.numel() + v.numel() + 2 * k0.numel()) * 2
    if R.available():
        rm = R.swiftllm("worker.kernels.rmsnorm")
        ro = R.swiftllm("worker.kernels.rotary_emb")
        kv = R.swiftllm("worker.kernels.kvcache_mgmt")

        def ref():
            rm.rmsnorm_inplace(q0.view(-1, D), wq, 1e-6)
            rm.rmsnorm_inplace(k0.view(-1, D), wk, 1e-6)
            ro.rotary_embedding_inplace(q0, k0, st)
            kv.store_kvcache(k0, v, b.k_cache, b.v_cache, b.block_table, mc, ec, st, layer)

        ref()  # JIT compile on first use
        torch.cuda.synchronize()
        out["reference_launches"] = 4
        out["reference_us"] = round(_time_steps(ref, 200, 5) * 1e3, 2)
        out["ours_speedup"] = round(out["reference_us"] / out["ours_us"], 3)
    k_cache_free(b)
    torch.cuda.empty_cache()
    return out


def cpu_baseline(workload: str, budget_s: float):
    """The fp32 PyTorch-eager reference semantics on the host cores, on a bounded sample."""
    from nebulasd_b200.workloads import CONFIGS, make_paged_batch
    from oracle.attention import paged_attention as oracle_attention
    torch.set_num_threads(os.cpu_count() or 1)
    cfg = dict(CONFIGS[workload])
    cfg.pop("num_layers", None)
    b = make_paged_batch(1234, num_layers=1, cur_layer=0, device="cpu", **cfg)
    per_call = step_bytes(b, 1)
    t0 = time.perf_counter()
    calls = 0
    while True:
        oracle_attention(b.q, b.k_cache, b.v_cache, b.block_table, b.seq_lens_list, b.seq_ids_list, 0,
                         b.q.shape[-1] ** -0.5)
        calls += 1
        el = time.perf_counter() - t0
        if el >= budget_s or calls >= 200:
            break
    return {"value": round(per_call * calls / el / 1e12, 6), "unit": UNIT, "cores": torch.get_num_threads(),
            "kind": "port", "sample": f"{calls} full layer calls of {workload} (one layer, {b.num_rows} rows) "
                                      f"in {el:.1f} s, fp32 eager oracle"}


def run_reference(args):
    world, rank, _ = _dist()
    if rank != 0:
        return
    from nebulasd_b200.workloads import CONFIGS, make_paged_batch
    from oracle.attention import paged_attention as oracle_attention
    torch.set_num_threads(os.cpu_count() or 1)
    cfg = dict(CONFIGS[args.workload])
    cfg.pop("num_layers", None)
    b = make_paged_batch(1234, num_layers=1, cur_layer=0, device="cpu", **cfg)
    per_call = step_bytes(b, 1)
    scale = b.q.shape[-1] ** -0.5

    def step():
        oracle_attention(b.q, b.k_cache, b.v_cache, b.block_table, b.seq_lens_list, b.seq_ids_list, 0, scale)

    for _ in range(max(args.warmup, 1)):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    el = time.perf_counter() - t0
    value = per_call * args.steps / el / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 6), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(el * 1e3 / args.steps, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": args.workload, "requests": cfg["num_requests"], "depth": cfg["depth"],
                   "ctx": [cfg["ctx_lo"], cfg["ctx_hi"]], "num_q_heads": cfg["num_q_heads"],
                   "num_kv_heads": cfg["num_kv_heads"], "head_dim": 128, "calls_per_step": 1},
        "cpu_baseline": {"value": round(value, 6), "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
                         "sample": f"one layer call of {args.workload} per step ({b.num_rows} rows, all requests), "
                                   "fp32 PyTorch-eager restatement of the reference's Triton kernels"},
        "e2e": {"value": round(value, 6), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_hostkv(args):
    """HostKV restore/writeback bandwidth (rank 0 only; the copies are per GPU and PCIe-bound).

    The arena, extents and plans are the reference's own (``SharedHostKVArena``,
    ``CopyRegion``, ``CopyPlan`` from ``baseline/_ref``); without them the line
    says unavailable."""
    world, rank, local = _dist()
    if rank != 0:
        return
    import numpy as np
    from baseline import reference as R
    from nebulasd_b200.hostkv import NativeCopyBackend
    metric = "HostKV restore GB/s (both planes, Qwen3-8B blocks)"
    if not R.available():
        print(json.dumps({"metric": metric, "unavailable": "reference not installed under baseline/_ref"}), flush=True)
        return
    arena_mod, tr = R.nebulasd("kv.arena"), R.nebulasd("kv.transfer")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    layers, hk = 36, 8
    gpu_blocks, host_blocks = 1280, 1024
    shape = (gpu_blocks, layers, hk, 16, 128)
    k_cache = torch.zeros(shape, dtype=torch.float16, device=dev)
    v_cache = torch.zeros(shape, dtype=torch.float16, device=dev)
    block_bytes = k_cache[0].numel() * 2
    try:
        arena = arena_mod.SharedHostKVArena.create(total_blocks=host_blocks, block_bytes=block_bytes,
                                                   dtype=str(k_cache.dtype), kv_block_shape=shape[1:])
    except OSError as e:  # POSIX shared memory smaller than the 2.4 GB arena
        print(json.dumps({"metric": metric, "unavailable": f"shared-memory arena: {e}"}), flush=True)
        return
    rng = np.random.default_rng(1234)
    # Four requests' block runs (ctx U[1 K, 4 K] tokens): host extents and GPU
    # ranges disjoint; at most 4 * 256 blocks, so GPU blocks 200.. stay below 1280.
    counts = rng.integers(64, 257, 4).tolist()
    host_off = np.cumsum([0] + counts[:-1]).tolist()
    gpu_off = (np.cumsum([0] + counts[:-1]) + 200).tolist()
    extents = [arena.make_extent(request_slot=i, request_epoch=1, host_slot=i, host_slot_generation=1,
                                 writer_lease_generation=1, offset_blocks=h, capacity_blocks=c)
               for i, (h, c) in enumerate(zip(host_off, counts))]
    regions = tuple(tr.CopyRegion(e, g, 0, c) for e, g, c in zip(extents, gpu_off, counts))
    moved = 2 * sum(counts) * block_bytes  # both planes
    out = {}
    for mode in ("auto", "kernel", "memcpy"):
        be = NativeCopyBackend(arena=arena, k_cache=k_cache, v_cache=v_cache, mode=mode)
        be.initialize()
        res = {}
        for direction in ("H2D", "D2H"):
            plan = tr.CopyPlan(direction, regions)
            for _ in range(max(args.warmup, 3)):
                be.launch(plan).synchronize()
            ms = [0.0]
            steps = max(1, min(args.steps, 20))
            for _ in range(steps):
                t = be.launch(plan)
                t.synchronize()
                ms.append(t.duration_ms())
            res[direction] = moved * steps / (sum(ms) * 1e-3) / 1e9
        be.close()
        out[mode] = res
    # Roofline: one contiguous pinned buffer of the same size through the copy engine.
    host = torch.empty(moved // 2, dtype=torch.uint8, pin_memory=True)
    devb = torch.empty(moved // 2, dtype=torch.uint8, device=dev)
    peak = {}
    for direction in ("H2D", "D2H"):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        for i in range(4):
            if i == 1:
                e0.record()
            if direction == "H2D":
                devb.copy_(host, non_blocking=True)
            else:
                host.copy_(devb, non_blocking=True)
        e1.record()
        torch.cuda.synchronize()
        peak[direction] = 3 * (moved // 2) / (e0.elapsed_time(e1) * 1e-3) / 1e9
    val = out["auto"]["H2D"]
    line = {
        "metric": "HostKV restore GB/s (both planes, Qwen3-8B blocks)", "value": round(val, 2), "unit": "GB/s",
        "n_gpus": 1, "steps": max(1, min(args.steps, 20)), "warmup": max(args.warmup, 3),
        "higher_is_better": True, "scaling": "none", "vs_baseline": None, "dtype": "u8", "data": "synthetic",
        "config": {"workload": "hostkv_copy", "requests": 4, "blocks": counts, "block_bytes": block_bytes,
                   "bytes_per_plan": moved, "arena": "reference SharedHostKVArena (POSIX shared memory)"},
        "writeback_gbs": round(out["auto"]["D2H"], 2),
        "kernel_mode": {k: round(v, 2) for k, v in out["kernel"].items()},
        "memcpy_mode": {k: round(v, 2) for k, v in out["memcpy"].items()},
        "roofline": {"bound": "pcie", "achieved": round(val, 2), "peak": round(peak["H2D"], 2), "unit": "GB/s",
                     "frac": round(val / peak["H2D"], 4), "peak_kind": "single pinned copy, same run",
                     "peak_d2h": round(peak["D2H"], 2)},
        "e2e": {"value": round(val, 2), "unit": "GB/s", "h2d_bytes_per_step": moved, "d2h_bytes_per_step": 0},
    }
    arena.close()
    arena.unlink()
    print(json.dumps(line), flush=True)


def run_migrate(args):
    """Same-role KV migration GPU 0 -> GPU 1 over NVLink (one process, two GPUs)."""
    world, rank, _ = _dist()
    if rank != 0:
        return
    metric = "KV migration GB/s (NVLink peer, both planes, Qwen3-8B blocks)"
    if torch.cuda.device_count() < 2:
        print(json.dumps({"metric": metric, "unavailable": "needs two visible GPUs"}), flush=True)
        return
    import numpy as np
    from nebulasd_b200.hostkv import migrate_blocks
    src, dst = torch.device("cuda", 0), torch.device("cuda", 1)
    shape = (1280, 36, 8, 16, 128)
    sk = torch.full(shape, 1.0, dtype=torch.float16, device=src)
    sv = torch.full(shape, 2.0, dtype=torch.float16, device=src)
    dk = torch.zeros(shape, dtype=torch.float16, device=dst)
    dv = torch.zeros(shape, dtype=torch.float16, device=dst)
    block_bytes = sk[0].numel() * 2
    rng = np.random.default_rng(1234)
    counts = rng.integers(64, 257, 4).tolist()
    soff = np.cumsum([0] + counts[:-1]).tolist()
    doff = (np.cumsum([0] + counts[:-1]) + 200).tolist()  # at most 1024 + 200 < 1280 blocks
    regions = [(a, b, c) for a, b, c in zip(soff, doff, counts)]
    moved = 2 * sum(counts) * block_bytes
    steps = max(1, min(args.steps, 20))
    stream = torch.cuda.Stream(device=dst)
    res = {}
    for mode in ("kernel", "memcpy"):
        for _ in range(max(args.warmup, 3)):
            migrate_blocks(sk, sv, dk, dv, regions, mode=mode, stream=stream)
        torch.cuda.synchronize(dst)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            migrate_blocks(sk, sv, dk, dv, regions, mode=mode, stream=stream)
        e1.record(stream)
        torch.cuda.synchronize(dst)
        res[mode] = moved * steps / (e0.elapsed_time(e1) * 1e-3) / 1e9
    # Roofline: one contiguous peer copy of one plane's bytes, on the same stream.
    nbytes = moved // 2
    a = sk.view(torch.uint8).reshape(-1)[:nbytes]
    b = dk.view(torch.uint8).reshape(-1)[:nbytes]
    with torch.cuda.stream(stream):
        for _ in range(2):
            b.copy_(a, non_blocking=True)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(5):
            b.copy_(a, non_blocking=True)
        e1.record(stream)
    torch.cuda.synchronize(dst)
    peak = 5 * nbytes / (e0.elapsed_time(e1) * 1e-3) / 1e9
    val = res["kernel"]
    print(json.dumps({
        "metric": metric, "value": round(val, 2), "unit": "GB/s", "n_gpus": 2, "steps": steps,
        "warmup": max(args.warmup, 3), "higher_is_better": True, "scaling": "none", "vs_baseline": None,
        "dtype": "u8", "data": "synthetic",
        "config": {"workload": "kv_migrate", "blocks": counts, "block_bytes": block_bytes, "bytes_per_step": moved},
        "memcpy_mode": round(res["memcpy"], 2),
        "roofline": {"bound": "nvlink", "achieved": round(val, 2), "peak": round(peak, 2), "unit": "GB/s",
                     "frac": round(val / peak, 4), "peak_kind": "single peer copy, same run"},
        "e2e": {"value": round(val, 2), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def run_fused(args):
    """Config 2b on its own line: the fused QK-RMSNorm + RoPE + KV store of the
    Draft's 64 decode tokens, one launch, against the reference's four Triton
    launches on the same inputs (rank 0 only)."""
    world, rank, local = _dist()
    if rank != 0:
        return
    torch.cuda.set_device(local)
    r = fused_bar(torch.device("cuda", local), args.layers)
    line = {"metric": "fused QK-RMSNorm + RoPE + KV-store us per call (Qwen3-0.6B, 64 decode tokens)",
            "value": r["ours_us"], "unit": "us", "n_gpus": 1, "higher_is_better": False, "scaling": "none",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": "fused_store_0p6b", "tokens": r["tokens"], "launches": r["ours_launches"],
                       "num_layers": args.layers or 28,
                       "bytes_per_call": r["bytes"]},
            "reference_gpu": {k: r[k] for k in ("reference_launches", "reference_us", "ours_speedup") if k in r}}
    print(json.dumps(line), flush=True)


def accept_line(dev, steps_arg, warmup_arg, requests=None):
    """Greedy acceptance of a Qwen3-8B verify batch (16 requests x (k+1 = 5)
    rows x 151,936 fp16 logits, 24.3 MB): the device kernel (arg-max and
    acceptance, results left on the GPU) against the reference's tail on the
    same GPU: ``torch.argmax``, ``.tolist()`` and ``compute_greedy_acceptance``
    per request (``post_layer.py:72``, ``model.py:465``, ``speculative.py:122-156``)."""
    from nebulasd_b200.accept import greedy_accept
    from baseline import reference as R
    reqs, depth, vocab = 16, 4, 151936
    rows = reqs * (depth + 1)
    g = torch.Generator(device=dev).manual_seed(99)
    logits = (torch.randn((rows, vocab), generator=g, device=dev) * 4).half()
    am = logits.argmax(1).view(reqs, depth + 1)
    drafts = am[:, :depth].clone()
    drafts[::2, 2] += 1  # half the requests stop accepting at their third draft
    row_start = torch.arange(0, rows + 1, depth + 1, dtype=torch.int32, device=dev)
    flat = drafts.to(torch.int32).reshape(-1).contiguous()

    from nebulasd_b200 import _lib
    from nebulasd_b200.accept import _workspace
    result = torch.empty(reqs * (depth + 1) + 2 * reqs + rows, dtype=torch.int32, device=dev)  # one readback
    tokens = result[:reqs * (depth + 1)].view(reqs, depth + 1)
    count = result[reqs * (depth + 1):reqs * (depth + 2)]
    accepted = result[reqs * (depth + 2):reqs * (depth + 3)]
    amax = result[reqs * (depth + 3):]
    stream = torch.cuda.current_stream(dev)
    ws = _workspace(dev, stream, rows)
    args_c = (logits.data_ptr(), vocab, vocab, rows, row_start.data_ptr(), reqs, flat.data_ptr(), None, None, 0,
              depth + 1, amax.data_ptr(), tokens.data_ptr(), count.data_ptr(), accepted.data_ptr(), ws.data_ptr(),
              ws.numel(), stream.cuda_stream)

    def kernel_only():  # the C ABI with resident buffers: device time of the kernel
        _lib.lib.neb_greedy_accept(*args_c)

    def api():  # the Python API, results read back as the reference's tuples need them
        greedy_accept(logits, row_start, flat, out=(tokens, count, accepted, amax))
        return result.cpu()

    steps = max(steps_arg, 50)
    us = _time_queued(kernel_only, steps, max(warmup_arg, 3)) * 1e3
    for _ in range(3):
        api()
    t0 = time.perf_counter()
    for _ in range(20):
        api()
    api_us = (time.perf_counter() - t0) / 20 * 1e6
    moved = rows * vocab * 2
    peak, peak_kind = _peaks()
    achieved = moved / (us * 1e-6) / 1e9
    line = {"metric": "greedy accept us per verify batch (Qwen3-8B: 16 requests x 5 rows x 151,936 logits)",
            "value": round(us, 2), "unit": "us", "n_gpus": 1, "steps": steps, "warmup": max(warmup_arg, 3),
            "higher_is_better": False, "scaling": "none", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": "greedy_accept_8b", "requests": reqs, "depth": depth, "vocab": vocab,
                       "l2": "the 24.3 MB of logits fit L2, as they do after the lm_head GEMM that writes them"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_kind": peak_kind, "bytes_per_call": moved},
            "gpu_launches": steps,
            "e2e": {"value": round(api_us, 2), "unit": "us", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": result.numel() * 4,
                    "api": "nebulasd_b200.accept.greedy_accept + copy of the results to the host"}}
    if R.available():
        spec = R.swiftllm("speculative")
        dl = drafts.tolist()

        def ref():
            post = torch.argmax(logits, dim=1).tolist()
            return [spec.compute_greedy_acceptance(dl[r], post[r * (depth + 1):(r + 1) * (depth + 1)])
                    for r in range(reqs)]

        for _ in range(3):
            ref()
        t0 = time.perf_counter()
        for _ in range(20):
            ref()
        ref_us = (time.perf_counter() - t0) / 20 * 1e6
        line["reference_gpu"] = {"impl": "torch.argmax + .tolist() + compute_greedy_acceptance (host), same logits",
                                 "us": round(ref_us, 2), "host_sync": True}
    return line


def run_accept(args):
    world, rank, local = _dist()
    if rank != 0:
        return
    torch.cuda.set_device(local)
    line = accept_line(torch.device("cuda", local), args.steps, args.warmup, args.requests)
    print(json.dumps(line), flush=True)


def prefill_line(dev, steps_arg, warmup_arg, requests=None):
    """Causal prefill attention of one Qwen3-8B layer (32 q / 8 kv heads, head
    dim 128) over a packed batch of ragged prompts (seeded lengths U[64, 2048],
    --requests prompts, default 16): the drop-in ``flash_attn_varlen_func``
    (a one-CTA plan launch, then the tcgen05 prefill kernel) against the
    reference's own function on the same GPU (``transformer_layer.py:7-32``:
    ``cu_seqlens`` to the host, one ``scaled_dot_product_attention`` per
    prompt).  q, k and v (about 170 MB) are larger than L2."""
    from nebulasd_b200.kernels import flash_attn_varlen_func
    from baseline import reference as R
    nseq = requests or 16
    g = torch.Generator().manual_seed(4242)
    lens = torch.randint(64, 2049, (nseq,), generator=g).tolist()
    heads, kv_heads, dim = 32, 8, 128
    tokens = sum(lens)
    gd = torch.Generator(device=dev).manual_seed(17)
    q = torch.randn((tokens, heads, dim), generator=gd, device=dev).half()
    k = torch.randn((tokens, kv_heads, dim), generator=gd, device=dev).half()
    v = torch.randn((tokens, kv_heads, dim), generator=gd, device=dev).half()
    cu = torch.tensor([0] + torch.cumsum(torch.tensor(lens), 0).tolist(), dtype=torch.int32, device=dev)
    scale = dim ** -0.5

    def ours():
        return flash_attn_varlen_func(q, k, v, cu, cu, max(lens), max(lens), softmax_scale=scale, causal=True)

    steps, warm = max(steps_arg, 20), max(warmup_arg, 3)
    ms = _time_steps(ours, steps, warm)
    # QK^T and PV over the causal triangle: 4 * heads * dim FLOPs per (query, key) pair
    flops = sum(4 * heads * dim * n * (n + 1) / 2 for n in lens)
    peak = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())["bf16_tflops"] \
        if (ROOT / "MEASURED_PEAKS.json").exists() else 1590.0
    tflops = flops / (ms * 1e-3) / 1e12
    line = {"metric": "prefill attention ms per layer call (Qwen3-8B heads, packed ragged prompts)",
            "value": round(ms, 4), "unit": "ms", "n_gpus": 1, "steps": steps, "warmup": warm,
            "higher_is_better": False, "scaling": "none", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": "prefill_8b", "prompts": nseq, "tokens": tokens, "max_len": max(lens),
                       "heads": heads, "kv_heads": kv_heads},
            "tokens_per_s": round(tokens / (ms * 1e-3)),
            "roofline": {"bound": "tensor", "achieved": round(tflops, 1), "peak": peak, "unit": "TFLOP/s",
                         "frac": round(tflops / peak, 4), "flops_per_call": flops,
                         "note": "whole call (plan launch included) against the fp16 causal-triangle FLOPs"},
            "gpu_launches": 2 * steps}
    if R.available():
        ref_fn = R.swiftllm("worker.layers.transformer_layer").flash_attn_varlen_func

        def ref():
            return ref_fn(q, k, v, cu, cu, max(lens), max(lens), softmax_scale=scale, causal=True)

        for _ in range(warm):
            ref()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(steps):
            ref()
        torch.cuda.synchronize()
        ref_ms = (time.perf_counter() - t0) / steps * 1e3
        err = (ours().float() - ref().float()).abs().max().item()
        line["reference_gpu"] = {"impl": "the reference's flash_attn_varlen_func (per-prompt SDPA, host sync)",
                                 "ms": round(ref_ms, 4), "speedup": round(ref_ms / ms, 3),
                                 "max_abs_diff": err}
        # One 8,192-token prompt: the reference's loop is then a single SDPA call.
        n1 = 8192
        q1 = torch.randn((n1, heads, dim), generator=gd, device=dev).half()
        k1 = torch.randn((n1, kv_heads, dim), generator=gd, device=dev).half()
        v1 = torch.randn((n1, kv_heads, dim), generator=gd, device=dev).half()
        cu1 = torch.tensor([0, n1], dtype=torch.int32, device=dev)
        ours_1 = _time_steps(lambda: flash_attn_varlen_func(q1, k1, v1, cu1, cu1, n1, n1, softmax_scale=scale),
                             steps, warm)
        for _ in range(warm):
            ref_fn(q1, k1, v1, cu1, cu1, n1, n1, softmax_scale=scale, causal=True)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(steps):
            ref_fn(q1, k1, v1, cu1, cu1, n1, n1, softmax_scale=scale, causal=True)
        torch.cuda.synchronize()
        ref_1 = (time.perf_counter() - t0) / steps * 1e3
        fl1 = 4 * heads * dim * n1 * (n1 + 1) / 2
        line["one_prompt_8k"] = {"ours_ms": round(ours_1, 4), "ours_tflops": round(fl1 / ours_1 / 1e9, 1),
                                 "reference_ms": round(ref_1, 4), "reference_tflops": round(fl1 / ref_1 / 1e9, 1)}
    return line


def run_prefill(args):
    world, rank, local = _dist()
    if rank != 0:
        return
    torch.cuda.set_device(local)
    line = prefill_line(torch.device("cuda", local), args.steps, args.warmup, args.requests)
    print(json.dumps(line), flush=True)


def run_long_hostkv(args):
    world, rank, local = _dist()
    if rank != 0:
        return
    torch.cuda.set_device(local)
    line = long_hostkv_line(args.workload.replace("_hostkv", ""), torch.device("cuda", local), args.steps,
                            args.requests)
    line["config"]["workload"] = args.workload
    print(json.dumps(line), flush=True)


def long_hostkv_line(workload, dev, steps_arg, requests=None):
    """Config 4 with its HostKV traffic (rank 0): 64 requests, ctx U[8K, 32K];
    bank B (a quarter of the requests) restores its full KV from the pinned
    host arena through NativeCopyBackend while bank A (the rest) runs
    long-context verify, and every verify round writes bank A's changed blocks
    (the k+1 new tokens) back on a second backend stream (``fork``).  The arena,
    extents and plans are the reference's (``SharedHostKVArena``, ``CopyPlan``)."""
    import numpy as np
    from baseline import reference as R
    from nebulasd_b200.hostkv import NativeCopyBackend
    from nebulasd_b200.kernels import paged_attention_raw
    metric = f"long-context verify TB/s with HostKV restore overlapped ({workload})"
    if not R.available():
        return {"metric": metric, "unavailable": "reference not installed under baseline/_ref", "config": {}}
    arena_mod, tr = R.nebulasd("kv.arena"), R.nebulasd("kv.transfer")
    b, layers, cfg = build_workload(workload, 1234, dev, None, requests)
    nreq = cfg["num_requests"]
    nb_restore = nreq // 4
    bt = b.block_table.cpu().numpy()
    depths = list(b.depths)
    ctx = list(b.ctx)
    row_first = np.cumsum([0] + [d + 1 for d in depths])
    # Bank A: requests nb_restore.. (their rows are the tail of the batch).
    ra = int(row_first[nb_restore])
    qa, lens_a, ids_a = b.q[ra:].contiguous(), b.seq_lens[ra:].contiguous(), b.seq_ids[ra:].contiguous()
    oa = torch.empty_like(qa)
    scale = b.q.shape[-1] ** -0.5
    a_bytes = int(sum(-(-(c + d + 1) // 16) for c, d in zip(ctx[nb_restore:], depths[nb_restore:]))) \
        * b.num_kv_heads * 16 * 128 * 2 * 2
    block_bytes = b.k_cache[0].numel() * 2
    kv_shape = tuple(b.k_cache.shape[1:])
    restore_blocks = [-(-ctx[i] // 16) for i in range(nb_restore)]
    wb_blocks = 2
    total_host = sum(restore_blocks) + wb_blocks * (nreq - nb_restore)
    try:
        arena = arena_mod.SharedHostKVArena.create(total_blocks=total_host, block_bytes=block_bytes,
                                                   dtype=str(b.k_cache.dtype), kv_block_shape=kv_shape)
    except OSError as e:
        return {"metric": metric, "unavailable": f"shared-memory arena: {e}", "config": {}}
    host = np.ctypeslib.as_array((__import__("ctypes").c_uint8 * arena.descriptor.total_bytes)
                                 .from_address(arena.address()))
    host[:] = np.random.default_rng(7).integers(0, 256, host.shape[0], dtype=np.uint8)
    regions, off = [], 0
    for i in range(nb_restore):
        ext = arena.make_extent(request_slot=i, request_epoch=1, host_slot=i, host_slot_generation=1,
                                writer_lease_generation=1, offset_blocks=off, capacity_blocks=restore_blocks[i])
        j = 0
        while j < restore_blocks[i]:  # one region per run of consecutive GPU blocks
            n = 1
            while j + n < restore_blocks[i] and bt[i, j + n] == bt[i, j] + n:
                n += 1
            regions.append(tr.CopyRegion(ext, int(bt[i, j]), j, n))
            j += n
        off += restore_blocks[i]
    restore_plan = tr.CopyPlan("H2D", tuple(regions))
    wb_regions = []
    for k, i in enumerate(range(nb_restore, nreq)):
        ext = arena.make_extent(request_slot=nb_restore + k, request_epoch=1, host_slot=nb_restore + k,
                                host_slot_generation=1, writer_lease_generation=1, offset_blocks=off,
                                capacity_blocks=wb_blocks)
        first, last = ctx[i] // 16, (ctx[i] + depths[i]) // 16
        for j, blk in enumerate(range(first, last + 1)):
            wb_regions.append(tr.CopyRegion(ext, int(bt[i, blk]), j, 1))
        off += wb_blocks
    wb_plan = tr.CopyPlan("D2H", tuple(wb_regions))
    restore_bytes = 2 * sum(restore_blocks) * block_bytes
    be = NativeCopyBackend(arena=arena, k_cache=b.k_cache, v_cache=b.v_cache)
    be.initialize()
    wb = be.fork()
    wb.initialize()
    comp = torch.cuda.current_stream(dev)

    def verify_round():
        paged_attention_raw(qa, b.k_cache, b.v_cache, b.block_table, lens_a, ids_a, 0, scale, oa,
                            max_len=max(b.seq_lens_list[ra:]))

    for _ in range(3):
        verify_round()
    be.launch(restore_plan).synchronize()
    torch.cuda.synchronize()
    # 1. attention alone
    steps = max(steps_arg, 10)
    ms_alone = _time_steps(verify_round, steps)
    # 2. restore alone
    t = be.launch(restore_plan)
    t.synchronize()
    restore_alone = restore_bytes / (t.duration_ms() * 1e-3) / 1e9
    restore_mode = be.last_mode
    # 3. both: verify rounds (each followed by its writeback) until the restore is done
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t = be.launch(restore_plan)
    e0.record(comp)
    rounds = 0
    while True:
        verify_round()
        ready = torch.cuda.Event()
        ready.record(comp)
        wb.launch(tr.CopyPlan("D2H", wb_plan.regions, dependencies=(ready,)))
        rounds += 1
        if rounds >= 4 and t.query():
            break
        if rounds > 20000:
            break
    e1.record(comp)
    t.synchronize()
    torch.cuda.synchronize()
    ms_both = e0.elapsed_time(e1) / rounds
    restore_both = restore_bytes / (t.duration_ms() * 1e-3) / 1e9
    # bytes check: the restored GPU blocks equal the arena (both planes, a sample of blocks)
    plane = arena.descriptor.plane_bytes
    ok = True
    for r_ in regions[:: max(1, len(regions) // 64)]:
        hb = (r_.extent.offset_blocks + r_.host_begin_block) * block_bytes
        g = b.k_cache[r_.gpu_begin_block].view(torch.uint8).cpu().numpy().reshape(-1)
        ok &= bool((g == host[hb:hb + block_bytes]).all())
        g = b.v_cache[r_.gpu_begin_block].view(torch.uint8).cpu().numpy().reshape(-1)
        ok &= bool((g == host[plane + hb:plane + hb + block_bytes]).all())
    wb.close()
    be.close()
    del host
    arena.close()
    arena.unlink()
    peak, peak_kind = _peaks()
    tb_alone = a_bytes / (ms_alone * 1e-3) / 1e12
    tb_both = a_bytes / (ms_both * 1e-3) / 1e12
    line = {"metric": metric, "value": round(tb_both, 4), "unit": "TB/s", "n_gpus": 1, "steps": rounds,
            "warmup": 3, "higher_is_better": True, "scaling": "none", "vs_baseline": None,
            "dtype": "f16 (fp32 accumulate)", "data": "synthetic",
            "config": {"workload": workload + "_hostkv", "requests": nreq, "restoring": nb_restore,
                       "verifying": nreq - nb_restore, "depth": cfg["depth"], "ctx": [cfg["ctx_lo"], cfg["ctx_hi"]],
                       "restore_regions": len(regions), "restore_bytes": restore_bytes,
                       "writeback_bytes_per_round": 2 * len(wb_regions) * block_bytes,
                       "arena": "reference SharedHostKVArena (POSIX shared memory)"},
            "attention_alone": {"tb_s": round(tb_alone, 4), "frac_of_measured_peak": round(tb_alone * 1e3 / peak, 4),
                                "launch_us": round(ms_alone * 1e3, 2)},
            "attention_during_restore": {"tb_s": round(tb_both, 4), "launch_us": round(ms_both * 1e3, 2),
                                         "rounds": rounds},
            "restore_gbs": {"alone": round(restore_alone, 2), "during_attention": round(restore_both, 2),
                            "mode": restore_mode},
            "restored_bytes_match_arena": ok,
            "roofline": {"bound": "hbm", "achieved": round(tb_both * 1e3, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(tb_both * 1e3 / peak, 4), "peak_kind": peak_kind}}
    k_cache_free(b)
    torch.cuda.empty_cache()
    return line


class _B200Ops:
    """``nebulasd_b200.install()`` for one block, then the reference's ops back."""

    def __init__(self, R):
        self.layer_mod = R.swiftllm("worker.layers.transformer_layer")
        names = (("paged_attention", "paged_attn"), ("store_kvcache", "kvcache_mgmt"),
                 ("rotary_embedding_inplace", "rotary_emb"), ("rmsnorm_inplace", "rmsnorm"))
        self.kernel_mods = {n: R.swiftllm(f"worker.kernels.{m}") for n, m in names}
        self.saved = {n: (getattr(self.layer_mod, n), getattr(self.kernel_mods[n], n)) for n, _ in names}
        self.prefill = self.layer_mod.flash_attn_varlen_func
        self.copy_mod = sys.modules.get("nebulasd.kv.cuda_transfer")
        self.copy_backend = getattr(self.copy_mod, "CudaCopyBackend", None)

    def __enter__(self):
        import nebulasd_b200
        nebulasd_b200.install()
        return self

    def __exit__(self, *exc):
        for n, (layer_fn, mod_fn) in self.saved.items():
            setattr(self.layer_mod, n, layer_fn)
            setattr(self.kernel_mods[n], n, mod_fn)
        self.layer_mod.flash_attn_varlen_func = self.prefill
        if self.copy_mod is not None:
            self.copy_mod.CudaCopyBackend = self.copy_backend
        return False


def run_spec_e2e(args):
    """Config 5 reduced to one GPU: greedy speculative decoding (depth 4) of
    16 requests (prompts of U[128, 1024] random token ids) by a random-init
    Qwen3-0.6B Draft and Qwen3-8B Target, both the reference's own
    ``LlamaModel`` (``swiftLLM/swiftllm/worker/model.py``) on one B200, each
    round: the Draft catches up on the committed tokens and proposes 4, the
    Target verifies the 5 rows per request, ``compute_greedy_acceptance``
    (``speculative.py:122-156``) commits.  Run twice, with the reference's
    kernels and after ``nebulasd_b200.install()``; reports tokens/s and the
    share of the rounds' time spent in paged attention."""
    world, rank, local = _dist()
    if rank != 0:
        return
    import random
    import tempfile
    from baseline import reference as R
    metric = "speculative decoding tokens/s (random-init Qwen3-0.6B Draft + Qwen3-8B Target, one B200, depth 4)"
    if not R.available():
        print(json.dumps({"metric": metric, "unavailable": "reference not installed under baseline/_ref"}), flush=True)
        return
    torch.cuda.set_device(local)
    spec = R.swiftllm("speculative")
    reqs, depth, rounds = args.requests or 16, 4, max(args.steps, 8)
    rng = random.Random(2026)
    prompts = [[rng.randrange(151936) for _ in range(rng.randint(128, 1024))] for _ in range(reqs)]
    mbs = (1024 + (rounds + 2) * (depth + 1)) // 16 + 2
    tmp = tempfile.mkdtemp(prefix="neb_spec_")
    kw = dict(max_seqs=reqs, max_blocks_per_seq=mbs, num_blocks=reqs * mbs, max_batch=reqs * (depth + 2) * 4,
              max_tokens=sum(len(p) for p in prompts) + 64)
    draft = R.random_llama(R.QWEN3_0P6B, tmp + "/draft", 1, **kw)
    target = R.random_llama(R.QWEN3_8B, tmp + "/target", 2, **kw)
    bt = torch.arange(reqs * mbs, dtype=torch.int32, device="cuda").view(reqs, mbs).contiguous()
    ids = list(range(reqs))
    layer_mod = R.swiftllm("worker.layers.transformer_layer")

    def arm():
        attn = []
        inner = layer_mod.paged_attention

        def timed(*a, **k):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            inner(*a, **k)
            e1.record()
            attn.append((e0, e1))

        layer_mod.paged_attention = timed
        try:
            committed = [list(p) for p in prompts]
            first = target.forward(prompts, ids, [], kv_block_table=bt)
            draft.forward(prompts, ids, [], kv_block_table=bt)
            for r in ids:
                committed[r].append(first[r])
            draft_len = [len(p) for p in prompts]
            torch.cuda.synchronize()
            attn.clear()
            t0 = time.perf_counter()
            for _ in range(rounds):
                rows, rids, lens, last = [], [], [], []
                for r in ids:  # the Draft catches up, then proposes
                    for pos in range(draft_len[r], len(committed[r])):
                        rows.append([committed[r][pos]])
                        rids.append(r)
                        lens.append(pos + 1)
                    last.append(len(rows) - 1)
                    draft_len[r] = len(committed[r])
                out = draft.forward(rows, rids, lens, kv_block_table=bt)
                drafts = [[out[i]] for i in last]
                for j in range(1, depth):
                    out = draft.forward([[d[-1]] for d in drafts], ids, [len(committed[r]) + j for r in ids],
                                        kv_block_table=bt)
                    for r in ids:
                        drafts[r].append(out[r])
                vrows = [[t] for r in ids for t in [committed[r][-1]] + drafts[r]]
                vlens = [len(committed[r]) + i for r in ids for i in range(depth + 1)]
                post = target.forward(vrows, [r for r in ids for _ in range(depth + 1)], vlens, kv_block_table=bt)
                for r in ids:
                    acc, _ = spec.compute_greedy_acceptance(drafts[r], post[r * (depth + 1):(r + 1) * (depth + 1)])
                    committed[r] += acc
            torch.cuda.synchronize()
            secs = time.perf_counter() - t0
            attn_ms = sum(a.elapsed_time(b) for a, b in attn)
        finally:
            layer_mod.paged_attention = inner
        new = sum(len(c) - len(p) - 1 for c, p in zip(committed, prompts))
        return {"tokens_per_s": round(new / secs, 1), "round_ms": round(secs * 1e3 / rounds, 3),
                "attention_ms_per_round": round(attn_ms / rounds, 3),
                "attention_share": round(attn_ms / (secs * 1e3), 4), "tokens": new}, committed

    arm()  # warm-up: Triton JIT and the first calls of both models
    ref, ref_tokens = arm()
    with _B200Ops(R):
        arm()
        ours, our_tokens = arm()
    same = sum(a == b for a, b in zip(ref_tokens, our_tokens))
    line = {"metric": metric, "value": ours["tokens_per_s"], "unit": "tokens/s", "n_gpus": 1, "steps": rounds,
            "warmup": 1, "higher_is_better": True, "scaling": "none", "vs_baseline": None,
            "dtype": "f16", "data": "synthetic (random-init models, random prompt ids)",
            "config": {"workload": "spec_decode_1d1t", "requests": reqs, "depth": depth,
                       "prompt_len": [128, 1024], "rounds": rounds,
                       "models": "Qwen3-0.6B Draft (28 layers) + Qwen3-8B Target (36 layers), random init"},
            "ours": ours, "reference_kernels": ref,
            "speedup": round(ours["tokens_per_s"] / ref["tokens_per_s"], 3),
            "requests_with_identical_tokens": same}
    print(json.dumps(line), flush=True)


def main():
    args = _args()
    if args.workload == "spec_decode_1d1t":
        run_spec_e2e(args)
    elif args.workload.endswith("_hostkv"):
        run_long_hostkv(args)
    elif args.workload == "greedy_accept_8b":
        run_accept(args)
    elif args.workload == "prefill_8b":
        run_prefill(args)
    elif args.workload == "fused_store_0p6b":
        run_fused(args)
    elif args.workload == "hostkv_copy":
        run_hostkv(args)
    elif args.workload == "kv_migrate":
        run_migrate(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
