"""Benchmark: WKV-7 slot decode on B200, RWKV-7 1.5B state shape.

Workload (one "step" = one decode token for every active slot through all
layers): L=24 layers, H=32 heads, head dim N=64, a 1024-slot fp32 arena
(+ reserved slot 0, 12.9 GB), 256 active slots drawn without replacement by
seeded int32 ids. Each layer is one wkv7_decode_slots launch that reads the
256x32 head states from the arena, applies the RWKV-7 update and writes them
back in place. Inputs are seeded synthetic activations with the op-level
distributions of the reference configuration (no dataset exists for this
path). The per-step state traffic (6.4 GB) exceeds the 126 MB L2, so no L2
flush is needed between steps.

  value  — device-timed tokens/s (inputs resident in HBM, CUDA graph of the
           24 launches per step, CUDA events on the launching stream)
  e2e    — tokens/s through the public op (ops.wkv7_decode_slots) with host
           buffers: every step copies its r,w,k,v,kk,a for all layers and the
           slot ids from pinned host memory and reads every layer's o back.
  roofline — algorithmic bytes per launch / average launch time, vs the
           measured HBM copy bandwidth.

Multi-GPU: one process per GPU (torchrun), each GPU holds its own arena
shard and 256 active slots; no collective on the data path (weak scaling).

Other workloads (--workload): prefill (config 2, RWKV-7 chunk prefill into
slots), gdn-decode / gdn-prefill (config 3), model-decode (config 1 as fla's
whole RWKV-7 model step), cfg4 (config 4: 7.2B-shape decode with forks,
host snapshots and NCCL slot migration every step) and hibernate (batched
snapshot / wake of 64 sessions against wkvm's per-session copies).
``--impl reference`` times the CPU restatement of the reference recurrence
(oracle/, fp32, all host threads) on a bounded sample of the same workload.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import tempfile
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
L, H, N, NUM_SLOTS, ACTIVE = 24, 32, 64, 1024, 256
# N > 1 migration leg of the default run: 10 sessions every 4 steps (2.5 per
# step, 1 % of the 256 active), drawn from PARKED live sessions
MIG_EVERY, MIG_SLOTS, PARKED = 4, 10, 128
BYTES_PER_HEAD = 2 * N * N * 4 + 6 * N * 2 + N * 2  # state r+w, 6 inputs, o = 33,664 B
METRIC = "WKV-7 slot-decode tokens/s @1/2/4/8 B200; achieved HBM GB/s vs peak"
PROFILE = ROOT / "profiles" / "wkv7_decode_slots_cfg1.txt"


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def profiled_traffic():
    """dram bytes per launch recorded from an ncu capture (profiles/)."""
    if not PROFILE.exists():
        return None
    for line in PROFILE.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            return float(line.split(":", 1)[1])
    return None


class Clocks:
    """Samples SM clocks and throttle reasons with nvidia-smi while running."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.file = None

    def __enter__(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=self.file, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if self.proc is None or self.file is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for line in Path(self.file.name).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[5:9]))
            except ValueError:
                continue
        os.unlink(self.file.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, r in rows for i, v in enumerate(r) if v == "Active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows),
                "sm_max_mhz": max(r[1] for r in rows), "reasons": reasons,
                "samples": len(rows)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x: float, world: int, dev) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def make_inputs(dev, seed):
    from wkvm_b200 import synth
    per_layer = []
    for layer in range(L):
        x = synth.rwkv7_inputs(ACTIVE, 1, H, N, seed=seed * 1000 + layer, device=dev,
                               state=False)
        per_layer.append([x[n] for n in ("r", "w", "k", "v", "kk", "a")])
    return per_layer


def run_ours(args, world, rank, local):
    from wkvm_b200 import ops, synth
    from wkvm_b200.state import RWKV7StateBank, RWKV7StateLayout

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    layout = RWKV7StateLayout(n_layer=L, hidden_size=H * N, num_heads=H, head_dim=N,
                              head_v_dim=N, dtype=torch.bfloat16)
    bank = RWKV7StateBank(layout, NUM_SLOTS, device=dev)
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    bank.wkv.normal_(0.0, 0.1, generator=g)
    ids_host = synth.slot_ids(ACTIVE, NUM_SLOTS + 1, seed=rank)
    ids = ops.slot_ids_tensor(ids_host, NUM_SLOTS + 1, dev)
    inputs = make_inputs(dev, seed=rank)
    outs = [torch.empty(ACTIVE, 1, H, N, dtype=torch.bfloat16, device=dev) for _ in range(L)]
    ops.status_word(dev)
    # Consecutive layers overlap their launch tails (programmatic dependent
    # launch): each launch touches another layer's state, which meets the
    # op's contract for the overlap mode.
    ops.set_decode_overlap(not args.no_overlap)

    def step():
        for layer in range(L):
            ops.wkv7_decode_slots(*inputs[layer], bank.wkv, layer, ids, out=outs[layer])

    stream = torch.cuda.Stream(dev)
    stream.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(stream):
        for _ in range(3):
            step()
    torch.cuda.current_stream(dev).wait_stream(stream)
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    # N > 1: live migration around the ring, the path's only exchange. Every
    # MIG_EVERY steps MIG_SLOTS parked sessions (live slots outside this
    # step's decode batch) go to rank + 1 over one NCCL send/recv pair while
    # rank - 1's arrive in newly allocated slots; a sent slot is freed only
    # after the receiver's acknowledgement. All of it is stream-ordered on a
    # side stream beside the decode graph; the host never waits.
    mig = None
    if world > 1 and not args.no_migration:
        from wkvm_b200 import shard
        arena = shard.ShardArena(NUM_SLOTS)
        arena.claim(ids_host.tolist())
        parked = arena.allocate(PARKED)
        pack, unpack, empty = shard.bank_packer(bank)
        mig = shard.RingMigrator(pack, unpack, empty, rank, world, device=dev, timeout=60.0)

    def migrate(i):
        if mig is None or i % MIG_EVERY:
            return
        arena.free(mig.reap())
        out_ids, parked[:] = parked[:MIG_SLOTS], parked[MIG_SLOTS:]
        in_ids = arena.allocate(MIG_SLOTS)
        mig.start(out_ids, in_ids)
        parked.extend(in_ids)

    for i in range(args.warmup):
        graph.replay()
        migrate(i)
    torch.cuda.synchronize(dev)

    barrier(world)
    torch.cuda.synchronize(dev)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(dev.index if dev.index is not None else 0) as clk:
        start.record()
        for i in range(args.steps):
            graph.replay()
            migrate(i)
        if mig is not None:
            torch.cuda.current_stream(dev).wait_stream(mig.stream)
        stop.record()
        torch.cuda.synchronize(dev)
    barrier(world)
    if mig is not None:
        arena.free(mig.reap(block=True))
    ms = max_over_ranks(start.elapsed_time(stop), world, dev)
    ops.check_device_status(dev)

    # ---- end-to-end through the public op with host buffers ----
    # Per layer: pinned-host inputs -> device on a copy stream, the op on the
    # compute stream once that layer's copy landed, o -> pinned host after it.
    e2e_ms, h2d, d2h, e_steps = None, 0, 0, max(1, args.steps)
    if not args.no_e2e:
        # one pinned host buffer per layer holding its six input tensors
        # ([6, B, 1, H, N]): one 6 MB copy per layer rather than six of 1 MB
        # (51 vs 41 GB/s over PCIe, against 55 GB/s for one large copy)
        host_in = [torch.stack([t.cpu() for t in layer_in]).pin_memory() for layer_in in inputs]
        host_out = [torch.empty_like(o, device="cpu").pin_memory() for o in outs]
        dev_in = [torch.empty_like(h, device=dev) for h in host_in]
        ids_list = ids_host.tolist()
        h2d = sum(t.numel() * t.element_size() for t in host_in) + 4 * ACTIVE
        d2h = sum(o.numel() * o.element_size() for o in host_out)
        comp = torch.cuda.current_stream(dev)
        copy = torch.cuda.Stream(dev)      # host -> device
        copy_out = torch.cuda.Stream(dev)  # device -> host (the other PCIe direction)
        in_ev = [torch.cuda.Event() for _ in range(L)]
        out_ev = [torch.cuda.Event() for _ in range(L)]

        def e2e_step():
            dids = ops.slot_ids_tensor(ids_list, NUM_SLOTS + 1, dev)
            copy.wait_stream(comp)
            with torch.cuda.stream(copy):
                for layer in range(L):
                    dev_in[layer].copy_(host_in[layer], non_blocking=True)
                    in_ev[layer].record(copy)
            for layer in range(L):
                comp.wait_event(in_ev[layer])
                ops.wkv7_decode_slots(*dev_in[layer].unbind(0), bank.wkv, layer, dids,
                                      out=outs[layer])
                out_ev[layer].record(comp)
            with torch.cuda.stream(copy_out):
                for layer in range(L):
                    copy_out.wait_event(out_ev[layer])
                    host_out[layer].copy_(outs[layer], non_blocking=True)
            comp.wait_stream(copy)
            comp.wait_stream(copy_out)

        for _ in range(args.warmup):
            e2e_step()
        torch.cuda.synchronize(dev)
        barrier(world)
        s2, t2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record()
        for _ in range(e_steps):
            e2e_step()
        t2.record()
        torch.cuda.synchronize(dev)
        e2e_ms = max_over_ranks(s2.elapsed_time(t2), world, dev)
        ops.check_device_status(dev)

    if rank != 0:
        return None
    step_ms = ms / args.steps
    launch_ms = step_ms / L
    per_slot_bytes = layout.wkv_bytes_per_slot() + layout.shift_bytes_per_slot()
    bytes_per_launch = ACTIVE * H * BYTES_PER_HEAD
    achieved = bytes_per_launch / (launch_ms * 1e-3) / 1e9
    peak, peak_kind = peaks()
    tokens_per_s = world * ACTIVE * args.steps / (ms * 1e-3)
    traffic = profiled_traffic()
    line = {
        "metric": METRIC,
        "value": round(tokens_per_s, 1),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(step_ms, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16 in/out, fp32 state",
        "data": "synthetic (seeded, reference op-level distributions)",
        "config": {
            "workload": f"RWKV-7 1.5B-shape WKV slot decode: L={L} H=32 N=64, 256 active of "
                        "1024 arena slots per GPU, all layers per step",
            "global_batch": ACTIVE * world,
            "slots_per_gpu": NUM_SLOTS,
            "parallelism": f"slot-sharded x{world}, no collective on the decode path"
                           + ("" if mig is None else "; ring migration over NCCL send/recv"),
            "graph": f"CUDA graph of {L} per-layer launches"
                     + ("" if args.no_overlap else ", programmatic dependent launch between layers"),
            "l2": "no flush: 6.4 GB state traffic per step > 126 MB L2",
            "migration": None if mig is None else (
                f"{MIG_SLOTS} parked sessions ({MIG_SLOTS * per_slot_bytes} B) every {MIG_EVERY} "
                "steps to rank+1 over one NCCL send/recv pair, restored on arrival, freed at "
                "the source after the receiver's acknowledgement; side stream, inside the "
                "timed region"),
        },
        "roofline": {
            "bound": "hbm",
            "kernel": "wkv7_recurrent_kernel<64,16,bf16,mul> (wkv7_decode_slots)",
            "achieved": round(achieved, 1),
            "peak": peak,
            "unit": "GB/s",
            "frac": round(achieved / peak, 4),
            "peak_kind": f"{peak_kind} hbm_gbs",
            "bytes_per_launch": bytes_per_launch,
            "traffic": traffic,
        },
        "clocks": clk.summary(),
        "gpu_launches": L * args.steps + (0 if mig is None else 4 * ((args.steps + MIG_EVERY - 1) // MIG_EVERY)),
        "e2e": None if e2e_ms is None else {
            "value": round(world * ACTIVE * e_steps / (e2e_ms * 1e-3), 1),
            "unit": "tokens/s",
            "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h,
            "path": "ops.wkv7_decode_slots with pinned-host inputs/outputs and host slot ids; "
                    "each layer's six inputs in one pinned buffer, one copy per layer and "
                    "direction on one stream per PCIe direction, overlapping the ops",
        },
    }
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args.cpu_sample_slots)
    return line


def run_prefill(args, world, rank, local):
    """Chunked RWKV-7 prefill of BASELINE config 2 (B=16 sequences x 4096
    tokens, H=32, N=64, chunk 64) through wkv7_prefill_slots: initial state
    read from and final state written to arena slots."""
    from wkvm_b200 import ops, synth

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    B, T = args.prefill_batch, 4096
    bank = torch.zeros(1, B + 1, H, N, N, device=dev)
    bank.normal_(0.0, 0.1, generator=torch.Generator(device=dev).manual_seed(7 + rank))
    x = synth.rwkv7_inputs(B, T, H, N, seed=rank, device=dev, state=False)
    ids = ops.slot_ids_tensor(list(range(1, B + 1)), B + 1, dev)
    o = torch.empty_like(x["v"])
    ops.status_word(dev)

    def step():
        ops.wkv7_prefill_slots(x["r"], x["w"], x["k"], x["v"], x["kk"], x["a"], bank, 0, ids,
                               out=o)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    barrier(world)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(dev.index if dev.index is not None else 0) as clk:
        start.record()
        for _ in range(args.steps):
            step()
        stop.record()
        torch.cuda.synchronize(dev)
    barrier(world)
    ms = max_over_ranks(start.elapsed_time(stop), world, dev)
    ops.check_device_status(dev)
    fla_arm = None
    if not args.no_fla:
        def fla_step():
            from fla.ops.rwkv7 import chunk_rwkv7 as fla_chunk
            a = -x["kk"]
            b = (x["kk"].float() * x["a"].float()).to(x["kk"].dtype)
            fla_chunk(x["r"], x["w"], x["k"], x["v"], a, b, scale=1.0,
                      initial_state=bank[0, 1:B + 1], output_final_state=True)
        fla_arm = time_fla(fla_step, args.steps, args.warmup, dev)
        fla_arm["path"] = "fla.ops.rwkv7.chunk_rwkv7 (Triton), same inputs, state from the bank"
    if rank != 0:
        return None
    step_ms = ms / args.steps
    token_heads = B * T * H
    flops = token_heads * 109.2e3          # WY-form FLOPs per token-head (N = 64, C = 64)
    byts = token_heads * 896 + 2 * B * H * N * N * 4
    hbm_peak, _ = peaks()
    return {
        "metric": "WKV-7 chunked prefill tokens/s (BASELINE config 2)",
        "value": round(world * B * T * args.steps / (ms * 1e-3), 1), "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(step_ms, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16 in/out, tf32 tensor-core operands, fp32 state",
        "data": "synthetic (seeded, reference op-level distributions)",
        "config": {"workload": f"B={B} T={T} H=32 N=64 chunk 64, state in arena slots",
                   "kernel": "dplr_chunk_kernel (tcgen05 kind::tf32)"},
        "roofline": {"bound": "hbm", "achieved": round(byts / (step_ms * 1e-3) / 1e9, 1),
                     "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(byts / (step_ms * 1e-3) / 1e9 / hbm_peak, 4),
                     "bytes_per_launch": int(byts), "flops_per_launch": int(flops),
                     **tensor_roof(flops, step_ms)},
        "clocks": clk.summary(), "gpu_launches": args.steps,
        "same_box_fla": fla_arm,
    }


def time_fla(fn, steps: int, warmup: int, dev) -> dict:
    """The same call through flash-linear-attention's own Triton kernel on the
    same box and inputs (the GPU implementation wkvm runs today), CUDA
    events; {"unavailable": why} when fla cannot run here."""
    try:
        for _ in range(max(warmup, 2)):
            fn()
        torch.cuda.synchronize(dev)
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        for _ in range(steps):
            fn()
        s1.record()
        torch.cuda.synchronize(dev)
        return {"ms_per_step": round(s0.elapsed_time(s1) / steps, 4)}
    except Exception as e:  # fla missing or failing on this box
        return {"unavailable": f"{type(e).__name__}: {str(e)[:160]}"}


def tensor_roof(flops: float, ms: float) -> dict:
    """Tensor-pipe figures of a tf32 tensor-core launch: achieved TFLOP/s
    against the tf32 dense rate, taken as half the measured bf16 GEMM rate,
    burst (the kernel timed alone) and sustained (under the power cap)."""
    p = ROOT / "MEASURED_PEAKS.json"
    d = json.loads(p.read_text()) if p.exists() else {}
    kind = "measured" if d else "fallback"
    burst = d.get("bf16_tflops", 1590.0) / 2
    sustained = d.get("bf16_tflops_sustained", 1400.0) / 2
    tf = flops / (ms * 1e-3) / 1e12
    return {"tensor_tflops": round(tf, 2), "tensor_peak_tflops": burst,
            "tensor_frac": round(tf / burst, 4),
            "tensor_peak_sustained_tflops": sustained,
            "tensor_frac_sustained": round(tf / sustained, 4),
            "tensor_peak_kind": f"{kind} bf16_tflops / 2 and bf16_tflops_sustained / 2 "
                                "(tf32 dense rate)"}


def run_gdn(args, world, rank, local):
    """BASELINE config 3, gated delta rule (H=16, K=V=128): decode of B=512
    slots in place in a 513-slot arena (--workload gdn-decode), or chunked
    prefill of B=4 x 8192 tokens into slots (--workload gdn-prefill)."""
    from wkvm_b200 import ops, synth

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    decode = args.workload == "gdn-decode"
    B, T, HG, K = (512, 1, 16, 128) if decode else (args.gdn_batch, 8192, 16, 128)
    bank = torch.empty(1, B + 1, HG, K, K, device=dev)
    bank.normal_(0.0, 0.1, generator=torch.Generator(device=dev).manual_seed(11 + rank))
    ids = ops.slot_ids_tensor(list(range(1, B + 1)), B + 1, dev)
    x = synth.gdn_inputs(B, T, HG, K, seed=rank, device=dev, state=False)
    o = torch.empty_like(x["v"])
    ops.status_word(dev)

    def step():
        if decode:
            ops.gdn_decode_slots(x["q"], x["k"], x["v"], x["g"], x["beta"], bank, 0, ids, out=o)
        else:
            from wkvm_b200 import prefill
            prefill.gdn_prefill_slots(x["q"], x["k"], x["v"], x["g"], x["beta"], bank, 0, ids,
                                      K ** -0.5, False, out=o)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    barrier(world)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(dev.index if dev.index is not None else 0) as clk:
        start.record()
        for _ in range(args.steps):
            step()
        stop.record()
        torch.cuda.synchronize(dev)
    barrier(world)
    ms = max_over_ranks(start.elapsed_time(stop), world, dev)
    ops.check_device_status(dev)
    fla_arm = None
    if not args.no_fla:
        def fla_step():
            h0 = bank[0, 1:B + 1]
            if decode:
                from fla.ops.gated_delta_rule import fused_recurrent_gated_delta_rule as f
            else:
                from fla.ops.gated_delta_rule import chunk_gated_delta_rule as f
            f(x["q"], x["k"], x["v"], x["g"], x["beta"], scale=K ** -0.5, initial_state=h0,
              output_final_state=True)
        fla_arm = time_fla(fla_step, args.steps, args.warmup, dev)
        fla_arm["path"] = (f"fla.ops.gated_delta_rule.{'fused_recurrent' if decode else 'chunk'}"
                           "_gated_delta_rule (Triton), same inputs, state gathered from the bank")
    if rank != 0:
        return None
    step_ms = ms / args.steps
    hbm_peak, kind = peaks()
    th = B * T * HG  # token-heads
    if decode:
        byts = B * HG * 132100          # state r+w 128 KiB + q,k,v,g,beta + o per slot-head
        line_roof = {"bound": "hbm", "achieved": round(byts / (step_ms * 1e-3) / 1e9, 1),
                     "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(byts / (step_ms * 1e-3) / 1e9 / hbm_peak, 4),
                     "peak_kind": f"{kind} hbm_gbs", "bytes_per_launch": byts}
        kernel = "gdn_recurrent_kernel<128,128,16> (gdn_decode_slots)"
    else:
        byts = th * 1028 + 2 * B * HG * K * K * 4
        line_roof = {"bound": "hbm", "achieved": round(byts / (step_ms * 1e-3) / 1e9, 1),
                     "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(byts / (step_ms * 1e-3) / 1e9 / hbm_peak, 4),
                     "peak_kind": f"{kind} hbm_gbs", "bytes_per_launch": int(byts),
                     "flops_per_launch": int(th * 183e3), **tensor_roof(th * 183e3, step_ms)}
        from wkvm_b200 import _lib
        line_roof["workspace_bytes_per_step"] = int(
            _lib.load().wkvm_gdn_chunk_workspace_bytes(B, T, HG, K, K))
        kernel = ("gdn_wy_kernel (chunk-parallel WY, tcgen05 kind::f16 + kind::tf32) -> "
                  "gdn_state_kernel (sequential state pass, tcgen05 kind::tf32)")
    return {
        "metric": f"GDN {'decode' if decode else 'chunked prefill'} tokens/s (BASELINE config 3)",
        "value": round(world * B * T * args.steps / (ms * 1e-3), 1), "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(step_ms, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16 in/out, fp32 state",
        "data": "synthetic (seeded, reference op-level distributions)",
        "config": {"workload": f"B={B} T={T} H=16 K=V=128, state in arena slots",
                   "kernel": kernel},
        "roofline": line_roof, "clocks": clk.summary(),
        "gpu_launches": args.steps * (1 if decode else 2),
        "same_box_fla": fla_arm,
    }


def run_cfg4(args, world, rank, local):
    """RWKV-7 7.2B-shape decode (L=32, D=4096, H=64, N=64)
    over 512 active slots per GPU, with 5 % of the slots forked or
    snapshotted every step and 1 % live-migrated to the next GPU.

    One step on every rank:
      decode   32 wkv7_decode_slots launches over the 512 active slots;
      fork     13 parents copied into 13 new slots (slot_copy, all families);
               13 other requests finish and free their slots (512 stay active);
      snapshot 13 slots packed on the device (slot_snapshot kernel), then
               copied to pinned host memory on a copy stream that overlaps the
               next step (wkvm's hibernate / StateStore.save tier);
      migrate  (N > 1) 5 slots packed and sent to rank+1 while 5 arrive from
               rank-1 into newly allocated slots: one NCCL send/recv pair per
               step over NVLink, the only collective traffic.
    The migration skips shard.send_slots' host acknowledgement (a bench has
    no peer failures to survive); the packed buffers are stream-ordered."""
    import random
    import torch.distributed as dist
    from wkvm_b200 import ops, shard, synth
    from wkvm_b200.state import RWKV7StateBank, RWKV7StateLayout

    L4, H4, ACT, SLOTS = 32, 64, 512, 600
    N_FORK, N_SNAP, N_MIG = 13, 13, (5 if world > 1 else 0)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    layout = RWKV7StateLayout(n_layer=L4, hidden_size=H4 * N, num_heads=H4, head_dim=N,
                              head_v_dim=N, dtype=torch.bfloat16)
    bank = RWKV7StateBank(layout, SLOTS, device=dev)
    bank.wkv.normal_(0.0, 0.1, generator=torch.Generator(device=dev).manual_seed(99 + rank))
    arena = shard.ShardArena(SLOTS)
    active = arena.allocate(ACT)
    inputs = []
    for layer in range(L4):
        x = synth.rwkv7_inputs(ACT, 1, H4, N, seed=rank * 1000 + layer, device=dev, state=False)
        inputs.append([x[n] for n in ("r", "w", "k", "v", "kk", "a")])
    outs = [torch.empty(ACT, 1, H4, N, dtype=torch.bfloat16, device=dev) for _ in range(L4)]
    pack, unpack, empty = shard.bank_packer(bank)
    per_slot = layout.wkv_bytes_per_slot() + layout.shift_bytes_per_slot()
    pinned = [torch.empty(N_SNAP * per_slot, dtype=torch.uint8).pin_memory() for _ in range(2)]
    snap_done = [None, None]
    copy = torch.cuda.Stream(dev)
    comp = torch.cuda.current_stream(dev)
    ids_host = [torch.empty(ACT, dtype=torch.int32).pin_memory() for _ in range(2)]
    ids_sent = [None, None]
    ids_dev = torch.empty(ACT, dtype=torch.int32, device=dev)
    rng = random.Random(1234 + rank)
    ops.status_word(dev)
    ops.set_decode_overlap(not args.no_overlap)
    dec_ev = []

    def step(i, timed):
        nonlocal active
        h = ids_host[i & 1]
        if ids_sent[i & 1] is not None:
            ids_sent[i & 1].synchronize()  # its previous upload has been read
        h.copy_(torch.tensor(active, dtype=torch.int32))
        ids_dev.copy_(h, non_blocking=True)
        ids_sent[i & 1] = torch.cuda.Event()
        ids_sent[i & 1].record(comp)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(comp)
        for layer in range(L4):
            ops.wkv7_decode_slots(*inputs[layer], bank.wkv, layer, ids_dev, out=outs[layer])
        e1.record(comp)
        if timed:
            dec_ev.append((e0, e1))
        # fork 13 parents into new slots; 13 other requests finish
        parents = rng.sample(active, N_FORK)
        children = arena.allocate(N_FORK)
        ops.slot_copy(bank.wkv, 1, parents, children)
        ops.slot_copy(bank.shift, 2, parents, children)
        done = rng.sample([a for a in active if a not in set(parents)], N_FORK)
        arena.free(done)
        gone = set(done)
        active = [a for a in active if a not in gone] + children
        # snapshot 13 slots: device pack, then device -> pinned host on the copy stream
        snap = rng.sample(active, N_SNAP)
        buf = pack(snap)
        b = i & 1
        if snap_done[b] is not None:
            snap_done[b].synchronize()  # that pinned buffer's previous copy landed
        copy.wait_stream(comp)
        with torch.cuda.stream(copy):
            pinned[b].copy_(buf, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(copy)
        buf.record_stream(copy)
        snap_done[b] = ev
        # live migration of 5 slots to the next rank, 5 in from the previous
        if N_MIG:
            out_ids = rng.sample(active, N_MIG)
            sendbuf = pack(out_ids)
            recvbuf = empty(N_MIG)
            reqs = dist.batch_isend_irecv([
                dist.P2POp(dist.isend, sendbuf, (rank + 1) % world),
                dist.P2POp(dist.irecv, recvbuf, (rank - 1) % world)])
            for r in reqs:
                r.wait()
            in_ids = arena.allocate(N_MIG)
            unpack(in_ids, recvbuf)
            arena.free(out_ids)
            gone = set(out_ids)
            active = [a for a in active if a not in gone] + in_ids

    for i in range(args.warmup):
        step(i, False)
    torch.cuda.synchronize(dev)
    barrier(world)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(dev.index if dev.index is not None else 0) as clk:
        start.record(comp)
        for i in range(args.steps):
            step(args.warmup + i, True)
        comp.wait_stream(copy)
        stop.record(comp)
        torch.cuda.synchronize(dev)
    barrier(world)
    ms = max_over_ranks(start.elapsed_time(stop), world, dev)
    dec_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in dec_ev) / args.steps, world, dev)
    ops.check_device_status(dev)
    if rank != 0:
        return None
    step_ms = ms / args.steps
    dec_bytes = ACT * L4 * H4 * BYTES_PER_HEAD
    peak, peak_kind = peaks()
    achieved = dec_bytes / (dec_ms * 1e-3) / 1e9
    return {
        "metric": "RWKV-7 7.2B-shape slot decode tokens/s with fork/snapshot/migration "
                  "(BASELINE config 4)",
        "value": round(world * ACT * args.steps / (ms * 1e-3), 1), "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(step_ms, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16 in/out, fp32 state",
        "data": "synthetic (seeded, reference op-level distributions)",
        "config": {"workload": f"L={L4} D=4096 H={H4} N=64, {ACT} active of {SLOTS} arena slots "
                               f"per GPU; per step {N_FORK} forks + {N_FORK} finished, "
                               f"{N_SNAP} snapshots to pinned host, {N_MIG} slots migrated to "
                               "the next GPU (NCCL send/recv)",
                   "global_batch": ACT * world,
                   "parallelism": f"slot-sharded x{world}; migration is the only exchange",
                   "l2": "no flush: 35 GB of state traffic per step > 126 MB L2"},
        "decode_ms_per_step": round(dec_ms, 4),
        "bytes_per_step": {"decode_state": dec_bytes,
                           "fork_copy": 2 * N_FORK * per_slot,
                           "snapshot_d2h": N_SNAP * per_slot,
                           "migration_nvlink_out": N_MIG * per_slot},
        "roofline": {"bound": "hbm",
                     "kernel": "wkv7_recurrent_kernel<64,16,bf16,mul> (wkv7_decode_slots)",
                     "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_kind": f"{peak_kind} hbm_gbs",
                     "bytes_per_launch": dec_bytes // L4, "traffic": None},
        "clocks": clk.summary(),
        "gpu_launches": args.steps * (L4 + 2 + 4 + (4 if N_MIG else 0)),
    }


def run_hibernate(args, world, rank, local):
    """Snapshot tier: hibernate 64 sessions of the RWKV-7
    1.5B state shape (12.19 MiB each) from the arena to pinned host memory
    and wake them back, batched (store_io: one kernel per family per batch)
    versus the reference's per-session flow (wkvm/store.py:127-133: strided
    view .copy_ into pinned memory, then a device synchronise per session)."""
    from wkvm_b200 import ops, store_io, synth
    from wkvm_b200.state import RWKV7StateBank, RWKV7StateLayout

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    NS = 64
    layout = RWKV7StateLayout(n_layer=L, hidden_size=H * N, num_heads=H, head_dim=N,
                              head_v_dim=N, dtype=torch.bfloat16)
    bank = RWKV7StateBank(layout, NUM_SLOTS, device=dev)
    bank.wkv.normal_(0.0, 0.1, generator=torch.Generator(device=dev).manual_seed(3))
    sess = synth.slot_ids(NS, NUM_SLOTS + 1, seed=rank).tolist()
    back = [s for s in range(1, NUM_SLOTS + 1) if s not in set(sess)][:NS]
    per = layout.wkv_bytes_per_slot() + layout.shift_bytes_per_slot()
    ops.status_word(dev)

    pool = store_io.pinned_buffers(bank, NS)

    def ours():  # steady state: a serving loop keeps its pinned buffers
        return store_io.hibernate(bank, sess, pool).wait()

    def ours_alloc():
        return store_io.hibernate(bank, sess).wait()

    def ref_save():
        out = []
        for s in sess:
            w = torch.empty(bank.wkv[:, s].shape, dtype=torch.float32, pin_memory=True)
            sh = torch.empty(bank.shift[:, :, s].shape, dtype=bank.shift.dtype, pin_memory=True)
            w.copy_(bank.wkv[:, s], non_blocking=True)
            sh.copy_(bank.shift[:, :, s], non_blocking=True)
            torch.cuda.synchronize(dev)
            out.append((w, sh))
        return out

    def wall(fn, reps):
        fn()
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        for _ in range(reps):
            r = fn()
        torch.cuda.synchronize(dev)
        return (time.perf_counter() - t0) / reps, r

    reps = max(1, args.steps)
    t_ours, batch = wall(ours, reps)
    t_alloc, _ = wall(ours_alloc, reps)
    t_ref, ref_tensors = wall(ref_save, reps)

    def ours_wake():
        store_io.wake(bank, back, batch)

    def ref_wake():
        for s, (w, sh) in zip(back, ref_tensors):
            bank.wkv[:, s].copy_(w, non_blocking=True)
            bank.shift[:, :, s].copy_(sh, non_blocking=True)
            torch.cuda.synchronize(dev)

    t_wake, _ = wall(ours_wake, reps)
    t_rwake, _ = wall(ref_wake, reps)
    ok = bool(torch.equal(bank.wkv[:, back], bank.wkv[:, sess]))
    if rank != 0:
        return None
    gb = NS * per / 1e9
    return {
        "metric": "slot hibernate (device -> pinned host) GB/s, 64 sessions of the 1.5B state",
        "value": round(gb / t_ours, 2), "unit": "GB/s", "n_gpus": world, "steps": reps,
        "warmup": 1, "ms_per_step": round(t_ours * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32 wkv + bf16 shift (bit copies)",
        "data": "synthetic states",
        "config": {"workload": f"{NS} sessions x {per / 2**20:.2f} MiB, L={L} H={H} N={N}, "
                               "host wall clock per batch incl. the final synchronise; "
                               "reused pinned buffers"},
        "with_new_pinned_buffers_gbs": round(gb / t_alloc, 2),
        "wake": {"value": round(gb / t_wake, 2), "unit": "GB/s", "ms": round(t_wake * 1e3, 3),
                 "bit_exact": ok},
        "same_box_reference": {"hibernate_gbs": round(gb / t_ref, 2),
                               "wake_gbs": round(gb / t_rwake, 2),
                               "path": "per-session strided copy_ + synchronize "
                                       "(wkvm StateStore.save / load)"},
        "gpu_launches": 2 * reps,
    }


def run_timemix(args, world, rank, local):
    """The fused time-mix decode core alone at the BASELINE config 1 shape:
    24 wkv7_timemix_decode_slots launches per step (layer 0 without v_first),
    256 active of 1024 arena slots, H=32, N=64, as a CUDA graph. Bytes per
    launch: the head states read and written (256 x 32 x 32 KiB) + the eight
    activation rows in, one out, the per-channel parameters."""
    from wkvm_b200 import ops, synth
    from wkvm_b200.state import RWKV7StateBank, RWKV7StateLayout

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    D = H * N
    layout = RWKV7StateLayout(n_layer=L, hidden_size=D, num_heads=H, head_dim=N, head_v_dim=N,
                              dtype=torch.bfloat16)
    bank = RWKV7StateBank(layout, NUM_SLOTS, device=dev)
    bank.wkv.normal_(0.0, 0.1, generator=torch.Generator(device=dev).manual_seed(5 + rank))
    ids = ops.slot_ids_tensor(synth.slot_ids(ACTIVE, NUM_SLOTS + 1, seed=rank).tolist(),
                              NUM_SLOTS + 1, dev)
    g = torch.Generator(device=dev).manual_seed(17 + rank)
    mk = lambda *sh, sc=1.0: (torch.randn(*sh, device=dev, generator=g) * sc).to(torch.bfloat16)
    acts = [[mk(ACTIVE, D) for _ in range(8)] for _ in range(L)]  # r w k v v_first v_raw a g
    prm = [[mk(D, sc=0.5), mk(D, sc=0.5), mk(H, N, sc=0.5), mk(D, sc=0.3), mk(D, sc=0.1)]
           for _ in range(L)]
    outs = [torch.empty(ACTIVE, D, dtype=torch.bfloat16, device=dev) for _ in range(L)]
    ops.status_word(dev)
    # Consecutive layers overlap their launch tails (programmatic dependent
    # launch): each launch touches another layer's state, which meets the
    # op's contract for the overlap mode.
    ops.set_decode_overlap(not args.no_overlap)

    def step():
        for layer in range(L):
            r, w, k, v, vf, vr, a, gg = acts[layer]
            kk_, ka, rk, gw, gb = prm[layer]
            ops.wkv7_timemix_decode_slots(r, w, k, v, vf if layer else None, vr if layer else None,
                                          a, gg, kk_, ka, rk, gw, gb, 64e-5, bank.wkv, layer, ids,
                                          out=outs[layer])

    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        for _ in range(3):
            step()
    torch.cuda.current_stream(dev).wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize(dev)
    barrier(world)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(dev.index if dev.index is not None else 0) as clk:
        start.record()
        for _ in range(args.steps):
            graph.replay()
        stop.record()
        torch.cuda.synchronize(dev)
    barrier(world)
    ms = max_over_ranks(start.elapsed_time(stop), world, dev)
    ops.check_device_status(dev)
    if rank != 0:
        return None
    step_ms = ms / args.steps
    per_launch = ACTIVE * H * 2 * N * N * 4 + ACTIVE * D * 2 * 9 + D * 2 * 5
    achieved = per_launch / (step_ms / L * 1e-3) / 1e9
    peak, kind = peaks()
    return {
        "metric": "fused RWKV-7 time-mix decode core tokens/s (config 1 shape)",
        "value": round(world * ACTIVE * args.steps / (ms * 1e-3), 1), "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(step_ms, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16 in/out, fp32 state and arithmetic",
        "data": "synthetic (seeded)",
        "config": {"workload": f"L={L} H={H} N={N}, {ACTIVE} active of {NUM_SLOTS} slots, "
                               "CUDA graph of the 24 launches"},
        "roofline": {"bound": "hbm", "kernel": "wkv7_timemix_decode_kernel<bf16>",
                     "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_kind": f"{kind} hbm_gbs",
                     "bytes_per_launch": per_launch, "traffic": None},
        "clocks": clk.summary(), "gpu_launches": L * args.steps,
    }


def run_model_decode(args, world, rank, local):
    """BASELINE config 1 as a whole decode step: fla's RWKV-7 model (the model
    wkvm serves) at the 1.5B shape (L=24, D=2048, H=32, vocab 65536, random
    bf16 weights, std 0.02), 256 active slots of a 1024-slot arena. Two arms
    on the same box and weights:
      ours      - fla model with wkvm_b200's ops installed, WKV state read and
                  written in the arena by slot id (fla_compat.slot_cache);
      reference - wkvm's gather -> fla model with fla's Triton ops -> scatter
                  (per-layer index_select / index_copy_, as
                  wkvm/runner/state.py:63-97 does)."""
    from fla.models.rwkv7 import RWKV7Config, RWKV7ForCausalLM
    from fla.models.utils import Cache
    from wkvm_b200 import fla_compat, ops, synth
    from wkvm_b200.state import RWKV7StateBank, RWKV7StateLayout

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    torch.manual_seed(rank)
    cfg = RWKV7Config(hidden_size=H * N, num_hidden_layers=L, head_dim=N, vocab_size=65536)
    with torch.device(dev):
        model = RWKV7ForCausalLM(cfg)
    model = model.to(torch.bfloat16).eval().requires_grad_(False)
    layout = RWKV7StateLayout(n_layer=L, hidden_size=H * N, num_heads=H, head_dim=N,
                              head_v_dim=N, dtype=torch.bfloat16)
    bank = RWKV7StateBank(layout, NUM_SLOTS, device=dev)
    gen = torch.Generator(device=dev).manual_seed(99 + rank)
    bank.wkv.normal_(0.0, 0.1, generator=gen)
    bank.shift.normal_(0.0, 0.5, generator=gen)
    ids_host = synth.slot_ids(ACTIVE, NUM_SLOTS + 1, seed=rank).tolist()
    ids_dev = torch.tensor(ids_host, dtype=torch.int32, device=dev)
    ids_long = ids_dev.long()
    tokens = torch.randint(0, 65536, (ACTIVE, 1), device=dev, generator=gen)

    def ref_step():
        cache = Cache()
        for i in range(L):
            cache.update(recurrent_state=bank.wkv[i].index_select(0, ids_long),
                         conv_state=bank.shift[i, 0].index_select(0, ids_long),
                         ffn_state=bank.shift[i, 1].index_select(0, ids_long),
                         layer_idx=i, offset=0)
        out = model(input_ids=tokens, past_key_values=cache, use_cache=True, logits_to_keep=1)
        for i in range(L):
            st = cache[i]
            bank.wkv[i].index_copy_(0, ids_long, st["recurrent_state"].float())
            bank.shift[i, 0].index_copy_(0, ids_long, st["conv_state"])
            bank.shift[i, 1].index_copy_(0, ids_long, st["ffn_state"])
        return out.logits

    def our_step():
        h = fla_compat.slot_cache(bank, ids_dev)
        out = model(input_ids=tokens, past_key_values=h.cache, use_cache=True, logits_to_keep=1)
        h.commit()
        return out.logits

    def fused_step():  # with install(fuse_time_mix=True): token shift rows stay in the bank
        h = fla_compat.slot_cache(bank, ids_dev, shift_in_bank=True)
        out = model(input_ids=tokens, past_key_values=h.cache, use_cache=True, logits_to_keep=1)
        h.commit()
        return out.logits

    def timed(step):
        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize(dev)
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        for _ in range(args.steps):
            step()
        s1.record()
        torch.cuda.synchronize(dev)
        return s0.elapsed_time(s1) / args.steps

    with torch.inference_mode():
        # parity: one step of each arm from the same state
        w0, sh0 = bank.wkv.clone(), bank.shift.clone()
        fla_compat.uninstall()
        ref_logits = ref_step().float()
        ref_state = bank.wkv[:, ids_long].clone()
        bank.wkv.copy_(w0)
        bank.shift.copy_(sh0)
        fla_compat.install()
        our_logits = our_step().float()
        our_state = bank.wkv[:, ids_long].clone()
        parity = {
            "logits_max_rel": float((our_logits - ref_logits).abs().max() / ref_logits.abs().max()),
            "argmax_agree": float((our_logits.argmax(-1) == ref_logits.argmax(-1)).float().mean()),
            "state_max_rel": float((our_state - ref_state).abs().max() / ref_state.abs().max()),
        }
        bank.wkv.copy_(w0)
        bank.shift.copy_(sh0)
        fla_compat.install(fuse_time_mix=True)
        fused_logits = fused_step().float()
        fused_state = bank.wkv[:, ids_long].clone()
        fla_compat.install(fuse_time_mix=False)
        parity_fused = {
            "logits_max_rel": float((fused_logits - ref_logits).abs().max()
                                    / ref_logits.abs().max()),
            "argmax_agree": float((fused_logits.argmax(-1) == ref_logits.argmax(-1))
                                  .float().mean()),
            "state_max_rel": float((fused_state - ref_state).abs().max()
                                   / ref_state.abs().max()),
            "note": "fla rounds every time-mix intermediate to bf16; the fused core keeps fp32",
        }
        bank.wkv.copy_(w0)
        bank.shift.copy_(sh0)
        del w0, sh0

        def graphed(step):
            """Whole decode step captured once as a CUDA graph, then replayed
            (the reference's engine bench graphs its decode step too)."""
            s = torch.cuda.Stream(dev)
            s.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(s):
                for _ in range(2):
                    step()
            torch.cuda.current_stream(dev).wait_stream(s)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                step()
            return g.replay

        ops_only_ms = timed(graphed(our_step))
        ops_only_eager_ms = timed(our_step)
        # the headline arm: time-mix core fused around the WKV step and the
        # token shift + lerp prologues on the bank's shift rows
        fla_compat.install(fuse_time_mix=True)
        # The kernel ahead of each time-mix core is a projection GEMM, which
        # writes neither the arena nor the slot ids: the overlap mode's
        # contract holds, so the core's launch overlaps that GEMM's tail.
        prev_overlap = ops.set_decode_overlap(not args.no_overlap)
        clk_ctx = Clocks(dev.index if dev.index is not None else 0)
        with clk_ctx as clk:
            ours_ms = timed(graphed(fused_step))
        ours_eager_ms = timed(fused_step)
        ops.set_decode_overlap(prev_overlap)
        core_only_ms = timed(graphed(our_step))
        fla_compat.install(fuse_time_mix=False)
        fla_compat.uninstall()
        ref_ms = timed(graphed(ref_step))
        ref_eager_ms = timed(ref_step)
    ops.check_device_status(dev)
    ours_ms = max_over_ranks(ours_ms, world, dev)
    ref_ms = max_over_ranks(ref_ms, world, dev)
    if rank != 0:
        return None
    return {
        "metric": "RWKV-7 1.5B-shape full decode step tokens/s (BASELINE config 1)",
        "value": round(world * ACTIVE / (ours_ms * 1e-3), 1), "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ours_ms, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16 weights and activations, fp32 WKV state",
        "data": "synthetic (random-init weights std 0.02, random tokens and states)",
        "config": {"workload": "fla RWKV7ForCausalLM L=24 D=2048 H=32 vocab 65536, 256 active "
                               "of 1024 arena slots, whole step as one CUDA graph, "
                               "logits_to_keep=1",
                   "global_batch": ACTIVE * world},
        "path": "fla model; fused time-mix decode core (gates, norms, WKV, GroupNorm, "
                "correction) and token-shift + lerp prologues on the arena rows"
                + ("" if args.no_overlap else "; time-mix core launched with programmatic "
                   "dependent launch"),
        "eager_ms_per_step": round(ours_eager_ms, 4),
        "ops_only": {"ms_per_step": round(ops_only_ms, 4),
                     "eager_ms_per_step": round(ops_only_eager_ms, 4),
                     "note": "fla forward unchanged, only the WKV ops swapped (slot-resident "
                             "state, shift rows gathered and restored)"},
        "core_only": {"ms_per_step": round(core_only_ms, 4),
                      "note": "fused time-mix core, fla's token shift + addcmul"},
        "same_box_reference": {"ms_per_step": round(ref_ms, 4),
                               "value": round(world * ACTIVE / (ref_ms * 1e-3), 1),
                               "eager_ms_per_step": round(ref_eager_ms, 4),
                               "path": "gather -> fla Triton ops -> scatter (wkvm's runner flow)"},
        "parity_one_step": {"ops_only": parity, "fused": parity_fused},
        "clocks": clk.summary(),
    }


def _cpu_sample(slots: int, threads: int, seed: int = 0):
    """One decode token through all 24 layers for ``slots`` slots with the
    fp32 oracle; returns seconds."""
    from oracle import oracle
    from wkvm_b200 import synth
    import numpy as np
    xs = []
    for layer in range(L):
        x = synth.rwkv7_inputs(slots, 1, H, N, seed=seed * 1000 + layer)
        xs.append([x[n].float().numpy() for n in ("r", "w", "k", "v", "kk", "a")] +
                  [x["h0"].numpy()])
    t0 = time.perf_counter()
    for r, w, k, v, kk, a, h0 in xs:
        oracle.rwkv7_recurrence(r, w, k, v, kk, a, initial_state=h0, threads=threads)
    return time.perf_counter() - t0


def torch_reference_cfg0(steps: int = 16, seed: int = 0) -> dict:
    """BASELINE config 0 (B=8 slots, L=12, H=12, N=64) through the reference's
    own PyTorch CPU recurrence, fla's dplr_recurrence
    (fla/ops/generalized_delta_rule/dplr/naive.py:16), fp32, on the host's
    cores: `steps` tokens per layer for every layer. fla forces a q * K^-0.5
    scale there; r is pre-multiplied by sqrt(K) so the work and the result are
    RWKV-7's scale-1 step."""
    try:
        from fla.ops.generalized_delta_rule.dplr.naive import dplr_recurrence
    except Exception as e:  # fla missing on this host
        return {"unavailable": f"{type(e).__name__}: {str(e)[:120]}"}
    from wkvm_b200 import synth
    B0, L0, H0, N0 = 8, 12, 12, 64
    hf = lambda t: t.float().transpose(1, 2).contiguous()  # [B, H, T, D]
    layers = []
    for layer in range(L0):
        x = synth.rwkv7_inputs(B0, steps, H0, N0, seed=seed * 100 + layer)
        layers.append((hf(x["r"]) * N0 ** 0.5, hf(x["k"]), hf(x["v"]), -hf(x["kk"]),
                       hf(x["kk"]) * hf(x["a"]), hf(x["w"]), x["h0"]))
    t0 = time.perf_counter()
    with torch.no_grad():
        for q, k, v, al, be, w, h0 in layers:
            dplr_recurrence(q, k, v, al, be, w, initial_state=h0.clone(), output_final_state=True)
    sec = time.perf_counter() - t0
    return {"value": round(B0 * steps / sec, 2), "unit": "tokens/s",
            "cores": torch.get_num_threads(), "kind": "reference",
            "sample": f"BASELINE config 0: {B0} slots x {L0} layers x {H0} heads, {steps} tokens, "
                      "fla's dplr_recurrence (torch, fp32, CPU)"}


def cpu_baseline(slots: int):
    threads = os.cpu_count() or 1
    reps, total = 0, 0.0
    while total < 10.0 and reps < 50:
        total += _cpu_sample(slots, threads, seed=reps)
        reps += 1
    return {"value": round(reps * slots / total, 2), "unit": "tokens/s", "cores": threads,
            "kind": "port",
            "sample": f"{reps} x ({slots} slots x 24 layers x 32 heads, one token) through the "
                      f"fp32 C oracle (oracle/wkv_oracle.c), {threads} threads"}


def run_reference(args, world, rank):
    if rank != 0:
        return None
    threads = os.cpu_count() or 1
    slots = args.cpu_sample_slots
    for i in range(args.warmup):
        _cpu_sample(slots, threads, seed=i)
    times = [_cpu_sample(slots, threads, seed=100 + i) for i in range(args.steps)]
    total = sum(times)
    value = round(slots * args.steps / total, 2)
    return {
        "metric": METRIC, "impl": "reference", "value": value, "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * total / args.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded, reference op-level distributions)",
        "config": {"workload": "RWKV-7 1.5B-shape WKV slot decode: L=24 H=32 N=64; each step a "
                               f"bounded sample of {slots} of the 256 active slots",
                   "global_batch": slots, "parallelism": "host threads"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": f"{slots} slots x 24 layers x 32 heads per step, fp32 C "
                                   "restatement of fla's recurrence (oracle/wkv_oracle.c)",
                         "reference_torch_cfg0": torch_reference_cfg0()},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def side_workloads(args, world, rank, local):
    """BASELINE configs 2 and 3 timed in the same run as the headline decode
    line (1 GPU): RWKV-7 chunked prefill, GDN decode and GDN chunked prefill,
    each with its own CUDA-event timing, roofline and clock record."""
    import copy
    out = {}
    for name, wl, fn in (("cfg2_wkv7_prefill", "prefill", run_prefill),
                         ("cfg3_gdn_decode", "gdn-decode", run_gdn),
                         ("cfg3_gdn_prefill", "gdn-prefill", run_gdn)):
        a = copy.copy(args)
        a.workload = wl
        r = fn(a, world, rank, local)
        torch.cuda.empty_cache()
        out[name] = {k: r[k] for k in ("metric", "value", "unit", "ms_per_step", "steps",
                                       "warmup", "config", "roofline", "clocks",
                                       "gpu_launches", "same_box_fla")}
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-sample-slots", type=int, default=16)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-migration", action="store_true",
                    help="N > 1: leave out the ring migration of parked sessions")
    ap.add_argument("--no-fla", action="store_true",
                    help="skip the same-box fla Triton timing of the prefill / GDN workloads")
    ap.add_argument("--no-workloads", action="store_true",
                    help="skip the config 2 / 3 lines the default 1-GPU run adds")
    ap.add_argument("--no-overlap", action="store_true",
                    help="plain launches instead of programmatic dependent launch")
    ap.add_argument("--layers", type=int, default=24,
                    help="layers per decode step (24 = the benchmark; fewer for profiling)")
    ap.add_argument("--workload", default="decode",
                    choices=["decode", "prefill", "gdn-decode", "gdn-prefill", "model-decode",
                             "cfg4", "hibernate", "timemix"])
    ap.add_argument("--prefill-batch", type=int, default=16)
    ap.add_argument("--gdn-batch", type=int, default=4,
                    help="sequences of the gdn-prefill workload (config 3: 4)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    global L
    L = args.layers
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        line = run_reference(args, world, rank)
    else:
        world, rank, local = dist_setup()
        if args.workload == "prefill":
            line = run_prefill(args, world, rank, local)
        elif args.workload == "model-decode":
            line = run_model_decode(args, world, rank, local)
        elif args.workload.startswith("gdn"):
            line = run_gdn(args, world, rank, local)
        elif args.workload == "cfg4":
            line = run_cfg4(args, world, rank, local)
        elif args.workload == "hibernate":
            line = run_hibernate(args, world, rank, local)
        elif args.workload == "timemix":
            line = run_timemix(args, world, rank, local)
        else:
            line = run_ours(args, world, rank, local)
            if world == 1 and not args.no_workloads:
                line["workloads"] = side_workloads(args, world, rank, local)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
    if line is not None:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
