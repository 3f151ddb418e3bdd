#!/usr/bin/env python
"""Benchmark: ms per 48-block Pairformer trunk pass at N = 512, master precision, on B200.

Workload (benchmark configuration 2): 48 AF3 Pairformer blocks (c_z 128, c_s 384), N = 512
tokens, the last 26 padded, z and s ~ N(0, 1), weights ~ N(0, 0.02) with LayerNorm gamma 1 /
beta 0, blocks drawn in order from one seed-0 generator; fp32 master weights, bf16
activations. One step = one trunk pass over one input.

* ``value``: device time of the trunk (CUDA events on the launching stream, graph-replayed,
  inputs resident in HBM, L2 flushed before every step), max over ranks.
* ``e2e``: the same pass through the public API from pinned HOST buffers: host->device copy
  of z and s, the trunk, device->host copy of the updated pair and single, all timed.
* ``roofline``: the dominant kernel (triangle attention core) timed alone on the same data.
* ``cpu_baseline``: the CPU oracle (a restatement of the reference's block) on this host's
  cores, one block at N = 512, times 48.

``--gpus N`` (torchrun, one rank per GPU, N > 1): the pair is ROW-SHARDED across the ranks
(axial parallelism, ``foldforge_b200/engine/sharded.py``: pair transposes between the row-wise
and column-wise triangle ops and row gathers of the TriMul right operand and the attention
biases, each written by one kernel straight into the peers' buffers over NVLink (CUDA IPC
peer memory, bounded waits); the single track replicated). ``value`` is ms per 48-block trunk pass of
the whole job (max over ranks) at N = 512 P^(1/3) rounded to a multiple of 8 P tokens (640,
800, 1024 on 2, 4, 8 GPUs): per-GPU work held at the N = 512 trunk's, ``scaling`` weak, so
value(1) / value(P) is the weak-scaling efficiency. ``ladder`` reports the benchmark's
N = 2048 length-ladder trunk (configuration 3, 5% padded suffix) on the same GPUs (strong
scaling; the N = 1 line carries the single-GPU figure).

``--impl reference``: the reference's algorithm (CPU oracle) on this host, same metric.
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
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "ms per 48-block Pairformer trunk at N=512 bf16; N=2048 at 1/2/4/8 B200"
N_TOKENS = 512
N_BLOCKS = 48
MASKED = 26
#: DRAM traffic of one triangle-attention core launch at N = 512 (dram__bytes_read.sum +
#: dram__bytes_write.sum of one ncu capture of ``--kernels-once --n 512``: 203.7 + 46.6 MB).
ATTN_TRAFFIC_BYTES: float | None = 250.3e6


def parse() -> argparse.Namespace:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("b200", "reference"), default="b200")
    ap.add_argument("--n", type=int, default=N_TOKENS)
    ap.add_argument("--blocks", type=int, default=N_BLOCKS)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-ladder", action="store_true", help="skip the N=2048 length-ladder measurement")
    ap.add_argument("--no-msa", action="store_true", help="skip the MSA-module measurement (configuration 4)")
    ap.add_argument("--no-dit", action="store_true",
                    help="skip the diffusion-transformer measurement (configuration 5's token transformer)")
    ap.add_argument("--eager-sharded", action="store_true",
                    help="with --gpus > 1: time eager launches instead of a captured CUDA graph of the sharded trunk")
    ap.add_argument("--breakdown", action="store_true",
                    help="with --gpus > 1: per-stage CUDA-event times of the N=2048 sharded trunk (max over ranks)")
    ap.add_argument("--dit-once", action="store_true",
                    help="run one token DiT block three times at configuration 5's shape (a driver for ncu captures)")
    ap.add_argument("--kernels-once", action="store_true",
                    help="launch every pair-stack kernel once at --n (a driver for ncu captures; no timing)")
    return ap.parse_args()


def weak_n(gpus: int) -> int:
    """Tokens of the weak-scaling trunk on ``gpus`` ranks: 512 P^(1/3), a multiple of 8 P."""
    unit = 8 * gpus
    return max(unit, round(N_TOKENS * gpus ** (1.0 / 3.0) / unit) * unit)


LADDER_N = 2048
LADDER_WARMUP, LADDER_STEPS = 3, 3  # the ladder trunk: untimed passes, then timed ones (L2 flushed before each)
SUB_WARMUP = 3  # untimed graph replays before the MSA-module and token-transformer lines


def peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        d = json.loads(path.read_text())
        return {"hbm": d["hbm_gbs"], "bf16": d["bf16_tflops"], "bf16_sustained": d["bf16_tflops_sustained"],
                "source": "measured"}
    return {"hbm": 6650.0, "bf16": 1590.0, "bf16_sustained": 1400.0, "source": "fallback"}


def block_flops(n: int) -> float:
    return 1536.0 * n**3 + 1_121_792.0 * n**2 + 5.0e6 * n


# ------------------------------------------------------------------------------ clocks
class ClockSampler:
    """``nvidia-smi`` samples every 200 ms while active (SM clock, reasons)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int) -> None:
        self.index = index
        self.lines: list[str] = []
        self.proc = None

    def start(self) -> None:
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.index)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        threading.Thread(target=self._read, daemon=True).start()

    def _read(self) -> None:
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        sm, smax, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax), "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------------------ distributed
def dist_setup(gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
        return rank, world, local, dist
    if gpus != 1:
        print(f"--gpus {gpus} needs torchrun (one process per GPU)", file=sys.stderr)
    return 0, 1, local, None


def max_over_ranks(value: float, dist) -> float:
    if dist is None:
        return value
    t = torch.tensor([value], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------------------------ CPU baseline
def cpu_block_ms(n: int, warm: bool = False) -> tuple[float, int]:
    """One block of the oracle (fp32, all host cores) at ``n`` tokens; returns (ms, threads)."""
    import oracle
    from foldforge_b200.synthetic import block_state, inputs

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    state = block_state(torch.Generator().manual_seed(0), scheme="baseline")
    z, s, tokens = inputs(n, 0, masked_suffix=round(MASKED * n / N_TOKENS))
    if warm:
        oracle.pairformer_block(z[:64, :64].contiguous(), s[:64], tokens[:64], state)
    t0 = time.perf_counter()
    with torch.no_grad():
        oracle.pairformer_block(z, s, tokens, state)
    return (time.perf_counter() - t0) * 1e3, threads


def run_reference(args, rank: int, world: int) -> None:
    """The reference arm: the CPU oracle (the reference block's equations, fp32, all host
    threads) on rank 0. One step = ONE block at the workload's N (the same N as the b200 arm
    at this GPU count); ``value`` extrapolates the median block to the 48-block trunk, and
    ``ms_per_step`` is the measured one-block time, so ``ms_per_step x steps`` is the wall
    time of the timed steps. Steps stop early once 150 s of CPU time have been timed."""
    if rank != 0:
        return
    n = args.n if world == 1 else weak_n(world)
    times = []
    threads = os.cpu_count() or 1
    budget_s, spent = 150.0, 0.0
    for i in range(1 + args.steps):
        ms, threads = cpu_block_ms(n, warm=(i == 0))
        if i == 0:
            continue  # the warm-up step
        times.append(ms)
        spent += ms / 1e3
        if spent > budget_s:
            break
    block_ms = statistics.median(times)
    value = block_ms * args.blocks
    masked = round(MASKED * n / N_TOKENS)
    sample = (f"one block of the {args.blocks}-block trunk at N={n} per step (fp32 CPU oracle, {threads} threads), "
              f"median of {len(times)} steps; value = median x {args.blocks} blocks (extrapolated)")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "ms", "n_gpus": world,
        "steps": len(times), "steps_requested": args.steps, "warmup": 1, "ms_per_step": round(block_ms, 3),
        "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"{args.blocks}-block Pairformer trunk, N={n}, last {masked} tokens masked",
                   "model": "AF3 Pairformer block (c_z 128, c_s 384)", "global_batch": 1, "seq_len": n,
                   "parallelism": "cpu", "step": "one block (value extrapolated to the trunk)"},
        "cpu_baseline": {"value": round(value, 3), "unit": "ms", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 3), "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------ the b200 arm
def run_b200(args, rank: int, world: int, local: int, dist) -> None:
    import foldforge_b200
    from foldforge_b200 import _lib, kernels
    from foldforge_b200.engine.capture import GraphedCall
    from foldforge_b200.synthetic import inputs, trunk_state

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    n, nb = args.n, args.blocks
    states = trunk_state(nb, seed=0, scheme="baseline")
    trunk = foldforge_b200.load(states, backend="b200", unsupported="error", dtype=torch.bfloat16, device=dev)
    z, s, tokens = inputs(n, seed=rank, masked_suffix=round(MASKED * n / N_TOKENS))
    mask = (tokens > 0)[None].to(dev)

    def step(zz: torch.Tensor, ss: torch.Tensor):
        return trunk(zz, mask, ss)

    z_dev = z.bfloat16()[None].to(dev)
    s_dev = s.bfloat16()[None].to(dev)
    _lib.launch_count = 0
    graphed = GraphedCall(step, [z_dev, s_dev], warmup=1)
    # launches recorded during the warm-up call and the capture: two passes
    launches = _lib.launch_count // 2
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)

    for _ in range(max(args.warmup, 3)):
        flush.fill_(1.0)
        graphed.replay()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()

    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    for start, end in events:
        flush.fill_(1.0)  # 256 MB write: L2 (126 MB) holds nothing of the previous step
        start.record()
        graphed.replay()
        end.record()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    clocks = sampler.stop()
    times = [a.elapsed_time(b) for a, b in events]
    local_ms = sum(times) / len(times)
    trunk_ms = max_over_ranks(local_ms, dist)
    value = trunk_ms / world
    err = _lib.device_error()
    if err:
        raise RuntimeError(f"device error word {err} after the timed region")

    # ---------------------------------------------------------------- dominant kernel alone
    block0 = trunk.blocks[0]
    zz = graphed.static_inputs[0]
    ta = block0.tri_atten_starting
    packed = ta._packed[1]
    ws = torch.empty(int(_lib.load().ffb_triattn_workspace_bytes(1, n)), dtype=torch.uint8, device=dev)
    out = torch.empty_like(zz)
    kernels.triattn(zz, mask, packed, starting=True, stages=1, workspace=ws, out=out)
    reps = 20
    for _ in range(3):
        kernels.triattn(zz, mask, packed, starting=True, stages=2, workspace=ws, out=out)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    a.record()
    for _ in range(reps):
        kernels.triattn(zz, mask, packed, starting=True, stages=2, workspace=ws, out=out)
    b.record()
    torch.cuda.synchronize()
    attn_ms = a.elapsed_time(b) / reps
    attn_flops = 4.0 * n**3 * 128  # Q K^T + P V, multiply-add = 2
    pk = peaks()
    achieved = attn_flops / (attn_ms * 1e-3) / 1e12

    # ---------------------------------------------------------------- end to end from host buffers
    e2e = None
    if not args.no_e2e:
        z_host = z.bfloat16()[None].pin_memory()
        s_host = s.bfloat16()[None].pin_memory()
        pair_host = torch.empty_like(z_host).pin_memory()
        single_host = torch.empty_like(s_host).pin_memory()
        stream = torch.cuda.current_stream()
        e_events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                    for _ in range(args.steps)]
        for start, end in e_events:
            flush.fill_(1.0)
            start.record(stream)
            pair_out, single_out = graphed(z_host, s_host)  # host -> static device inputs, then replay
            pair_host.copy_(pair_out, non_blocking=True)
            single_host.copy_(single_out, non_blocking=True)
            end.record(stream)
        torch.cuda.synchronize()
        e_ms = max_over_ranks(sum(x.elapsed_time(y) for x, y in e_events) / len(e_events), dist)
        e2e = {"value": round(e_ms / world, 3), "unit": "ms",
               "h2d_bytes_per_step": z_host.numel() * 2 + s_host.numel() * 2,
               "d2h_bytes_per_step": pair_host.numel() * 2 + single_host.numel() * 2}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        ms, threads = cpu_block_ms(n, warm=True)
        cpu = {"value": round(ms * nb, 1), "unit": "ms", "cores": threads, "kind": "port",
               "sample": f"one block at N={n} (fp32 CPU oracle, all host threads), x{nb} blocks"}

    if rank == 0:
        trunk_flops = block_flops(n) * nb
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": "ms", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(trunk_ms, 3), "higher_is_better": False,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {
                "workload": f"{nb}-block Pairformer trunk, N={n}, last {round(MASKED * n / N_TOKENS)} tokens masked, "
                            "master precision (fp32 weights, bf16 activations), CUDA-graph replay",
                "model": "AF3 Pairformer block (c_z 128, c_s 384, 4x32 / 16x24 heads)",
                "global_batch": world, "seq_len": n, "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                "l2": "flushed by a 256 MB write before every timed step",
                "trunk_tflops": round(trunk_flops / (trunk_ms * 1e-3) / 1e12, 1),
                "ms_per_block": round(trunk_ms / nb, 4),
            },
            "roofline": {
                "kernel": "triattn_attn_kernel (starting node, N=512)",
                "bound": "tensor", "achieved": round(achieved, 1), "peak": pk["bf16"], "unit": "TFLOP/s",
                "frac": round(achieved / pk["bf16"], 4), "traffic": ATTN_TRAFFIC_BYTES,
                "launch_ms": round(attn_ms, 4), "peak_source": f"{pk['source']} (burst: kernel timed alone)",
                "algorithmic": f"4 * N^3 * 128 = {attn_flops:.3e} flop per launch",
            },
            "clocks": clocks,
            "gpu_launches": launches * args.steps,
        }
        if e2e is not None:
            line["e2e"] = e2e
        if cpu is not None:
            line["cpu_baseline"] = cpu
        if world == 1 and not args.no_ladder:
            del graphed, trunk
            torch.cuda.empty_cache()
            line["ladder"] = ladder_single_gpu(dev)
        if world == 1 and not args.no_msa:
            torch.cuda.empty_cache()
            line["msa_module"] = msa_module_single_gpu(dev)
        if world == 1 and not args.no_dit:
            line["token_dit"] = token_dit_single_gpu(dev)
        print(json.dumps(line), flush=True)


def ladder_single_gpu(dev: torch.device) -> dict:
    """The N = 2048 length-ladder trunk on one GPU (CUDA-graph replay): 3 warm-up replays, 3 timed."""
    import math

    import foldforge_b200
    from foldforge_b200.engine.capture import GraphedCall
    from foldforge_b200.synthetic import inputs, trunk_state

    n = LADDER_N
    masked = math.ceil(0.05 * n)
    trunk = foldforge_b200.load(trunk_state(N_BLOCKS, seed=0, scheme="baseline"), backend="b200",
                                unsupported="error", dtype=torch.bfloat16, device=dev)
    z, s, tokens = inputs(n, seed=0, masked_suffix=masked)
    mask = (tokens > 0)[None].to(dev)
    graphed = GraphedCall(lambda zz, ss: trunk(zz, mask, ss), [z.bfloat16()[None].to(dev), s.bfloat16()[None].to(dev)],
                          warmup=1)
    del z
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    for _ in range(LADDER_WARMUP):
        graphed.replay()
    torch.cuda.synchronize()
    sampler = ClockSampler(dev.index or 0)
    sampler.start()
    time.sleep(0.3)
    ts = []
    for _ in range(LADDER_STEPS):
        flush.fill_(1.0)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        graphed.replay()
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b))
    clocks = sampler.stop()
    del graphed, trunk
    torch.cuda.empty_cache()
    ms = sum(ts) / len(ts)
    return {"n": n, "n_gpus": 1, "ms_per_trunk": round(ms, 1), "ms_per_block": round(ms / N_BLOCKS, 3),
            "masked_suffix": masked, "steps": LADDER_STEPS, "warmup": LADDER_WARMUP,
            "parallelism": "single GPU (CUDA-graph replay)",
            "clocks": clocks}


def msa_inputs_config4(dev: torch.device, n_seq: int = 1024, n: int = 512, seed: int = 0):
    """Benchmark configuration 4's MSA features: residue ids uniform in 0..31 (one-hot), has_deletion
    Bernoulli(0.1), deletion_value uniform [0, 1], embedded to c_m = 64 by a N(0, 0.02) linear map;
    the pair ~N(0, 1); every MSA position and token real."""
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, 32, (n_seq, n), generator=g)
    feats = torch.cat([torch.nn.functional.one_hot(ids, 32).float(),
                       (torch.rand(n_seq, n, 1, generator=g) < 0.1).float(),
                       torch.rand(n_seq, n, 1, generator=g)], dim=-1)  # [S, N, 34]
    w = 0.02 * torch.randn(64, 34, generator=g)
    msa = (feats @ w.t()).bfloat16()
    z = torch.randn(n, n, 128, generator=g).bfloat16()
    return msa[None].to(dev), z[None].to(dev), torch.ones(1, n_seq, n, device=dev), torch.ones(1, n, n, device=dev)


def token_dit_single_gpu(dev: torch.device, n_blocks: int = 24, samples: int = 5, n: int = 512) -> dict:
    """BASELINE configuration 5's token diffusion transformer: 24 AF3 TokenDiT blocks (c 768, 16
    heads, conditioning 384, pair 128) over 5 samples x N = 512 tokens, conditioned on fixed random
    trunk outputs (s, z ~ N(0, 1)), b200 backend. A sampler step (one pass of the stack) is timed
    as a CUDA-graph replay with the L2 flushed, 3 warm-up replays and 3 timed steps; the once-per-fold
    conditioning tables (AdaLN, gates, pair logits of every block) are timed separately. The
    atom encoder / decoder and the EDM update around the transformer are not part of this."""
    from foldforge_b200.engine import backends, policy
    from foldforge_b200.engine.capture import GraphedCall
    from foldforge_b200.engine.dit import TokenDiT, TokenDiTStack
    from foldforge_b200.synthetic import dit_inputs, dit_stack_state

    blocks = []
    for st in dit_stack_state(n_blocks, 0, "baseline"):
        blk = TokenDiT()
        blk.load_state_dict(st, strict=True)
        blocks.append(blk)
    stack = TokenDiTStack(blocks).to(dev).eval()
    plan = backends.BackendPlan.make("b200", unsupported="error").resolve(dev)
    policy.apply_plan(stack, plan, dev)
    x, cond, pair, mask = dit_inputs(samples, n, 0)
    x, cond, pair = x.bfloat16().to(dev), cond.bfloat16().to(dev), pair.bfloat16().to(dev)
    mask = mask.to(dev) > 0
    key_mask = mask[None]
    with torch.no_grad():
        stack(x, mask, cond, pair, key_mask=key_mask)  # weights packed, tables built
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for blk in stack.blocks:
        blk.release_fold()
        blk._conditioning(cond, pair, blk._pack(dev))
    b.record()
    torch.cuda.synchronize()
    cond_ms = a.elapsed_time(b)
    graphed = GraphedCall(lambda xx: stack(xx, mask, cond, pair, key_mask=key_mask), [x], warmup=1)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    for _ in range(SUB_WARMUP):
        graphed.replay()
    torch.cuda.synchronize()
    ts = []
    for _ in range(3):
        flush.fill_(1.0)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        graphed.replay()
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b))
    del graphed, stack
    torch.cuda.empty_cache()
    ms = sum(ts) / len(ts)
    m = samples * n
    per_block = 2.0 * m * 768 * (4 * 768 + 768 + 2 * 1536 + 1536) + 4.0 * samples * 16 * n * n * 48
    return {"config": "BASELINE configuration 5, token transformer: 24 TokenDiT blocks (768, 16 heads), "
                      f"{samples} samples x N={n}, bf16, conditioned on fixed s [512, 384], z [512, 512, 128]",
            "ms_per_sampler_step": round(ms, 3), "ms_per_block": round(ms / n_blocks, 4),
            "ms_per_200_steps": round(200 * ms, 1), "ms_conditioning_per_fold": round(cond_ms, 3),
            "steps": 3, "warmup": SUB_WARMUP, "tflops_approx": round(n_blocks * per_block / (ms * 1e-3) / 1e12, 1),
            "parallelism": "single GPU (CUDA-graph replay)"}


def msa_module_single_gpu(dev: torch.device, n_blocks: int = 4) -> dict:
    """the MSA module's 4 AF3 MSA-stack blocks at 1024 MSA rows x N = 512
    on one GPU (b200 backend, CUDA-graph replay, L2 flushed), 3 warm-up replays and 3 timed passes."""
    from foldforge_b200.engine import backends, policy
    from foldforge_b200.engine.capture import GraphedCall
    from foldforge_b200.engine.evoformer import EvoformerBlock
    from foldforge_b200.synthetic import evoformer_state

    g = torch.Generator().manual_seed(0)
    blocks = torch.nn.ModuleList()
    for _ in range(n_blocks):
        blk = EvoformerBlock(masked_update="zero")
        blk.load_state_dict(evoformer_state(g, scheme="baseline"), strict=True)
        blocks.append(blk)
    blocks = blocks.to(dev).eval()
    plan = backends.BackendPlan.make("b200", unsupported="error").resolve(dev)
    policy.apply_plan(blocks, plan, dev)
    msa, z, msa_mask, pair_mask = msa_inputs_config4(dev)

    def module(m, zz):
        for blk in blocks:
            m, zz = blk.batched(m, zz, msa_mask, pair_mask)
        return m, zz

    graphed = GraphedCall(module, [msa, z], warmup=1)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    for _ in range(SUB_WARMUP):
        graphed.replay()
    torch.cuda.synchronize()
    ts = []
    for _ in range(3):
        flush.fill_(1.0)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        graphed.replay()
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b))
    del graphed, blocks
    torch.cuda.empty_cache()
    ms = sum(ts) / len(ts)
    # outer product mean contraction + projection, averaging, projections; the pair track
    n, s = 512, 1024
    opm = 2.0 * (n * 32) ** 2 * s + 2.0 * n * n * 1024 * 128
    pwa = 2.0 * 8 * n * n * s * 8 + 2.0 * s * n * 64 * (128 + 64)
    tr = 2.0 * s * n * 64 * 256 * 3
    pair = 1536.0 * n**3 + 1_121_792.0 * n**2 - 2.0 * n * n * 128 * 16  # the Pairformer pair track
    flops = n_blocks * (opm + pwa + tr + pair)
    return {"config": "BASELINE configuration 4: 4 MSA-stack blocks, 1024 MSA rows x N=512, c_m 64, c_z 128, bf16",
            "ms_per_module": round(ms, 2), "ms_per_block": round(ms / n_blocks, 3), "steps": 3, "warmup": SUB_WARMUP,
            "tflops_approx": round(flops / (ms * 1e-3) / 1e12, 1), "parallelism": "single GPU (CUDA-graph replay)"}


def stage_breakdown(comm, run_trunk, data, nb: int, dist, dev) -> dict:
    """Per-stage times of one pass of the sharded trunk at the ladder length: CUDA events at
    every stage boundary of every block (``ShardComm.timer``), summed per stage name over
    the blocks, divided by the block count, max over ranks per stage."""
    import math

    from foldforge_b200.engine.sharded import StageTimer

    rows_h, s_h, mask = data(LADDER_N, math.ceil(0.05 * LADDER_N))
    rows, s = rows_h.to(dev), s_h.to(dev)
    run_trunk(rows, mask, s)
    torch.cuda.synchronize()
    dist.barrier()
    comm.timer = StageTimer()
    comm.mark("start")
    run_trunk(rows, mask, s)
    torch.cuda.synchronize()
    per = comm.timer.durations()
    comm.timer = None
    names = list(per)
    t = torch.tensor([per[k] / nb for k in names], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    stages = {k: round(float(v), 4) for k, v in zip(names, t.tolist())}
    return {"n": LADDER_N, "n_gpus": comm.world, "ms_per_block": stages,
            "sum_of_stage_maxima_ms": round(sum(stages.values()), 3),
            "note": "CUDA events at stage boundaries, eager launches; each stage's max over ranks"}


def run_sharded(args, rank: int, world: int, local: int, dist) -> None:
    """Row-sharded trunk over the ranks: weak-scaling ``value`` and the N = 2048 ladder."""
    import math

    import foldforge_b200
    from foldforge_b200 import _lib, kernels
    from foldforge_b200.engine.sharded import ShardComm, ShardedPairformerBlock
    from foldforge_b200.synthetic import inputs, trunk_state

    dev = torch.device("cuda", local)
    nb = args.blocks
    trunk = foldforge_b200.load(trunk_state(nb, seed=0, scheme="baseline"), backend="b200", unsupported="error",
                                dtype=torch.bfloat16, device=dev)
    comm = ShardComm()
    blocks = [ShardedPairformerBlock(b, comm, ops="b200", masked_zero=True) for b in trunk.blocks]
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)

    def run_trunk(z_rows, mask, s):
        for blk in blocks:
            z_rows, s = blk(z_rows, mask, s)
        return z_rows, s

    def data(n: int, masked: int):
        z, s, tokens = inputs(n, seed=0, masked_suffix=masked)
        r, row0 = comm.rows(n)
        rows = z[row0:row0 + r].bfloat16().contiguous()
        return rows, s.bfloat16(), (tokens > 0).to(dev)

    graph_note: dict = {}

    def runner(rows, mask, s):
        """The trunk as a CUDA graph (captured on every rank after an eager warm-up pass that
        also creates the exchange buffers; the exchanges count their epochs on the device, so
        replays synchronise like eager passes), or eager launches."""
        graph_note.clear()
        graph_note["captured"] = False
        if args.eager_sharded:
            return lambda: run_trunk(rows, mask, s)
        from foldforge_b200.engine.capture import GraphedCall

        _lib.launch_count = 0
        try:
            graphed = GraphedCall(lambda r, ss: run_trunk(r, mask, ss), [rows, s], warmup=1)
        except RuntimeError as exc:  # noqa: PERF203 - fall back to eager launches
            graph_note["error"] = str(exc).splitlines()[0][:160]
            torch.cuda.synchronize()
            return lambda: run_trunk(rows, mask, s)
        graph_note["captured"] = True
        # the library's launches of one pass (the warm-up call and the capture made two)
        graph_note["launches_per_pass"] = _lib.launch_count // 2
        return graphed.replay

    def measure(n: int, masked: int, steps: int, warmup: int, clocks: bool = False):
        rows_h, s_h, mask = data(n, masked)
        rows, s = rows_h.to(dev), s_h.to(dev)
        for _ in range(warmup):
            run_trunk(rows, mask, s)
        torch.cuda.synchronize()
        dist.barrier()
        step = runner(rows, mask, s)
        step()  # one untimed pass of what is timed (the captured graph, if capture succeeded)
        torch.cuda.synchronize()
        dist.barrier()
        sampler = ClockSampler(local) if clocks else None
        if sampler:
            sampler.start()
            time.sleep(0.3)
        _lib.launch_count = 0
        ts = []
        for _ in range(steps):
            flush.fill_(1.0)
            torch.cuda.synchronize()
            dist.barrier()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            step()
            b.record()
            torch.cuda.synchronize()
            ts.append(a.elapsed_time(b))
        launches = _lib.launch_count if not graph_note["captured"] else graph_note["launches_per_pass"] * steps
        dist.barrier()
        clk = sampler.stop() if sampler else None
        ms = max_over_ranks(sum(ts) / len(ts), dist)
        mode = "CUDA-graph replay" if graph_note["captured"] else "eager launches" + (
            f"; capture failed: {graph_note['error']}" if "error" in graph_note else "")
        return ms, clk, launches, (rows_h, s_h, mask), mode

    n_w = weak_n(world)
    masked_w = round(MASKED * n_w / N_TOKENS)
    value_ms, clocks, launches, (rows_h, s_h, mask), mode = measure(n_w, masked_w, args.steps, max(args.warmup, 3),
                                                                     True)
    err = _lib.device_error()
    if err:
        raise RuntimeError(f"device error word {err} after the timed region")

    e2e = None
    if not args.no_e2e:
        rows_pin, s_pin = rows_h.pin_memory(), s_h.pin_memory()
        out_pin, s_out_pin = torch.empty_like(rows_pin).pin_memory(), torch.empty_like(s_pin).pin_memory()
        ts = []
        for _ in range(max(1, min(args.steps, 3))):
            flush.fill_(1.0)
            torch.cuda.synchronize()
            dist.barrier()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            zo, so = run_trunk(rows_pin.to(dev, non_blocking=True), mask, s_pin.to(dev, non_blocking=True))
            out_pin.copy_(zo, non_blocking=True)
            s_out_pin.copy_(so, non_blocking=True)
            b.record()
            torch.cuda.synchronize()
            ts.append(a.elapsed_time(b))
        e2e = {"value": round(max_over_ranks(sum(ts) / len(ts), dist), 3), "unit": "ms",
               "h2d_bytes_per_step": rows_pin.numel() * 2 + s_pin.numel() * 2,
               "d2h_bytes_per_step": out_pin.numel() * 2 + s_out_pin.numel() * 2,
               "per": "rank (its pair rows and the replicated single), max over ranks"}

    parity = sharded_parity(trunk, blocks, comm, rows_h, s_h, mask, n_w, rank, dev, dist)

    ladder = None
    if not args.no_ladder:
        lad_ms, lad_clocks, _, _, lad_mode = measure(LADDER_N, math.ceil(0.05 * LADDER_N), LADDER_STEPS,
                                                     LADDER_WARMUP, True)
        ladder = {"n": LADDER_N, "n_gpus": world, "ms_per_trunk": round(lad_ms, 1),
                  "ms_per_block": round(lad_ms / nb, 3), "masked_suffix": math.ceil(0.05 * LADDER_N),
                  "steps": LADDER_STEPS, "warmup": LADDER_WARMUP,
                  "parallelism": f"axial row-sharding x{world} ({lad_mode})", "clocks": lad_clocks}

    breakdown = None
    if args.breakdown:
        breakdown = stage_breakdown(comm, run_trunk, data, nb, dist, dev)

    # dominant kernel alone (triangle-attention core at N = 512 on this GPU)
    n = N_TOKENS
    zz, _, tok = inputs(n, seed=0, masked_suffix=MASKED)
    zz = zz.bfloat16()[None].to(dev)
    m512 = (tok > 0)[None].to(dev)
    packed = kernels.triattn_prepare({k[len("tri_atten_starting") + 1:]: v for k, v in trunk.blocks[0].state_dict().items()
                                      if k.startswith("tri_atten_starting.")}, dev)
    ws = torch.empty(int(_lib.load().ffb_triattn_workspace_bytes(1, n)), dtype=torch.uint8, device=dev)
    out = torch.empty_like(zz)
    kernels.triattn(zz, m512, packed, starting=True, stages=1, workspace=ws, out=out)
    for _ in range(3):
        kernels.triattn(zz, m512, packed, starting=True, stages=2, workspace=ws, out=out)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    a.record()
    for _ in range(20):
        kernels.triattn(zz, m512, packed, starting=True, stages=2, workspace=ws, out=out)
    b.record()
    torch.cuda.synchronize()
    attn_ms = a.elapsed_time(b) / 20
    attn_flops = 4.0 * n**3 * 128
    pk = peaks()
    achieved = attn_flops / (attn_ms * 1e-3) / 1e12

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value_ms, 3), "unit": "ms", "n_gpus": world, "steps": args.steps,
            "warmup": max(args.warmup, 3), "ms_per_step": round(value_ms, 3), "higher_is_better": False,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {
                "workload": f"{nb}-block Pairformer trunk, N={n_w} row-sharded over {world} GPUs (per-GPU work "
                            f"{n_w ** 3 / world / N_TOKENS ** 3:.2f} x the N=512 trunk), last {masked_w} tokens "
                            f"masked, master precision, {mode}",
                "model": "AF3 Pairformer block (c_z 128, c_s 384, 4x32 / 16x24 heads)",
                "global_batch": 1, "seq_len": n_w, "parallelism": f"axial row-sharding x{world} (NVLink peer-memory "
                                                                  "transposes / row gathers)",
                "l2": "flushed by a 256 MB write before every timed step",
                "trunk_tflops": round(block_flops(n_w) * nb / (value_ms * 1e-3) / 1e12, 1),
                "ms_per_block": round(value_ms / nb, 4),
            },
            "roofline": {
                "kernel": "triattn_attn_kernel (starting node, N=512, one GPU)",
                "bound": "tensor", "achieved": round(achieved, 1), "peak": pk["bf16"], "unit": "TFLOP/s",
                "frac": round(achieved / pk["bf16"], 4), "traffic": ATTN_TRAFFIC_BYTES,
                "launch_ms": round(attn_ms, 4), "peak_source": f"{pk['source']} (burst: kernel timed alone)",
                "algorithmic": f"4 * N^3 * 128 = {attn_flops:.3e} flop per launch",
            },
            "clocks": clocks,
            "gpu_launches": launches,
        }
        if e2e is not None:
            line["e2e"] = e2e
        if ladder is not None:
            line["ladder"] = ladder
        if breakdown is not None:
            line["breakdown"] = breakdown
        line["parity"] = parity
        print(json.dumps(line), flush=True)
    comm.close()  # every rank: unmap the peers' exchange buffers before the group goes


def sharded_parity(trunk, blocks, comm, rows_h, s_h, mask, n: int, rank: int, dev, dist, nblocks: int = 2) -> dict:
    """The first ``nblocks`` blocks of the row-sharded trunk (the NVLink peer-memory exchanges,
    and the channel-sharded TriMul from four ranks) against the same blocks unsharded on rank
    0's GPU, on the weak-scaling workload's inputs: relative L2 of pair and single on real
    positions, and whether padded pairs / tokens kept their input exactly (masked "zero")."""
    rows, s = rows_h.to(dev), s_h.to(dev)
    with torch.no_grad():
        for blk in blocks[:nblocks]:
            rows, s = blk(rows, mask, s)
        pair = comm.gather_rows(rows).clone()  # every rank takes part in the gather
    torch.cuda.synchronize()
    dist.barrier()
    result = {"blocks": nblocks, "n": n, "reference": "the same blocks unsharded on one GPU (b200)"}
    if rank == 0:
        from foldforge_b200.synthetic import inputs

        z_full = inputs(n, seed=0)[0].bfloat16().to(dev)  # the whole input pair the ranks' rows came from
        key = mask[None]
        zz, ss = z_full[None], s_h.to(dev)[None]
        with torch.no_grad():
            for block in trunk.blocks[:nblocks]:
                zz, ss = block(zz, key, ss)
        torch.cuda.synchronize()
        tok = mask.bool()
        pm = tok[:, None] & tok[None, :]

        def rel(a, b, where):
            a, b = a.float()[where], b.float()[where]
            return float((a - b).norm() / b.norm().clamp_min(1e-30))

        result.update({
            "rel_l2_pair": round(rel(pair, zz[0], pm), 6),
            "rel_l2_single": round(rel(s, ss[0], tok), 6),
            "masked_exact": bool(torch.equal(pair[~pm], z_full[~pm]) and torch.equal(s[~tok], s_h.to(dev)[~tok])),
        })
    dist.barrier()
    return result


def dit_once() -> None:
    """One AF3 TokenDiT block (b200) on 5 samples x 512 tokens, three passes (the tables are
    built on the first): a driver for ncu launch lists and captures, no timing."""
    from foldforge_b200 import _lib
    from foldforge_b200.engine.dit import TokenDiT, TokenDiTStack
    from foldforge_b200.synthetic import dit_inputs, dit_stack_state

    dev = torch.device("cuda")
    blk = TokenDiT()
    blk.load_state_dict(dit_stack_state(1, 0, "baseline")[0], strict=True)
    stack = TokenDiTStack([blk]).to(dev).eval()
    blk.set_backend("b200")
    x, cond, pair, mask = dit_inputs(5, 512, 0)
    x, cond, pair, mask = x.bfloat16().to(dev), cond.bfloat16().to(dev), pair.bfloat16().to(dev), mask.to(dev) > 0
    with torch.no_grad():
        for _ in range(3):
            stack(x, mask, cond, pair, key_mask=mask[None])
    torch.cuda.synchronize()
    print(f"dit-once: device error word {_lib.device_error()}")


def kernels_once(n: int) -> None:
    """Each kernel of one block once on the bench's inputs: TriMul outgoing stages 1, 2, 4,
    TriAttn starting stages 1, 2, 4, pair transition, attention with pair bias, single
    transition."""
    from foldforge_b200 import _lib, kernels
    from foldforge_b200.synthetic import block_state, inputs

    st = block_state(torch.Generator().manual_seed(0))
    sub = lambda pre: {k[len(pre) + 1:]: v for k, v in st.items() if k.startswith(pre + ".")}  # noqa: E731
    dev = torch.device("cuda")
    z, s, tok = inputs(n, 0, masked_suffix=round(MASKED * n / N_TOKENS))
    z, s, mask = z.bfloat16()[None].to(dev), s.bfloat16()[None].to(dev), (tok > 0)[None].to(dev)
    lib = _lib.load()
    out = torch.empty_like(z)
    pk = kernels.trimul_prepare(sub("tri_multi_outgoing"), dev)
    ws = torch.empty(int(lib.ffb_trimul_workspace_bytes(1, n)), dtype=torch.uint8, device=dev)
    for stg in (1, 2, 4):
        kernels.trimul(z, mask, pk, outgoing=True, stages=stg, workspace=ws, out=out)
    pk = kernels.triattn_prepare(sub("tri_atten_starting"), dev)
    ws = torch.empty(int(lib.ffb_triattn_workspace_bytes(1, n)), dtype=torch.uint8, device=dev)
    for stg in (1, 2, 4):
        kernels.triattn(z, mask, pk, starting=True, stages=stg, workspace=ws, out=out)
    kernels.transition(z, mask, kernels.transition_prepare(sub("transition_pair"), dev))
    kernels.attention_pair_bias(s, z, mask, kernels.apb_prepare(sub("single_attention"), dev))
    kernels.single_transition(s, mask, kernels.single_transition_prepare(sub("single_transition"), dev))
    torch.cuda.synchronize()
    err = _lib.device_error()
    print(f"kernels-once N={n}: device error word {err}")
    if err:
        raise SystemExit(1)


def main() -> None:
    args = parse()
    if args.dit_once:
        dit_once()
        return
    if args.kernels_once:
        kernels_once(args.n)
        return
    rank, world, local, dist = dist_setup(args.gpus)
    try:
        if args.impl == "reference":
            run_reference(args, rank, world)
        elif world > 1:
            run_sharded(args, rank, world, local, dist)
        else:
            run_b200(args, rank, world, local, dist)
    finally:
        if dist is not None:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
