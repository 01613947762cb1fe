"""Pairformer trunk benchmark on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

One step = one forward pass of the full 48-block Pairformer trunk at
N_token = 512 (475 real tokens, token mask zeroes the rest), c_z = 128,
c_s = 384, bf16 activations with fp32 accumulation, random-init weights
(seed 0), z ~ N(0,1), s ~ N(0,1) — synthetic data of the reference's shapes.
``value`` is ms per Pairformer block (trunk time / 48), max over ranks.
With --gpus N > 1 the pair rows are sharded over the N ranks (NCCL
all-gathers / all-to-alls as in the reference's distributed blocks) on the same
workload (strong scaling); --n-token 2048 selects configs[4] (1931 real tokens).

``--impl reference`` times the reference's own CPU path (its
blocks.PairFormerIteration from the package installed under baseline/_ref,
backend "torch" on the CPU; the oracle restatement oracle/pairformer.py where
that package is absent) on this host's cores, one exact block of the same
workload per step, and prints the same JSON line.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

N_TOKEN, N_REAL, N_BLOCKS, C_Z, C_S = 512, 475, 48, 128, 384
METRIC = "pairformer_ms_per_block"
UNIT = "ms/block"


def block_flops(n: int) -> float:
  """Algorithmic FLOPs of one Pairformer block at padded N (1536 N^3 + 1,121,792 N^2 + 5,013,504 N)."""
  return 1536.0 * n**3 + 1121792.0 * n**2 + 5013504.0 * n


def tri_attention_core_flops(n: int, heads: int = 4, d: int = 32) -> float:
  """4 * Nq * Nk * d * H * batch for one triangle attention (batch = N rows)."""
  return 4.0 * n * n * d * heads * n


def load_peaks() -> dict:
  path = os.path.join(REPO, "MEASURED_PEAKS.json")
  if os.path.exists(path):
    with open(path) as f:
      p = json.load(f)
    return {"hbm_gbs": p["hbm_gbs"], "bf16_tflops": p["bf16_tflops"],
            "bf16_tflops_sustained": p.get("bf16_tflops_sustained", p["bf16_tflops"]), "source": "measured"}
  return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class ClockSampler:
  """nvidia-smi clocks and throttle reasons sampled every 50 ms while active."""

  FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
            "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
            "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

  def __init__(self, index: int):
    # nvidia-smi numbers GPUs physically; with CUDA_VISIBLE_DEVICES set, local device `index`
    # is another one, so the GPU is named by its UUID when torch reports it
    self.index = index
    try:
      import torch
      uuid = str(torch.cuda.get_device_properties(index).uuid)
      self.index = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
    except Exception:
      pass
    self.proc = None

  def __enter__(self):
    try:
      self.proc = subprocess.Popen(
          ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
           "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
    except OSError:
      self.proc = None
    return self

  def __exit__(self, *exc):
    self.lines = []
    if self.proc is not None:
      self.proc.terminate()
      try:
        out, _ = self.proc.communicate(timeout=5)
      except subprocess.TimeoutExpired:
        self.proc.kill()
        out, _ = self.proc.communicate()
      self.lines = [ln for ln in out.splitlines() if ln.strip()]
    return False

  def summary(self) -> dict:
    sm, mx, reasons = [], None, set()
    names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    for ln in getattr(self, "lines", []):
      parts = [p.strip() for p in ln.split(",")]
      if len(parts) < 9:
        continue
      try:
        sm.append(float(parts[1]))
        mx = float(parts[2])
      except ValueError:
        continue
      for name, flag in zip(names, parts[5:9]):
        if flag.lower().startswith("active"):
          reasons.add(name)
    return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
            "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
def dist_setup(n_gpus: int):
  import datetime
  import torch
  import torch.distributed as dist
  world = int(os.environ.get("WORLD_SIZE", "1"))
  rank = int(os.environ.get("RANK", "0"))
  local = int(os.environ.get("LOCAL_RANK", "0"))
  if world != n_gpus:
    raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}")
  if torch.cuda.is_available():
    torch.cuda.set_device(local)
  if world > 1:
    dist.init_process_group("nccl" if torch.cuda.is_available() else "gloo",
                            timeout=datetime.timedelta(seconds=300))
  return rank, world, local


def barrier(world):
  if world > 1:
    import torch.distributed as dist
    dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
  if world == 1:
    return x
  import torch
  import torch.distributed as dist
  t = torch.tensor([x], dtype=torch.float64, device="cuda")
  dist.all_reduce(t, op=dist.ReduceOp.MAX)
  return float(t.item())


def build_trunk(device, n_blocks=N_BLOCKS, seed=0):
  import torch
  from sparsefold_b200 import modules, synth
  trunk = modules.PairformerTrunk(n_blocks, C_Z, C_S)
  synth.init_params(trunk, seed=seed)
  trunk = trunk.to(device)
  modules.prepare(trunk)
  # the fp32 master parameters are not used by the bf16 kernels; drop them from HBM
  for p in trunk.parameters():
    p.data = torch.empty(0, device=device)
  return trunk


def flush_l2(buf):
  buf.add_(1)


def tri_attention_op_flops(n: int) -> float:
  """Algorithmic FLOPs of one GridSelfAttention call: core 512 N^3 + projections
  (q, k, v, gate, bias: 2*128*(512+4) per position) + output projection (2*128*128)."""
  return tri_attention_core_flops(n) + n * n * (2.0 * 128 * 516 + 2.0 * 128 * 128)


# DRAM bytes of one triangle attention (projection + core) at N=512, from one ncu capture
# (dram__bytes_read.sum + dram__bytes_write.sum; profiles/k_triatt_tc_n512.md).
TRI_ATT_TRAFFIC_N512 = int((67.32 + 215.30 + 337.74 + 55.81) * 1e6)


def tri_attention_exp2_count(n: int) -> float:
  """exp2 evaluations of one attention call: one per (row, head, query, key)."""
  return 4.0 * n * n * n


def time_kernel_probe(n: int, dtype, iters: int = 10) -> float:
  """Average device time (ms) of one triangle attention (starting node) on [n, n, 128]."""
  import torch
  from sparsefold_b200 import modules, synth
  m = modules.GridSelfAttention(128, 4, transpose=False)
  synth.init_params(m, seed=3)
  m = m.cuda()
  modules.prepare(m)
  z, _, mask = synth.pair_inputs(n, n_real=N_REAL * n // N_TOKEN, seed=3)
  z = z.to("cuda", dtype)
  mask = mask.cuda()
  for _ in range(2):
    m(z, mask)
  st = torch.cuda.current_stream()
  ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(iters)]
  torch.cuda.synchronize()
  for a, b in ev:
    a.record(st)
    m(z, mask)
    b.record(st)
  torch.cuda.synchronize()
  return sum(a.elapsed_time(b) for a, b in ev) / iters


def measure_configs4(trunk, world: int, rank: int, dev, l2_flush, steps: int = 2, warmup: int = 1) -> dict:
  """configs[4] beside the headline: the 48-block trunk at N_token=2048 (1931 real), pair rows sharded over
  the job's ranks, device time per block (max over ranks, L2 flushed before each step); with more than one
  rank, rank 0 also times the unsharded trunk alone on its GPU in the same run, so the parallel efficiency
  T1 / (P * TP) comes from one run on one box."""
  import torch
  from sparsefold_b200 import sharding, synth
  n4, r4 = 2048, 1931
  dt = torch.bfloat16
  shard = sharding.Shard(n4, world, rank)
  z_h, s_h, m_h = synth.pair_inputs(n4, C_Z, C_S, n_real=r4, seed=0)
  mask = m_h.to(dev)

  def timed(z, s, sharded):
    run = (lambda: sharding.pairformer_trunk(trunk, z, s, mask, shard)) if sharded else (lambda: trunk(z, s, mask))
    for _ in range(warmup):
      run()
    st = torch.cuda.current_stream()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    torch.cuda.synchronize()
    for a, b in evs:
      flush_l2(l2_flush)
      a.record(st)
      run()
      b.record(st)
    torch.cuda.synchronize()
    return sum(a.elapsed_time(b) for a, b in evs) / steps / N_BLOCKS

  if world > 1:
    zl, sl = shard.shard(z_h).contiguous().to(dev, dt), shard.shard(s_h).contiguous().to(dev, dt)
    barrier(world)
    tp = max_over_ranks(timed(zl, sl, True), world)
    del zl, sl
  t1 = None
  if rank == 0:
    t1 = timed(z_h.to(dev, dt), s_h.to(dev, dt), False)
    torch.cuda.empty_cache()
  barrier(world)
  if world == 1:
    tp = t1
  out = {"workload": "configs[4]: 48-block Pairformer trunk, N_token=2048 (1931 real), 4 chains of 512, bf16",
         "n_gpus": world, "ms_per_block": round(tp, 3), "steps": steps, "warmup": warmup,
         "block_gflop": round(block_flops(n4) / 1e9, 1), "trunk_tflop_per_s": round(block_flops(n4) / (tp * 1e-3) / 1e12, 2)}
  if rank == 0 and world > 1:
    out["ms_per_block_1gpu_same_run"] = round(t1, 3)
    out["efficiency_vs_1gpu_same_run"] = round(t1 / (world * tp), 4)
  return out


def run_b200(args) -> None:
  import torch
  from sparsefold_b200 import _native, synth
  rank, world, local = dist_setup(args.gpus)
  if not torch.cuda.is_available():
    raise SystemExit("bench.py --impl b200 needs a CUDA device")
  _native.check(_native.load().sf_device_check(), "sf_device_check")
  from sparsefold_b200 import sharding
  dev = torch.device("cuda", local)
  dt = torch.bfloat16
  n_tok = args.n_token
  n_real = {512: N_REAL, 2048: 1931}.get(n_tok, n_tok)
  trunk = build_trunk(dev)
  shard = sharding.Shard(n_tok, world, rank)
  # identical inputs on every rank (seed 0); each rank keeps its row shard
  z_h, s_h, m_h = synth.pair_inputs(n_tok, C_Z, C_S, n_real=n_real, seed=0)
  if world > 1:
    z_h = shard.shard(z_h).contiguous()
    s_h = shard.shard(s_h).contiguous()
  z0 = z_h.to(dev, dt)
  s0 = s_h.to(dev, dt)
  mask = m_h.to(dev)
  l2_flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)   # 2x the 126 MB L2
  st = torch.cuda.current_stream()

  def run_trunk(z, s, m):
    if world == 1:
      return trunk(z, s, m)
    return sharding.pairformer_trunk(trunk, z, s, m, shard)

  with torch.no_grad():
    for _ in range(args.warmup):
      run_trunk(z0, s0, mask)
    torch.cuda.synchronize()

    # ---- device-resident timing: K trunk passes, L2 flushed between them ----
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    barrier(world)
    torch.cuda.synchronize()
    launches0 = _native.launch_count()
    with ClockSampler(local) as clk:
      for a, b in evs:
        flush_l2(l2_flush)
        a.record(st)
        run_trunk(z0, s0, mask)
        b.record(st)
      torch.cuda.synchronize()
    launches = _native.launch_count() - launches0
    barrier(world)
    ms_total = sum(a.elapsed_time(b) for a, b in evs)
    ms_total = max_over_ranks(ms_total, world)
    ms_step = ms_total / args.steps
    ms_block = ms_step / N_BLOCKS

    # ---- end to end through the public module API with host buffers ----
    zp = z_h.to(dt).pin_memory()
    sp = s_h.to(dt).pin_memory()
    mp = m_h.pin_memory()
    zo = torch.empty_like(zp).pin_memory()
    so = torch.empty_like(sp).pin_memory()
    e2e_steps = max(1, min(args.steps, 3))
    eev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(e2e_steps)]
    barrier(world)
    torch.cuda.synchronize()
    for a, b in eev:
      flush_l2(l2_flush)
      a.record(st)
      zd = zp.to(dev, non_blocking=True)
      sd = sp.to(dev, non_blocking=True)
      md = mp.to(dev, non_blocking=True)
      zr, sr = run_trunk(zd, sd, md)
      zo.copy_(zr, non_blocking=True)
      so.copy_(sr, non_blocking=True)
      b.record(st)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in eev) / e2e_steps, world)
    h2d = zp.numel() * zp.element_size() + sp.numel() * sp.element_size() + mp.numel()
    d2h = zo.numel() * zo.element_size() + so.numel() * so.element_size()

    # ---- dominant-kernel roofline: triangle attention core ----
    probe_ms = time_kernel_probe(N_TOKEN, dt) if rank == 0 else 0.0

    # ---- the N=2048 trunk (1931 real tokens), rows sharded over the same ranks ----
    c4 = measure_configs4(trunk, world, rank, dev, l2_flush) if args.configs4 else None

  peaks = load_peaks()
  flops = tri_attention_op_flops(N_TOKEN)
  achieved = flops / (probe_ms * 1e-3) / 1e12 if probe_ms > 0 else 0.0
  cpu = cpu_baseline_sample(n_tok, n_real) if rank == 0 and world == 1 and not args.no_cpu_baseline else None
  if rank == 0:
    line = {
        "metric": METRIC, "value": round(ms_block, 4), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 3),
        "higher_is_better": False, "scaling": "strong" if world > 1 else "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) pair/single, random-init AF3-shaped weights)",
        "config": workload_config(n_tok, n_real, world),
        "trunk_tflop_per_s": round(block_flops(n_tok) / (ms_block * 1e-3) / 1e12, 2),
        "e2e": {"value": round(e2e_ms / N_BLOCKS, 4), "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "gpu_launches": int(launches),
        "roofline": {"kernel": "triangle attention op (sf_tri_attention: projection + tcgen05 attention core "
                               "with fused output projection), N=512, 4 heads x 32",
                     "bound": "tensor", "achieved": round(achieved, 2), "peak": peaks["bf16_tflops"],
                     "unit": "TFLOP/s", "frac": round(achieved / peaks["bf16_tflops"], 4),
                     "peak_source": peaks["source"], "launch_ms": round(probe_ms, 4),
                     "traffic": TRI_ATT_TRAFFIC_N512 if N_TOKEN == 512 else None,
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of k_triatt_project_tc + "
                                       "k_triatt_core_tc, profiles/k_triatt_tc_n512.md",
                     "exp2_bound_ms": round(tri_attention_exp2_count(N_TOKEN) / (16 * 148 * 1.9e9) * 1e3, 4)},
        "clocks": clk.summary(),
        "cpu_baseline": cpu,
        "configs4": c4,
    }
    print(json.dumps(line), flush=True)
  if world > 1:
    import torch.distributed as dist
    from sparsefold_b200 import sharding
    sharding.close_peer_exchanges()
    dist.destroy_process_group()


# ---------------------------------------------------------------------------
# CPU side: the reference's own PairFormerIteration (the pip-installed package
# under baseline/_ref, backend "torch" on the CPU with math SDPA: the path the
# reference runs without a GPU) on this host's cores.  Where that package is
# absent, the oracle restatement of the same path (oracle/pairformer.py) runs
# instead and the line says kind "port".
# ---------------------------------------------------------------------------
def _cpu_threads() -> int:
  import torch
  n = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
  torch.set_num_threads(n)
  return torch.get_num_threads()


def _reference_package() -> bool:
  """Put the installed reference (baseline/_ref) on sys.path; False when it is not there."""
  import types
  src = os.path.join(REPO, "baseline", "_ref")
  if not os.path.isdir(os.path.join(src, "sparsefold")):
    return False
  if src not in sys.path:
    sys.path.insert(0, src)
  try:
    import zstandard  # noqa: F401  (only checkpoint reading uses it)
  except ImportError:
    sys.modules["zstandard"] = types.ModuleType("zstandard")
  return True


def cpu_block_runner(n: int, n_real: int):
  """(run, kind, what): run() is one Pairformer block forward at N=n on the CPU in bf16."""
  import torch
  from sparsefold_b200 import synth
  dt = torch.bfloat16
  z, s, mask = synth.pair_inputs(n, C_Z, C_S, n_real=n_real, seed=0)
  z, s = z.to(dt), s.to(dt)
  if _reference_package():
    from sparsefold.runtime import config
    from sparsefold import backends
    config.configure_runtime(backend="torch", device="cpu", sdpa_implementation="math", enable_sharding=False,
                             enable_compile=False, logs=set())
    backends.init()
    from sparsefold.model.trunk import blocks, network
    from sparsefold.model import config as mc
    blk = blocks.PairFormerIteration(network.Evoformer.Config().pairformer, mc.GlobalConfig(), with_single=True,
                                     num_channels=C_Z, seq_channels=C_S)
    synth.init_params(blk, seed=0)
    blk = blk.to(dt).eval()

    def run():
      with torch.no_grad():
        blk(z, seq_mask=mask, single_act=s)
    return run, "reference", ("the reference's own blocks.PairFormerIteration (baseline/_ref, backend torch, "
                              "device cpu, math SDPA), bf16 weights and activations")
  from oracle import pairformer as orc
  from sparsefold_b200 import modules
  holder = modules.PairFormerIteration(C_Z, C_S)
  p = {k: v.to(dt) for k, v in synth.init_params(holder, seed=0).items()}

  def run():
    with torch.no_grad():
      orc.pairformer_block(z, s, mask, p)
  return run, "port", "oracle/pairformer.py restatement of the reference Torch CPU math path, bf16 tensors"


def _time_cpu(run, steps: int, warmup: int) -> list:
  out = []
  for i in range(warmup + steps):
    t0 = time.perf_counter()
    run()
    if i >= warmup:
      out.append(time.perf_counter() - t0)
  return out


def cpu_baseline_sample(n_tok: int, n_real: int) -> dict:
  """One exact Pairformer block of the bench workload on the host (after one untimed block)."""
  cores = _cpu_threads()
  run, kind, what = cpu_block_runner(n_tok, n_real)
  t = min(_time_cpu(run, 1, 1))
  return {"value": round(t * 1e3, 2), "unit": UNIT, "cores": cores, "kind": kind,
          "sample": f"1 Pairformer block at N={n_tok} ({n_real} real) timed exactly: {what}"}


def workload_config(n_tok: int, n_real: int, world: int) -> dict:
  """The `config` object both arms print (the driver compares them)."""
  tag = "configs[1]" if n_tok == 512 else "configs[4]" if n_tok == 2048 else "custom"
  return {"workload": f"{tag}: 48-block Pairformer trunk, N_token={n_tok} ({n_real} real), c_z=128, c_s=384",
          "n_token": n_tok, "n_real": n_real, "blocks": N_BLOCKS,
          "block_gflop": round(block_flops(n_tok) / 1e9, 1),
          "l2": "b200 arm: flushed (256 MiB write) before every timed step",
          "parallelism": f"pair rows sharded over {world} GPUs (NCCL)" if world > 1 else "single"}


def run_reference(args) -> None:
  """The reference arm: one exact Pairformer block of the workload per step on the host cores."""
  rank = int(os.environ.get("RANK", "0"))
  world = int(os.environ.get("WORLD_SIZE", "1"))
  if rank != 0:
    return
  cores = _cpu_threads()
  n_tok = args.n_token
  n_real = {512: N_REAL, 2048: 1931}.get(n_tok, n_tok)
  n_s = args.sample_n or n_tok
  n_real_s = n_real if n_s == n_tok else max(1, n_s * n_real // n_tok)
  run, kind, what = cpu_block_runner(n_s, n_real_s)
  times = _time_cpu(run, args.steps, args.warmup)
  ms_block = statistics.median(times) * 1e3
  sample = f"per step 1 Pairformer block at N={n_s} ({n_real_s} real) timed exactly: {what}"
  line = {
      "metric": METRIC, "value": round(ms_block, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
      "warmup": args.warmup, "ms_per_step": round(ms_block, 1), "higher_is_better": False,
      "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
      "data": "synthetic (seeded N(0,1) pair/single, random-init AF3-shaped weights)",
      "config": workload_config(n_tok, n_real, 1),
      "impl": "reference",
      "cpu_baseline": {"value": round(ms_block, 2), "unit": UNIT, "cores": cores, "kind": kind, "sample": sample},
      "e2e": {"value": round(ms_block, 2), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
  }
  print(json.dumps(line), flush=True)


OPS = ("tri_attention_start", "tri_attention_end", "tri_mult_outgoing", "tri_mult_incoming", "pair_transition",
       "single_update", "single_attention", "diffusion_transformer", "diffusion_step", "atom_transformer",
       "msa_attention", "outer_product_mean", "pair_embedding", "diffusion_pair_cond")


def op_flops(op: str, n: int) -> float:
  """Algorithmic FLOPs of one op at its workload (pair ops at N_token = n)."""
  if op.startswith("tri_attention"):
    return tri_attention_op_flops(n)
  if op.startswith("tri_mult"):
    return 256.0 * n**3 + n * n * 2.0 * 128 * (512 + 128 + 128)
  if op == "pair_transition":
    return n * n * 2.0 * 128 * (1024 + 512)
  if op == "single_attention":           # 16 heads x 24: 4 N^2 d H
    return 4.0 * n * n * 24 * 16
  return 0.0


def _diffusion_token_flops(s: int, n: int, c: int, h: int, d: int, blocks: int, sc: int, pc: int) -> float:
  """One denoising step of the token transformer (diffusion/transformer.py:348-477), s samples."""
  per = (2.0 * s * n * c * 4 * c          # q, k, v, gate
         + 4.0 * s * h * n * n * d        # attention core
         + 2.0 * s * n * c * c            # adaptive-zero transition2 of the attention
         + 2.0 * s * n * c * 4 * c        # transition W1 (2 x 2c)
         + 2.0 * s * n * 2 * c * c        # transition W2
         + 2 * (2.0 * 2 * n * sc * c)     # AdaLN scale and bias of both sub-blocks
         + 2 * 2.0 * n * sc * c)          # adaptive-zero gates
  return blocks * per + 2.0 * n * n * pc * blocks * h


def _atom_flops(s: int, nsub: int, q: int, k: int, c: int, h: int, d: int, blocks: int) -> float:
  """CrossAttTransformer (transformer.py:588-693): s samples, nsub windows of q queries x k keys."""
  nq, nk = nsub * q, nsub * k
  per = (2.0 * s * nq * c * 2 * h * d     # q and gate
         + 2.0 * s * nk * c * 2 * h * d   # k and v of the gathered windows
         + 4.0 * s * nsub * h * q * k * d # attention core
         + 2.0 * s * nq * h * d * c       # adaptive-zero transition2
         + 2.0 * s * nq * c * 4 * c       # transition W1
         + 2.0 * s * nq * 2 * c * c       # transition W2
         + 2.0 * (2 * nq + 2 * nk) * c * c + 4.0 * nq * c * c)   # AdaLN (queries, keys) and gates
  return blocks * per


def op_bytes(op: str, n: int) -> float:
  """Algorithmic HBM bytes of one call of the bandwidth-bound ops (each input read once, the result
  written once, bf16)."""
  if op == "pair_embedding":     # relative encoding (139) + contact (1) + previous pair in, pair out
    return n * n * 2.0 * (139 + 1 + 128 + 128)
  if op == "diffusion_pair_cond":   # [pair | relative encoding] (128 + 139) in, pair_cond out
    return n * n * 2.0 * (128 + 139 + 128)
  return 0.0


def _one_hot_rel(n: int, g):
  """Relative-encoding-shaped features [n, n, 139]: one-hot position (66), token (66), chain (6) bins and a
  0/1 same-entity flag (trunk/network.py:171-186)."""
  import torch
  x = torch.zeros(n, n, 139)
  i = torch.arange(n)
  x[i[:, None], i[None, :], torch.clamp(i[:, None] - i[None, :] + 32, 0, 64)] = 1.0
  x[i[:, None], i[None, :], 66 + torch.clamp(i[:, None] - i[None, :] + 32, 0, 64)] = 1.0
  x[..., 132] = 1.0
  x[i[:, None], i[None, :], 133 + torch.randint(0, 6, (n, n), generator=g)] = 1.0
  return x


def _workload_op(op: str, n: int):
  """(run, flops, what) for the workload ops of configs[2] and configs[3] and the single attention."""
  import types
  import torch
  from sparsefold_b200 import modules, ops, synth
  dt = torch.bfloat16
  g = torch.Generator().manual_seed(4)
  rn = lambda *shape: torch.randn(*shape, generator=g).to("cuda", dt)
  if op == "pair_embedding":
    # Evoformer pair embedding (computed once per prediction) and one recycling step
    # (trunk/network.py:344-372) on the b200 kernels, N = n tokens, bf16
    tf = rn(n, 447)
    wl, wr = rn(128, 447) * 0.05, rn(128, 447) * 0.05
    w_pos = (torch.randn(139, 128, generator=g) * 0.1).cuda()
    w_bond = (torch.randn(1, 128, generator=g) * 0.1).cuda()
    rel = _one_hot_rel(n, g).to("cuda", dt)
    contact = (torch.rand(n, n, 1, generator=g) > 0.99).to("cuda", dt)
    prev = rn(n, n, 128)
    ln_w, ln_b = torch.ones(128, device="cuda"), torch.zeros(128, device="cuda")
    wp = rn(128, 128) * 0.09

    def run():
      pos = ops.pair_sparse_linear(rel, w_pos)
      pair = ops.pair_outer_sum(ops.linear(tf, wl), ops.linear(tf, wr), addend=pos)
      pair = ops.pair_sparse_linear(contact, w_bond, residual=pair)
      return ops.linear(ops.layer_norm(prev, ln_w, ln_b), wp, residual=pair)
    return (run, 0.0, f"Evoformer pair embedding (outer sum of the single projections + relative-position "
                      f"encoding 139 one-hot + bonds) and one recycling step (LayerNorm + linear + residual), N={n}")
  if op == "diffusion_pair_cond":
    # DiffusionHead._get_base_cond, the pair half (diffusion/generator.py:367-391) at configs[2]'s N=768:
    # LayerNorm over [pair | relative encoding] (267), the fp32 ("highest") projection, two transitions
    n_ = 768
    pair, rel = rn(n_, n_, 128), _one_hot_rel(n_, g).to("cuda", dt)
    w_ln = torch.ones(267, device="cuda")
    w_proj = (torch.randn(128, 267, generator=g) * 0.06).cuda()
    tr = [modules.DiffusionTransitionBlock(128, 2) for _ in range(2)]
    for i, t in enumerate(tr):
      synth.init_params(t, seed=4 + i)
    tr = [t.cuda() for t in tr]
    for t in tr:
      modules.prepare(t)

    def run():
      f2 = torch.cat((pair, rel), dim=-1)
      pc = ops.linear(ops.layer_norm(f2, w_ln, None).float(), w_proj).to(dt)
      for t in tr:
        pc = t(pc)
      return pc
    fl = 2.0 * n_ * n_ * 267 * 128 + 2 * (2.0 * n_ * n_ * 128 * 512 + 2.0 * n_ * n_ * 256 * 128)
    return (run, fl, "DiffusionHead pair conditioning at N=768: LayerNorm(267) + fp32 projection 267->128 + "
                     "2 transitions")
  if op == "single_attention":
    h, d = 16, 24
    y = rn(n, 4, h, d)
    bias = rn(h, n, n)
    mk = (torch.arange(n) < max(1, N_REAL * n // N_TOKEN)).cuda()
    return (lambda: ops.attention(y[:, 0], y[:, 1], y[:, 2], mask_k=mk, bias=bias, gate=y[:, 3]), op_flops(op, n),
            f"Pairformer single attention core (sf_attention), N={n}, 16 heads x 24, pair-logit bias, gate")
  if op in ("diffusion_transformer", "diffusion_step"):
    s_, n_, c, sc, pc = 5, 768, 768, 384, 128
    m = modules.DiffusionTransformer(c, sc, pc, num_head=16, num_blocks=24, super_block_size=4)
    synth.init_params(m, seed=4)
    m = m.cuda()
    modules.prepare(m)
    act, single, pair = rn(s_, n_, c), rn(n_, sc), rn(n_, n_, pc)
    mask = torch.ones(n_, dtype=torch.bool, device="cuda")
    if op == "diffusion_step":   # the pack computed once, as for every step of a denoising loop
      with torch.no_grad():
        pack = m.pair_logits_pack(pair, dt)
      fl = _diffusion_token_flops(s_, n_, c, 16, 48, 24, sc, pc) - 2.0 * n_ * n_ * pc * 24 * 16
      return (lambda: m(act, mask, single, pair_logits_pack=pack), fl,
              "configs[2] token transformer, one step of a denoising loop: pair-logit pack cached, 24 blocks, "
              "5 samples, N=768, c=768, 16 x 48")
    return (lambda: m(act, mask, single, pair), _diffusion_token_flops(s_, n_, c, 16, 48, 24, sc, pc),
            "configs[2] token transformer, one denoising step: 24 blocks, 5 samples, N=768, c=768, 16 x 48, "
            "pair-logit pack from z [768,768,128]")
  if op == "atom_transformer":
    s_, nsub, q_, k_, c, pc = 5, 192, 32, 128, 128, 16
    m = modules.CrossAttTransformer(c, pc, num_head=4, key_dim=128, num_blocks=3, num_intermediate_factor=2)
    synth.init_params(m, seed=4)
    m = m.cuda()
    modules.prepare(m)
    starts = torch.clamp(32 * torch.arange(nsub) + 16 - 64, 0, nsub * q_ - k_)
    idx = (starts[:, None] + torch.arange(k_)[None, :]).to(torch.int32).cuda()
    info = types.SimpleNamespace(gather_idxs=idx, gather_mask=torch.ones(nsub, k_, dtype=torch.bool, device="cuda"))
    qact, qsc, ksc, pcq = rn(s_, nsub, q_, c), rn(nsub, q_, c), rn(nsub, k_, c), rn(nsub, q_, k_, pc)
    qmask = torch.ones(nsub, q_, dtype=torch.bool, device="cuda")
    kmask = torch.ones(nsub, k_, dtype=torch.bool, device="cuda")
    return (lambda: m(qact, qmask, info, kmask, qsc, ksc, pcq), _atom_flops(s_, nsub, q_, k_, c, 4, 32, 3),
            "configs[2] atom encoder: 3 blocks, 5 samples, 6144 atoms in 192 windows of 32 queries x 128 keys, "
            "c_atom=128, 4 x 32")
  if op in ("msa_attention", "outer_product_mean"):
    m_, n_ = 1024, 768
    act = torch.nn.functional.one_hot(torch.randint(0, 32, (m_, n_), generator=g), 32).float()
    act = torch.cat([act, torch.randn(m_, n_, 32, generator=g)], -1).to("cuda", dt)   # c_m = 64
    mask = (torch.rand(m_, n_, generator=g) > 0.15).cuda()
    if op == "msa_attention":
      m = modules.MSAAttention(64, 128, 8)
      synth.init_params(m, seed=4)
      m = m.cuda()
      modules.prepare(m)
      pair = rn(n_, n_, 128)
      fl = 2.0 * 8 * m_ * 8 * n_ * n_ + 3 * 2.0 * m_ * n_ * 64 * 64 + 2.0 * n_ * n_ * 128 * 8
      return (lambda: m(act, mask, pair), fl,
              "configs[3] MSA pair-weighted averaging (MSAAttention), 1024 MSA rows x 768 tokens, 8 x 8")
    m = modules.OuterProductMean(64, 128, 32)
    synth.init_params(m, seed=4)
    m = m.cuda()
    modules.prepare(m)
    fl = 2.0 * m_ * (n_ * 32) ** 2 + 2.0 * n_ * n_ * 1024 * 128 + 2 * 2.0 * m_ * n_ * 64 * 32
    return (lambda: m(act, mask), fl, "configs[3] outer-product mean, 1024 MSA rows x 768 tokens, c=32 -> 128")
  raise ValueError(op)


def run_op(args) -> None:
  """Time one op alone (per-kernel rooflines, small ncu captures, the configs[2]/[3] workloads)."""
  import torch
  from sparsefold_b200 import _native, modules, synth
  _native.check(_native.load().sf_device_check(), "sf_device_check")
  n = args.n
  pair_ops = {
      "tri_attention_start": lambda: modules.GridSelfAttention(128, 4, transpose=False),
      "tri_attention_end": lambda: modules.GridSelfAttention(128, 4, transpose=True),
      "tri_mult_outgoing": lambda: modules.TriangleMultiplication(128, "...ikc,...jkc->...ijc"),
      "tri_mult_incoming": lambda: modules.TriangleMultiplication(128, "...kjc,...kic->...ijc"),
      "pair_transition": lambda: modules.TransitionBlock(128, 4),
      "single_update": lambda: modules.SingleActUpdate(128, 384),
  }
  if args.op in pair_ops:
    m = pair_ops[args.op]()
    synth.init_params(m, seed=4)
    m = m.cuda()
    modules.prepare(m)
    z, s, mask = synth.pair_inputs(n, n_real=max(1, N_REAL * n // N_TOKEN), seed=4)
    z, s, mask = z.to("cuda", torch.bfloat16), s.to("cuda", torch.bfloat16), mask.cuda()
    run = {
        "pair_transition": lambda: m(z),
        "single_update": lambda: m(z, s, mask),
    }.get(args.op, lambda: m(z, mask))
    fl, what = op_flops(args.op, n), f"{args.op}, N={n}"
  else:
    run, fl, what = _workload_op(args.op, n)
  with torch.no_grad():
    for _ in range(args.warmup):
      run()
    torch.cuda.synchronize()
    l0 = _native.launch_count()
    run()
    torch.cuda.synchronize()
    launches = _native.launch_count() - l0
    # device time per call: the call captured once in a CUDA graph and replayed, so that the host's
    # Python and ctypes work between launches (which a small op cannot hide) is not timed
    graph = None
    if not args.no_graph:
      try:
        cap = torch.cuda.Stream()
        cap.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(cap):
          run()
        torch.cuda.current_stream().wait_stream(cap)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
          run()
        graph.replay()
        torch.cuda.synchronize()
      except Exception:   # an op that cannot be captured is timed eagerly
        graph = None
    st = torch.cuda.current_stream()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    torch.cuda.synchronize()
    for a, b in ev:
      a.record(st)
      graph.replay() if graph is not None else run()
      b.record(st)
    torch.cuda.synchronize()
  ms = sum(a.elapsed_time(b) for a, b in ev) / args.steps
  peaks = load_peaks()
  nbytes = op_bytes(args.op, n)
  hbm = ({"gbytes": round(nbytes / 1e9, 4), "gb_per_s": round(nbytes / (ms * 1e-3) / 1e9, 1),
          "frac_of_hbm_peak": round(nbytes / (ms * 1e-3) / 1e9 / peaks["hbm_gbs"], 4)} if nbytes else {})
  print(json.dumps({"op": args.op, "what": what, "n_token": n, "ms": round(ms, 4), **hbm,
                    "timing": "CUDA graph replay" if graph is not None else "eager launches",
                    "gflop": round(fl / 1e9, 2) if fl else None,
                    "tflop_per_s": round(fl / (ms * 1e-3) / 1e12, 2) if fl else None,
                    "frac_of_bf16_peak": round(fl / (ms * 1e-3) / 1e12 / peaks["bf16_tflops"], 4) if fl else None,
                    "peak_source": peaks["source"], "launches_per_call": int(launches),
                    "device_status": _native.device_status()}), flush=True)


def main():
  ap = argparse.ArgumentParser()
  ap.add_argument("--gpus", type=int, default=1)
  ap.add_argument("--steps", type=int, default=3)
  ap.add_argument("--warmup", type=int, default=3)
  ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
  ap.add_argument("--no-cpu-baseline", action="store_true")
  ap.add_argument("--no-configs4", dest="configs4", action="store_false",
                  help="skip the configs[4] (N_token=2048) trunk measured beside the headline")
  ap.add_argument("--op", choices=OPS, default=None, help="time one op alone instead of the trunk")
  ap.add_argument("--n", type=int, default=N_TOKEN, help="N_token for --op")
  ap.add_argument("--no-graph", action="store_true", help="--op: time eager launches instead of a graph replay")
  ap.add_argument("--n-token", type=int, default=N_TOKEN, help="N_token of the trunk (512 = configs[1], 2048 = configs[4])")
  ap.add_argument("--sample-n", type=int, default=None,
                  help="reference arm only: time blocks of this N instead of the workload's (quick CPU checks)")
  args = ap.parse_args()
  if args.op:
    run_op(args)
    return
  if args.warmup < 3 and args.impl == "b200":
    raise SystemExit("--warmup must be >= 3")
  if args.impl == "reference":
    run_reference(args)
  else:
    run_b200(args)


if __name__ == "__main__":
  main()
