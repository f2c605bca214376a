#!/usr/bin/env python
"""Headline benchmark: bias-fused attention forward + backward at N_res = 1024 (bf16).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One "step" is one forward (with lse) plus one backward (dq, dk, dv, dbias) of MSA-row attention with pair
bias at (batch, heads, seq, head_dim) = (512, 8, 1024, 32), 'seq' layout, Bernoulli(0.95) key mask, on
synthetic seeded inputs.  With N > 1 (launched by torch.distributed.run, one rank per GPU) every rank runs
its own 512 batch rows: the batch axis is independent, so there is no data-path collective ("weak" scaling).

The JSON line carries:
  value         whole-job TFLOP/s, inputs resident in HBM, CUDA-event timed, max over ranks
  e2e           the same metric through the public selector API with pinned HOST buffers: host->device copies
                of q, k, v, bias, mask and the cotangent and device->host copies of out, dq, dk, dv, dbias are
                inside the timed region (the batch streams through in chunks so that copies and kernels overlap)
  roofline      the dominant kernel (the backward) against the measured dense-bf16 peak
  cpu_baseline  the CPU oracle (a port of the reference's fp32 ref_attn and flash backward) timed on this
                box's host cores on a bounded sample of the same workload
`--impl reference` prints the CPU arm alone (the reference's own path needs JAX, which is not installed: the
port of its jnp reference stands in, kind "port").
"""
import argparse
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "colabfold-kernels_b200"))
sys.path.insert(0, ROOT)

B, H, S, D = 512, 8, 1024, 32
METRIC = "biased_attention_fwd_bwd_tflops"


def workload():
  return f"msa_row_attention_pair_bias fwd+bwd b={B} h={H} s={S} d={D} layout=seq mask=bernoulli0.95"


def flops(b):
  return 14.0 * b * H * S * S * D  # 4 forward + 10 backward (five GEMMs incl. the recompute), dense


def peaks():
  path = os.path.join(ROOT, "MEASURED_PEAKS.json")
  if os.path.exists(path):
    d = json.load(open(path))
    return float(d["bf16_tflops"]), float(d["hbm_gbs"]), "measured"
  return 1590.0, 6650.0, "fallback"


def sustained_peak():
  """Dense bf16 TFLOP/s of a seconds-long GEMM loop under the power cap: the denominator for a whole block."""
  path = os.path.join(ROOT, "MEASURED_PEAKS.json")
  if os.path.exists(path):
    return float(json.load(open(path)).get("bf16_tflops_sustained", 1400.0))
  return 1400.0


class ClockSampler(threading.Thread):
  """nvidia-smi clocks and throttle reasons every 200 ms while the timed region runs."""

  def __init__(self, index):
    super().__init__(daemon=True)
    self.rows, self.stop_flag, self.index = [], threading.Event(), index

  def run(self):
    q = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    while not self.stop_flag.is_set():
      try:
        out = subprocess.run(["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}", "--format=csv,noheader,nounits"],
                             capture_output=True, text=True, timeout=5).stdout.strip()
        if out:
          self.rows.append([c.strip() for c in out.split(",")])
      except Exception:
        pass
      self.stop_flag.wait(0.2)

  def summary(self):
    if not self.rows:
      return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
    mhz = sorted(int(r[0]) for r in self.rows if r[0].isdigit())
    names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    reasons = [n for i, n in enumerate(names) if any(r[2 + i].lower().startswith("active") for r in self.rows)]
    mx = [int(r[1]) for r in self.rows if r[1].isdigit()]
    return {"sm_mhz": mhz[len(mhz) // 2] if mhz else None, "sm_max_mhz": max(mx) if mx else None, "reasons": reasons}


def cpu_arm(steps, warmup, sample_b=32):
  """The CPU oracle on a bounded sample (sample_b batch rows of the same heads/seq/head_dim) on every host core.
  The thread count is set here: under torch.distributed.run the environment pins OMP_NUM_THREADS to 1."""
  import torch
  import oracle as O
  cores = os.cpu_count() or 1
  torch.set_num_threads(cores)
  g = torch.Generator().manual_seed(0)
  q, k, v, do = (torch.randn(sample_b, H, S, D, generator=g) for _ in range(4))
  bias = torch.randn(H, S, S, generator=g)
  kmask = torch.rand(sample_b, S, generator=g) < 0.95
  scale = D ** -0.5

  def step():
    out = O.ref_attn(q, k, v, bias, kmask, scale)
    lse = O.ref_attn_lse(q, k, bias, kmask, scale)
    return O.ref_attn_bwd(q, k, v, bias, kmask, out, do, lse, scale)

  n_warm, n_timed = max(1, min(warmup, 1)), max(1, min(steps, 3))
  for _ in range(n_warm):
    step()
  times = []
  for _ in range(n_timed):
    t0 = time.perf_counter()
    step()
    times.append(time.perf_counter() - t0)
  sec = sorted(times)[len(times) // 2]
  return {"value": flops(sample_b) / sec / 1e12, "unit": "TFLOP/s", "cores": torch.get_num_threads(), "kind": "port",
          "sample": f"{sample_b} of {B} batch rows (h={H}, s={S}, d={D}), fp32 PyTorch-CPU port of ref_attn + flash backward, "
                    f"median of {n_timed} timed samples after {n_warm} warm-up",
          "ms_per_sample": sec * 1e3, "steps_timed": n_timed, "warmup_run": n_warm, "sample_b": sample_b}


_PEER = {}


def peer_exchange(dev, want=True):
  """One PeerExchange per process (the all-to-alls of the sharded block as the library's kernels over NVLink peer
  memory), or None with the reason when symmetric memory cannot be set up: the block then uses NCCL's all-to-all."""
  if not want:
    return None, "nccl all_to_all_single / all_gather (peer exchange switched off)"
  if "x" not in _PEER:
    from colabfold_kernels import evoformer
    try:
      _PEER["x"], _PEER["how"] = evoformer.PeerExchange(None, dev), "cfk_peer_alltoall: all-to-alls and all-gathers as stores into NVLink peer memory"
    except Exception as e:  # no symmetric memory on this box / build
      _PEER["x"], _PEER["how"] = None, f"nccl all_to_all_single / all_gather (peer exchange unavailable: {type(e).__name__}: {str(e)[:120]})"
  return _PEER["x"], _PEER["how"]


def evoformer_block_ms(world, rank, dev, iters=3, n_seq=512, n_res=1024, fp8_trimul=False, fp8_attention=False, graph=True,
                       peer=True):
  """Second metric: one Evoformer block (inference wiring of the fused ops) at N_seq=512, N_res=1024, device-timed,
  max over ranks.  One GPU: the whole block; N GPUs: the same block row-sharded (total work fixed).  fp8_trimul: the
  reference's opt-in e4m3 contractions (triangle multiplication: half the bytes of the operand the ranks exchange; and
  the outer product of the MSA projections).  fp8_attention: e4m3 q and k in the four attentions."""
  import torch
  import torch.distributed as dist
  from colabfold_kernels import evoformer
  bf = torch.bfloat16
  g = torch.Generator().manual_seed(5)
  msa = torch.randn(n_seq, n_res, 256, generator=g).to(bf)
  pair = torch.randn(n_res, n_res, 128, generator=g).to(bf)
  msa_mask = (torch.rand(n_seq, n_res, generator=g) < 0.95).float().to(dev)
  pair_mask = (torch.rand(n_res, n_res, generator=g) < 0.95).float().to(dev)
  params = evoformer.init_params(device=dev)
  K = evoformer.cuda_kernels()
  if world > 1:
    blk = evoformer.ShardedBlock(K, params, fp8_trimul=fp8_trimul, fp8_attention=fp8_attention, fp8_opm=fp8_trimul,
                                 peer_exchange=peer_exchange(dev, peer)[0])
    msa_l, pair_l = msa[blk.shard(n_seq)].to(dev), pair[blk.shard(n_res)].to(dev)
    run = lambda: blk(msa_l, pair_l, msa_mask, pair_mask)
  else:
    msa_l, pair_l = msa.to(dev), pair.to(dev)
    run = lambda: evoformer.block(K, msa_l, pair_l, msa_mask, pair_mask, params, fp8_trimul=fp8_trimul, fp8_attention=fp8_attention,
                                  fp8_opm=fp8_trimul)
  for _ in range(2):
    run()
  if world > 1:
    dist.barrier()
  torch.cuda.synchronize()
  launch = "eager"
  if graph:
    # the block is ~100 short launches: one graph launch keeps the host out of the timed region
    run, _ = evoformer.capture(run)
    launch = "cuda graph"
    run()
    if world > 1:
      dist.barrier()
    torch.cuda.synchronize()
  e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
  e0.record()
  for _ in range(iters):
    run()
  e1.record()
  torch.cuda.synchronize()
  ms = torch.tensor([e0.elapsed_time(e1) / iters], device=dev)
  if world > 1:
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
  return float(ms), launch


def block_matches_single_gpu(world, rank, dev, n_seq=64, n_res=256, peer=True):
  """The row-sharded block against the one-GPU block on the same inputs at a small size: every rank runs its shard,
  rank 0 also runs the whole block and compares (max-abs error over max-abs value, both representations)."""
  import torch
  import torch.distributed as dist
  from colabfold_kernels import evoformer
  bf = torch.bfloat16
  n_res = max(n_res, 128 * world)  # the exchanged triangle multiplication wants 128 rows per rank: the form that is timed
  g = torch.Generator().manual_seed(7)
  msa = torch.randn(n_seq, n_res, 256, generator=g).to(bf).to(dev)
  pair = torch.randn(n_res, n_res, 128, generator=g).to(bf).to(dev)
  msa_mask = (torch.rand(n_seq, n_res, generator=g) < 0.95).float().to(dev)
  pair_mask = (torch.rand(n_res, n_res, generator=g) < 0.95).float().to(dev)
  params = evoformer.init_params(device=dev)
  K = evoformer.cuda_kernels()
  blk = evoformer.ShardedBlock(K, params, exchange_triangle=True,  # the form the large ranks counts take
                               peer_exchange=peer_exchange(dev, peer)[0])
  m_l, p_l = blk(msa[blk.shard(n_seq)].contiguous(), pair[blk.shard(n_res)].contiguous(), msa_mask, pair_mask)
  m_all = torch.empty((world,) + tuple(m_l.shape), dtype=bf, device=dev)
  p_all = torch.empty((world,) + tuple(p_l.shape), dtype=bf, device=dev)
  dist.all_gather_into_tensor(m_all, m_l.contiguous())
  dist.all_gather_into_tensor(p_all, p_l.contiguous())
  err = None
  if rank == 0:
    m1, p1 = evoformer.block(K, msa, pair, msa_mask, pair_mask, params)
    rel = lambda a, b: float((a.float() - b.float()).abs().max() / b.float().abs().max().clamp_min(1e-3))
    err = max(rel(m_all.reshape(m1.shape), m1), rel(p_all.reshape(p1.shape), p1))
  dist.barrier()
  return err, n_res


def main():
  ap = argparse.ArgumentParser()
  ap.add_argument("--gpus", type=int, default=1)
  ap.add_argument("--steps", type=int, default=5)
  ap.add_argument("--warmup", type=int, default=3)
  ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
  ap.add_argument("--block", type=int, default=1, help="also time one Evoformer block (0 to skip)")
  ap.add_argument("--block-graph", type=int, default=1, help="replay the block as one CUDA graph (0: launch op by op)")
  ap.add_argument("--peer-exchange", type=int, default=1,
                  help="sharded block: all-to-alls as the library's kernels over NVLink peer memory (0: NCCL)")
  ap.add_argument("--e2e-chunks", type=int, default=8, help="pieces the batch is streamed in by the end-to-end step")
  ap.add_argument("--batch", type=int, default=B, help="batch rows per GPU (smaller values are for profiler captures only)")
  args = ap.parse_args()
  globals()["B"] = args.batch
  # NCCL writes its log (NCCL_DEBUG) to file descriptor 1.  The JSON line must stand alone on stdout, so the process's
  # descriptor 1 is pointed at stderr and the line goes to a private copy of the original stdout.
  sys.stdout.flush()
  real_stdout = os.fdopen(os.dup(1), "w")
  os.dup2(2, 1)
  rank = int(os.environ.get("RANK", "0"))
  world = int(os.environ.get("WORLD_SIZE", "1"))
  local_rank = int(os.environ.get("LOCAL_RANK", "0"))

  if args.impl == "reference":
    if rank != 0:
      return
    cb = cpu_arm(args.steps, args.warmup)
    # `steps` / `warmup` are what was run (the sample is bounded, so at most three timed samples); ms_per_step is the
    # estimate for the whole workload: the time of the sample times B / sample rows (the work is linear in the batch)
    line = {"impl": "reference", "metric": METRIC, "value": cb["value"], "unit": "TFLOP/s", "n_gpus": args.gpus,
            "steps": cb["steps_timed"], "warmup": cb["warmup_run"], "ms_per_step": cb["ms_per_sample"] * B / cb["sample_b"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": workload(), "ms_per_sample": cb["ms_per_sample"], "sample_rows": cb["sample_b"],
                       "steps_requested": args.steps,
                       "note": "reference's jnp path needs JAX (absent): CPU port of it; each timed sample is "
                               f"{cb['sample_b']} of the {B} batch rows and ms_per_step scales it to the whole batch"},
            "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": cb["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), file=real_stdout, flush=True)
    return

  import torch
  import torch.distributed as dist
  from colabfold_kernels import _lib, attention, dispatch, ops
  if not torch.cuda.is_available():
    raise SystemExit("bench.py needs a CUDA device: the library has no CPU path")
  torch.cuda.set_device(local_rank)
  dev = torch.device("cuda", local_rank)
  if world > 1:
    dist.init_process_group("nccl", device_id=dev)
  lib = _lib.load()
  bf = torch.bfloat16
  g = torch.Generator().manual_seed(1000 + rank)
  host = {n: torch.randn(B, S, H, D, generator=g).to(bf).pin_memory() for n in ("q", "k", "v", "do")}
  host["bias"] = torch.randn(H, S, S, generator=g).to(bf).pin_memory()
  mask_bool = torch.rand(B, S, generator=g) < 0.95
  host["mask_bias"] = ((~mask_bool).to(torch.float32) * -1e9).to(bf).reshape(B, 1, 1, S).pin_memory()
  scale = D ** -0.5
  q, k, v, do, bias = (host[n].to(dev) for n in ("q", "k", "v", "do", "bias"))
  kmask = mask_bool.to(dev)

  def barrier():
    if world > 1:
      dist.barrier()
    torch.cuda.synchronize()

  fwd_ms, bwd_ms = [], []

  def step(timed=False):
    if timed:
      e = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
      e[0].record()
    out, lse = ops.attention_fwd(q, k, v, bias, kmask, scale, seq_major=True, want_lse=True)
    if timed:
      e[1].record()
    grads = ops.attention_bwd(q, k, v, bias, kmask, out, do, lse, scale, seq_major=True, want_dbias=True)
    if timed:
      e[2].record()
      return e
    return grads

  for _ in range(max(args.warmup, 3)):
    step()
  barrier()
  sampler = ClockSampler(local_rank)
  if rank == 0:
    sampler.start()
  lib.cfk_launch_count(1)
  t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
  t0.record()
  evs = [step(timed=True) for _ in range(args.steps)]
  t1.record()
  barrier()
  launches = lib.cfk_launch_count(0)
  ms = torch.tensor([t0.elapsed_time(t1)], device=dev)
  if world > 1:
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
  ms_per_step = float(ms) / args.steps
  for e in evs:
    fwd_ms.append(e[0].elapsed_time(e[1]))
    bwd_ms.append(e[1].elapsed_time(e[2]))
  status = ops.device_status()

  # ---- end to end through the public selector API with host buffers ---------------------------------------
  kernel = attention(dispatch(), bf, D, D, layout="seq")
  out_host = {n: torch.empty(B, S, H, D, dtype=bf).pin_memory() for n in ("out", "dq", "dk", "dv")}
  out_host["dbias"] = torch.empty(H, S, S, dtype=bf).pin_memory()

  # The step streams the batch through the device in chunks: while chunk c computes, chunk c + 1 is on its way in and the
  # results of chunk c - 1 are on their way out (three streams, two device slots).  Every chunk is one call of the public
  # selector callable and one backward through it; dBias accumulates over the chunks in the bias leaf's gradient.
  n_chunks = args.e2e_chunks if B % args.e2e_chunks == 0 and B >= 8 * args.e2e_chunks else 1
  bc = B // n_chunks
  s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
  names = ("q", "k", "v", "do", "mask_bias")
  slots = [{n: torch.empty((bc,) + tuple(host[n].shape[1:]), dtype=bf, device=dev) for n in names} for _ in range(2)]
  bias_dev = torch.empty(H, S, S, dtype=bf, device=dev)
  ev_in = [torch.cuda.Event() for _ in range(2)]
  ev_free = [torch.cuda.Event() for _ in range(2)]
  for e in ev_free:
    e.record()

  def e2e_step():
    cur = torch.cuda.current_stream()
    s_in.wait_stream(cur)  # the step before has finished with the bias buffer
    with torch.cuda.stream(s_in):
      bias_dev.copy_(host["bias"], non_blocking=True)
    cur.wait_stream(s_in)
    bias_leaf = bias_dev.detach().requires_grad_(True)
    for c in range(n_chunks):
      sl, rows = c % 2, slice(c * bc, (c + 1) * bc)
      with torch.cuda.stream(s_in):
        s_in.wait_event(ev_free[sl])  # the chunk that used this slot has been computed
        for n in names:
          slots[sl][n].copy_(host[n][rows], non_blocking=True)
        ev_in[sl].record(s_in)
      cur.wait_event(ev_in[sl])
      qc, kc, vc = (slots[sl][n].detach().requires_grad_(True) for n in ("q", "k", "v"))
      o = kernel(qc, kc, vc, slots[sl]["mask_bias"], bias_leaf, scale)
      o.backward(slots[sl]["do"])
      ev_free[sl].record(cur)
      s_out.wait_stream(cur)
      with torch.cuda.stream(s_out):
        for n, t in (("out", o.detach()), ("dq", qc.grad), ("dk", kc.grad), ("dv", vc.grad)):
          out_host[n][rows].copy_(t, non_blocking=True)
          t.record_stream(s_out)
    s_out.wait_stream(cur)
    with torch.cuda.stream(s_out):
      out_host["dbias"].copy_(bias_leaf.grad, non_blocking=True)
      bias_leaf.grad.record_stream(s_out)
    cur.wait_stream(s_out)  # the step ends when its last result is in host memory

  h2d = sum(host[n].numel() * host[n].element_size() for n in ("q", "k", "v", "do", "bias", "mask_bias"))
  d2h = sum(t.numel() * t.element_size() for t in out_host.values())
  e2e_step()
  barrier()
  n_e2e = max(1, min(args.steps, 3))
  t0.record()
  for _ in range(n_e2e):
    e2e_step()
  t1.record()
  barrier()
  e2e_ms = torch.tensor([t0.elapsed_time(t1) / n_e2e], device=dev)
  # the streamed step must give what the resident step gives (forward bit for bit; dk through the same kernels)
  ref_out, ref_lse = ops.attention_fwd(q, k, v, bias, kmask, scale, seq_major=True, want_lse=True)
  ref_dk = ops.attention_bwd(q, k, v, bias, kmask, ref_out, do, ref_lse, scale, seq_major=True, want_dbias=False)[1]
  e2e_ok = bool(torch.equal(out_host["out"].to(dev), ref_out)) and bool(torch.equal(out_host["dk"].to(dev), ref_dk))
  del ref_out, ref_lse, ref_dk
  if world > 1:
    dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
  block_ms = block_f8_ms = block_f8a_ms = block_launch = block_1gpu_ms = block_err = block_nccl_ms = block_exchange = None
  if args.block:
    graph = args.block_graph != 0
    peer = args.peer_exchange != 0
    if world > 1:
      block_exchange = peer_exchange(dev, peer)[1]
      block_err, block_check_res = block_matches_single_gpu(world, rank, dev, peer=peer)
      if rank == 0:  # the same block on this GPU alone: the denominator of the strong-scaling figure
        block_1gpu_ms, _ = evoformer_block_ms(1, 0, dev, graph=graph)
      dist.barrier()
    block_ms, block_launch = evoformer_block_ms(world, rank, dev, graph=graph, peer=peer)
    if world > 1 and peer and peer_exchange(dev)[0] is not None:  # the same block with NCCL's collectives, for comparison
      block_nccl_ms, _ = evoformer_block_ms(world, rank, dev, graph=graph, peer=False)
    block_f8_ms, _ = evoformer_block_ms(world, rank, dev, fp8_trimul=True, graph=graph, peer=peer)
    block_f8a_ms, _ = evoformer_block_ms(world, rank, dev, fp8_trimul=True, fp8_attention=True, graph=graph, peer=peer)
  status = ops.device_status()
  if rank == 0:
    sampler.stop_flag.set()
    sampler.join(timeout=2)

  if rank == 0:
    peak_tf, _, peak_kind = peaks()
    sustained_tf = sustained_peak()
    fwd = sorted(fwd_ms)[len(fwd_ms) // 2]
    bwd = sorted(bwd_ms)[len(bwd_ms) // 2]
    dominant, dom_ms, dom_flops = ("attention_bwd", bwd, 10.0 * B * H * S * S * D) if bwd >= fwd else \
                                  ("attention_fwd", fwd, 4.0 * B * H * S * S * D)
    achieved = dom_flops / (dom_ms * 1e-3) / 1e12
    # DRAM bytes of one launch: the ncu capture of a small batch of the same shape, listed by kernel in the capture
    # table beside the profiles, scaled by batch (every term but the 16.8 MB bias tile grows with it); null without it
    traffic = traffic_src = None
    try:
      cap = json.load(open(os.path.join(ROOT, "profiles", "attention_dram_traffic.json")))[dominant]
      traffic = float(cap["dram_bytes_per_launch"]) * B / float(cap["batch"])
      traffic_src = f"ncu capture of {cap['kernel']} at {cap['capture']}, scaled by batch {B}/{cap['batch']}"
    except Exception:
      pass
    line = {
        "metric": METRIC, "value": flops(B) * world / (ms_per_step * 1e-3) / 1e12, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": workload(), "global_batch": B * world, "parallelism": f"batch-sharded x{world}, no collective",
                   "l2": "inputs (1.1 GB per rank) exceed the 126 MB L2; no flush between steps",
                   "fwd_ms": fwd, "bwd_ms": bwd, "pct_of_peak": 100.0 * flops(B) / (ms_per_step * 1e-3) / 1e12 / peak_tf,
                   "device_status": status,
                   "evoformer_block": None if block_ms is None else {
                       "ms": block_ms, "ms_e4m3_contractions": block_f8_ms, "ms_e4m3_contractions_and_attention": block_f8a_ms, "launch": block_launch, "n_seq": 512, "n_res": 1024, "flop": 6.138e12,
                       "tflops": 6.138e12 / (block_ms * 1e-3) / 1e12,
                       "ms_nccl_collectives": block_nccl_ms, "collectives": block_exchange,
                       "mode": "one GPU" if world == 1 else f"row-sharded over {world} GPUs (strong scaling)"}},
        "e2e": {"value": flops(B) * world / (float(e2e_ms) * 1e-3) / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": float(e2e_ms), "chunks": n_chunks,
                "matches_resident_step": e2e_ok},
        "gpu_launches": int(launches),
        "block_ms": block_ms,
        "block_roofline": None if block_ms is None else {
            "bound": "tensor", "flop": 6.138e12, "achieved": 6.138e12 / (block_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
            "peak": sustained_tf * world, "frac": 6.138e12 / (block_ms * 1e-3) / 1e12 / (sustained_tf * world),
            "peak_source": f"{peak_kind} sustained bf16 x {world} GPUs"},
        "block_speedup_vs_1gpu": None if not block_1gpu_ms else block_1gpu_ms / block_ms,
        "block_ms_1gpu": block_1gpu_ms,
        "block_matches_single_gpu": None if block_err is None else {"max_rel_err": block_err, "ok": block_err <= 2e-2,
                                                                    "n_seq": 64, "n_res": block_check_res},
        "roofline": {"bound": "tensor", "kernel": dominant, "achieved": achieved, "peak": peak_tf, "unit": "TFLOP/s",
                     "frac": achieved / peak_tf, "traffic": traffic, "traffic_unit": "bytes per launch (DRAM read + write)",
                     "traffic_source": traffic_src,
                     "peak_source": f"{peak_kind} burst bf16"},
        "clocks": sampler.summary(),
    }
    if world == 1:  # the CPU arm is reported at N = 1 only
      cb = cpu_arm(3, 1)
      line["cpu_baseline"] = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}
    print(json.dumps(line), file=real_stdout, flush=True)
  if world > 1:
    dist.destroy_process_group()


if __name__ == "__main__":
  main()
