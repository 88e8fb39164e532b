#!/usr/bin/env python
"""Benchmark of the paged-Q8 attention path on B200.

Metric: paged-Q8 attention -- decode HBM GB/s and prefill
TFLOP/s at 32K context, GQA 48/8, head_dim 128.

  step (value, the headline line):  one decode batch of BASELINE config 3 --
      64 sequences, 1 query token each, context lengths ~ U[1K, 32K]
      (seeded), Hq/Hkv = 48/8, bf16 Q, Q8_0 K + fp16 V paged cache
      (block_size 16, shuffled pages) built by the store kernel from
      N(0,1) fp16.  value = algorithmic bytes / time, bytes =
      sum_s L_s*Hkv*(136 + 256) + Q + O + block table.
  prefill (extra key): BASELINE config 4 at 32 768 tokens -- one sequence,
      chunks of 8192 queries against all earlier keys (causal inside the
      chunk), bf16 Q, same cache format.  FLOPs = 4*D*Hq*sum_chunks
      [C*s0 + C(C+1)/2].

Multi-GPU (torchrun, one rank per GPU): the kv heads are split across ranks
as vLLM tensor parallelism does (rank r owns kv heads [r*8/N, (r+1)*8/N) and
their 6 query heads each); total work is fixed, so scaling is "strong".  No
collective touches the data path; NCCL is used only for the start barrier
and the max-over-ranks timing.

`--impl reference` times the CPU restatement of the reference's path
(oracle/, all host threads) on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "gfx906-fa-vllm_b200")
sys.path.insert(0, PKG)

METRIC = "paged-Q8 attn: decode HBM GB/s & prefill TFLOP/s @32K ctx, GQA 48/8 d128"
HQ, HKV, D, BS = 48, 8, 128, 16
RB = D // 32 * 34


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        j = json.load(open(p))
        return float(j["hbm_gbs"]), float(j["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def tensor_peak(clocks, burst, burst_kind):
    """Denominator for a tensor-bound region: the sustained (power-capped)
    GEMM rate when the region's clocks sat below maximum under sw_power_cap,
    else the burst rate."""
    sus, sus_kind = sustained_tflops()
    capped = (clocks.get("sm_mhz") and clocks.get("sm_max_mhz") and "sw_power_cap" in clocks.get("reasons", [])
              and clocks["sm_mhz"] < 0.97 * clocks["sm_max_mhz"])
    if capped:
        return sus, f"{sus_kind} bf16 sustained (clocks power-capped during the region)"
    return burst, f"{burst_kind} bf16 burst (clocks at maximum during the region)"


def sustained_tflops():
    """The measured bf16 GEMM rate under the power cap (seconds-long loop), the
    denominator for a kernel timed inside a long dense step; fallback 1400."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        j = json.load(open(p))
        if "bf16_tflops_sustained" in j:
            return float(j["bf16_tflops_sustained"]), "measured"
    return 1400.0, "fallback"


def config3_lens(seed=3):
    rng = np.random.default_rng(seed)
    return rng.integers(1024, 32769, size=64).astype(np.int64)


def config5_batch(seed=5):
    """Mixed serving batch (config 5): 32 decode sequences with contexts
    U[16K, 100K], each verifying 4 speculative tokens (causal within the 4),
    plus 2 prefill chunks of 4096 tokens at offsets 0 and 24K.  Returns
    (kv_lens, n_q) per sequence."""
    rng = np.random.default_rng(seed)
    dec = rng.integers(16384, 100001, size=32).astype(np.int64)
    kv = np.concatenate([dec, [4096, 24576 + 4096]])
    nq = np.concatenate([np.full(32, 4), [4096, 4096]])
    return kv, nq


def config5_work(kv, nq, hkv, hq, v_row):
    """Algorithmic bytes (every visible K/V row once, Q in, O out, block
    table) and FLOPs (4*D per visible (query head, key) pair, causal)."""
    byt = int(np.sum(kv)) * hkv * (RB + v_row) + int(np.sum(nq)) * hq * D * 4
    byt += int(sum((int(L) + BS - 1) // BS for L in kv)) * 4
    pairs = sum(int(n) * int(L) - int(n) * (int(n) - 1) // 2 for L, n in zip(kv, nq))
    return byt, 4 * D * hq * pairs


# ---------------------------------------------------------------------------
# clocks sampling
# ---------------------------------------------------------------------------
class ClockSampler:
    """Samples SM clocks and throttle reasons while the timed region runs:
    NVML (opened once, on the calling thread) polled every 5 ms from a
    background thread and, through sample_until, from the main thread while
    the queued steps run; nvidia-smi every 200 ms when NVML is unavailable."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")
    REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
               ("sw_power_cap", 0x4))

    def __init__(self, index):
        self.index = index
        self.rows = []           # (sm_mhz, max_mhz, set of active reason names)
        self._stop = threading.Event()
        self._t = None
        self._nv = self._h = None
        self._max = None
        try:
            import pynvml as nv
            nv.nvmlInit()
            self._h = self._handle(nv)
            self._max = float(nv.nvmlDeviceGetMaxClockInfo(self._h, nv.NVML_CLOCK_SM))
            self._get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                nv.nvmlDeviceGetCurrentClocksThrottleReasons
            self._nv = nv
        except Exception:
            self._nv = None

    def _handle(self, nv):
        """NVML handle of CUDA device `index` (matched by PCI bus id: NVML
        and CUDA may number the GPUs differently)."""
        try:
            import torch
            pr = torch.cuda.get_device_properties(self.index)
            bus = "%08x:%02x:%02x.0" % (pr.pci_domain_id, pr.pci_bus_id, pr.pci_device_id)
            return nv.nvmlDeviceGetHandleByPciBusId(bus.encode())
        except Exception:
            return nv.nvmlDeviceGetHandleByIndex(self.index)

    def _sample_nvml(self):
        try:
            nv = self._nv
            bits = int(self._get_reasons(self._h))
            self.rows.append((float(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)), self._max,
                              {n for n, b in self.REASONS if bits & b}))
        except Exception:
            pass

    def _run_smi(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                                      "--format=csv,noheader,nounits"], capture_output=True, text=True,
                                     timeout=5).stdout.strip()
                r = [x.strip() for x in out.split(",")] if out else []
                if len(r) >= 8 and r[1].replace(".", "").isdigit():
                    names = [n for n, _ in self.REASONS]
                    self.rows.append((float(r[1]), float(r[2]) if r[2].replace(".", "").isdigit() else None,
                                      {names[i] for i in range(4) if r[4 + i] == "Active"}))
            except Exception:
                pass
            self._stop.wait(0.2)

    def _run(self):
        if self._nv is None:
            self._run_smi()
            return
        while not self._stop.is_set():
            self._sample_nvml()
            self._stop.wait(0.005)

    def __enter__(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        self._t.join(timeout=10)

    def sample_until(self, event):
        """Poll the clocks from this thread until `event` completes (the
        timed region is already queued), so that a region of a few
        milliseconds still gets samples."""
        if self._nv is None:
            return
        while not event.query():
            self._sample_nvml()
            time.sleep(0.0002)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [r[0] for r in self.rows]
        mx = [r[1] for r in self.rows if r[1]]
        reasons = sorted(set().union(*[r[2] for r in self.rows]))
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


# ---------------------------------------------------------------------------
# workload construction (on the GPU)
# ---------------------------------------------------------------------------
def build_cache(lens, hkv, seed, device, v_fmt="fp16"):
    """Paged Q8_0 K + V cache for sequences of `lens` tokens, shuffled pages,
    filled by the fused store kernel from N(0,1) fp16 K/V.  v_fmt: "fp16",
    "q8_0" (page-transposed Q8_0 records) -- both in the backend's vLLM-shaped
    allocation -- or "q8_0rows" (Q8_0 token rows in separate tensors)."""
    import torch
    import gfx906_fa
    g = torch.Generator(device=device).manual_seed(seed)
    npg = [(int(L) + BS - 1) // BS for L in lens]
    NB = sum(npg) + 64
    perm = torch.randperm(NB, generator=g, device=device).to(torch.int32)
    MB = max(npg)
    bt = torch.full((len(lens), MB), -1, dtype=torch.int32, device=device)
    c = 0
    for b, n in enumerate(npg):
        bt[b, :n] = perm[c:c + n]
        c += n
    if v_fmt == "q8_0rows":
        k_cache = torch.zeros((NB, BS, hkv, RB), dtype=torch.uint8, device=device)
        v_cache = torch.zeros((NB, BS, hkv, RB), dtype=torch.uint8, device=device)
    else:
        # the backend's own layout: one vLLM allocation [NB, 2, bs, Hkv, D] with
        # Q8_0 K rows (and page-transposed Q8_0 V records) at each page's start
        from gfx906_fa_paged import kv_cache_views
        kv = torch.zeros((NB, 2, BS, hkv, D), dtype=torch.float16, device=device)
        k_cache, v_cache = kv_cache_views(kv, v_fmt)
    chunk = 1 << 16
    for b, L in enumerate(lens):
        for t0 in range(0, int(L), chunk):
            n = min(chunk, int(L) - t0)
            tpos = torch.arange(t0, t0 + n, device=device)
            slots = bt[b, tpos // BS].to(torch.int64) * BS + tpos % BS
            k = torch.randn((n, hkv, D), generator=g, device=device, dtype=torch.float16)
            v = torch.randn((n, hkv, D), generator=g, device=device, dtype=torch.float16)
            gfx906_fa.store_kv(k, v, slots, k_cache, v_cache, {"q8_0": 3, "q8_0rows": 2}.get(v_fmt, 1))
    return k_cache, v_cache, bt


# DRAM bytes (read + write) of one decode_kernel launch per algorithmic byte,
# from ncu --metrics dram__bytes_read.sum,dram__bytes_write.sum on the first
# 16 sequences of config 3: page-transposed Q8_0 V read 462.75 MB and wrote
# 21.81 MB against 462.36 MB of algorithmic bytes; fp16 V read 666.97 MB and
# wrote 20.39 MB against 666.14 MB.  The writes are the split-K partials.
DECODE_TRAFFIC_RATIO = {"q8_0": (462.63 + 5.18) / 462.36, "fp16": (666.54 + 5.09) / 666.14}


# DRAM bytes (read + write) per FLOP of prefill_kernel, from one ncu capture
# (dram__bytes_read.sum + dram__bytes_write.sum) of the last 8192-query chunk
# of the 32K prefill: 1.389 GB + 0.107 GB for 5.773 TFLOP.
PREFILL_TRAFFIC_PER_FLOP = (1.384802e9 + 0.109156e9) / 5.77253670912e12
PREFILL_TRAFFIC_NOTE = ("ncu dram read+write of prefill_kernel on the chunk at offset 24576 of config 4 "
                        "(profiles/prefill_kernel_config4_chunk24k.md) per algorithmic FLOP, scaled to this "
                        "workload's FLOPs")


def decode_bytes(lens, hkv, hq, v_row=256):
    kv = int(np.sum(lens)) * hkv * (RB + v_row)
    q = len(lens) * hq * D * 2
    o = len(lens) * hq * D * 2
    bt = int(sum((int(L) + BS - 1) // BS for L in lens)) * 4
    return kv + q + o + bt


def prefill_flops(n_tokens, chunk, hq):
    f = 0
    for s0 in range(0, n_tokens, chunk):
        C = min(chunk, n_tokens - s0)
        f += C * s0 + C * (C + 1) // 2
    return 4 * D * hq * f


# ---------------------------------------------------------------------------
# CPU baseline (oracle restatement, test infrastructure)
# ---------------------------------------------------------------------------
def cpu_baseline(seconds_target=10.0, threads=None, v_fmt="q8_0"):
    """Oracle attention (fp32 dequant + softmax, double accumulation) on the
    host cores over a bounded sample of config 3: the first sequences until
    ~seconds_target of work.  Returns GB/s in the decode metric's bytes.
    v_fmt "q8_0": page-transposed Q8_0 V records; else fp16 V rows."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    threads = threads or os.cpu_count()
    lens = config3_lens()
    rng = np.random.default_rng(0)
    done_bytes, elapsed, nseq = 0, 0.0, 0
    for L in lens:
        L = int(L)
        nb = (L + BS - 1) // BS
        kq = rng.integers(0, 256, size=(nb, BS, HKV, RB), dtype=np.uint8)
        kq[..., 0::34] = 0x00          # small scales keep the values finite
        kq[..., 1::34] = 0x20
        q = rng.standard_normal((1, HQ, D)).astype(np.float32)
        bt = np.arange(nb, dtype=np.int32).reshape(1, nb)
        if v_fmt == "q8_0":
            vc = rng.integers(0, 256, size=(nb, HKV, BS * RB), dtype=np.uint8)
            vc[..., :2 * (D // 32) * BS:2] = 0x00    # fp16 scales 0x2000: small, finite
            vc[..., 1:2 * (D // 32) * BS:2] = 0x20
            kw = dict(v_fmt="q8t", v_strides=(HKV * BS * RB, 0, BS * RB))
            v_row = RB
        else:
            vc = rng.standard_normal((nb, BS, HKV, D)).astype(np.float16)
            kw, v_row = {}, 2 * D
        t0 = time.perf_counter()
        O.attention_paged(q, None, np.array([0]), np.array([1]), kq, vc, bt, np.array([L]), 1 / np.sqrt(D),
                          HKV, nthreads=threads, **kw)
        elapsed += time.perf_counter() - t0
        done_bytes += decode_bytes([L], HKV, HQ, v_row)
        nseq += 1
        if elapsed > seconds_target:
            break
    return {"value": done_bytes / elapsed / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{nseq} of the 64 config-3 sequences ({done_bytes / 1e9:.2f} GB of algorithmic bytes), "
                      f"oracle/q8_oracle.c attention, OpenMP"}, elapsed


def cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def torch_cpu_baseline(seconds_target=10.0, v_fmt="q8_0"):
    """The reference's own torch CPU pipeline (restated in
    oracle/torch_path.py: page gather by fancy indexing, dequantize_q8_0,
    repeat_interleave for GQA, torch SDPA in fp32) over the config-3
    sequences until ~seconds_target of work, with torch's full host thread
    pool.  Returns GB/s in the decode metric's bytes."""
    import torch
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import torch_path as TP
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    lens = config3_lens()
    g = torch.Generator().manual_seed(0)
    done_bytes, elapsed, nseq = 0, 0.0, 0
    for L in lens:
        L = int(L)
        nb = (L + BS - 1) // BS
        kq = torch.randint(0, 256, (nb, BS, HKV, RB), generator=g, dtype=torch.uint8)
        kq.view(-1, 34)[:, 0] = 0x00              # fp16 scale 0x2000: small, finite
        kq.view(-1, 34)[:, 1] = 0x20
        if v_fmt.startswith("q8_0"):
            vc = kq.clone()
            v_row = RB
        else:
            vc = torch.randn((nb, BS, HKV, D), generator=g).half()
            v_row = 2 * D
        q = torch.randn((1, HQ, D), generator=g).to(torch.bfloat16)
        bt = torch.arange(nb, dtype=torch.int32).view(1, nb)
        t0 = time.perf_counter()
        TP.attention_varlen(q, kq, vc, bt, [L], [1], 1 / np.sqrt(D), v_q8=v_fmt.startswith("q8_0"))
        elapsed += time.perf_counter() - t0
        done_bytes += decode_bytes([L], HKV, HQ, v_row)
        nseq += 1
        if elapsed > seconds_target:
            break
    return {"value": done_bytes / elapsed / 1e9, "unit": "GB/s", "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": f"{nseq} of the 64 config-3 sequences ({done_bytes / 1e9:.2f} GB of algorithmic bytes) "
                      "through the reference's torch CPU pipeline (gather by fancy indexing, dequantize_q8_0, "
                      "repeat_interleave, F.scaled_dot_product_attention fp32; restated in oracle/torch_path.py)",
            "host": {"cpu_model": cpu_model(), "os_cpu_count": os.cpu_count(),
                     "torch_threads": torch.get_num_threads()}}, elapsed


# ---------------------------------------------------------------------------
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--v-fmt", default="q8_0", choices=["fp16", "q8_0", "q8_0rows"],
                    help="V cache format: q8_0 = page-transposed Q8_0 (config 3's Q8_0 K/V cache)")
    ap.add_argument("--no-fp16v", action="store_true", help="skip the extra fp16-V decode measurement")
    ap.add_argument("--decode-seqs", type=int, default=64,
                    help="first N sequences of config 3 (profiling uses a smaller case)")
    ap.add_argument("--prefill-tokens", type=int, default=32768)
    ap.add_argument("--prefill-long", default="65536,130000,133120",
                    help="extra config-4 context lengths timed after the headline 32K (comma list, '' for none)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-mixed", action="store_true", help="skip the config-5 mixed-batch measurement")
    ap.add_argument("--no-kv", action="store_true", help="skip the config-2 KV store + gather measurement")
    ap.add_argument("--tp-emulate", type=int, default=1,
                    help="single GPU: run rank 0's kv-head share of N-way tensor parallelism (profiling)")
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank != 0:
            return
        budget = max(3.0, min(20.0, 2.0 * args.steps))
        res, el = torch_cpu_baseline(seconds_target=budget, v_fmt=args.v_fmt)
        res_c, _ = cpu_baseline(seconds_target=budget / 2, v_fmt=args.v_fmt)
        line = {"metric": METRIC, "value": res["value"], "unit": "GB/s", "n_gpus": args.gpus,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": None, "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
                "impl": "reference",
                "config": {"workload": "config3 decode (64 seqs, L~U[1K,32K], GQA 48/8, d128, Q8_0 K, "
                                       + ("Q8_0 V" if args.v_fmt.startswith("q8_0") else "fp16 V") + ")",
                           "sample": res["sample"]},
                "cpu_baseline": res,
                "cpu_baseline_c_oracle": res_c,
                "e2e": {"value": res["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    import torch
    import gfx906_fa
    from gfx906_fa_paged import forward_paged

    dist = None
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl")
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    from gfx906_fa_shard import head_shard
    # vLLM-style tensor-parallel head groups; --tp-emulate N times rank 0's
    # share of N-way tensor parallelism on this one GPU (profiling aid)
    shard = head_shard(HQ, HKV, world, rank) if args.tp_emulate <= 1 else head_shard(HQ, HKV, args.tp_emulate, 0)
    hkv, hq = shard.num_heads_kv, shard.num_heads_q

    # ---------------- decode workload (config 3) ----------------------------
    lens = config3_lens()[:args.decode_seqs]
    B = len(lens)
    k_cache, v_cache, bt = build_cache(lens, hkv, seed=1000 + rank, device=device, v_fmt=args.v_fmt)
    sl = torch.tensor(lens, dtype=torch.int32, device=device)
    cu = torch.arange(B + 1, dtype=torch.int32, device=device)
    gq = torch.Generator(device=device).manual_seed(7 + rank)
    q = torch.randn((B, hq, D), generator=gq, device=device).to(torch.bfloat16)
    out = torch.empty_like(q)
    ones = [1] * B
    lens_l = [int(x) for x in lens]
    max_l = int(lens.max())
    scale = 1.0 / np.sqrt(D)

    def decode_step():
        gfx906_fa.paged_attention(q, k_cache, v_cache, bt, sl, cu, 1, max_l, scale, out=out,
                                  query_lens_host=ones, seq_lens_host=lens_l)

    def barrier():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
            torch.cuda.synchronize()

    def max_over_ranks(x):
        if dist is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(max(3, args.warmup)):
        decode_step()
    barrier()
    sampler = ClockSampler(local_rank)
    with sampler:
        barrier()
        t_start = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        t_start.record()
        for i in range(args.steps):
            decode_step()
        t_end.record()
        sampler.sample_until(t_end)          # clocks while the queued steps run
        barrier()
    total_ms = max_over_ranks(t_start.elapsed_time(t_end))
    # one step = one paged_attention call = the decode kernel and its split-K
    # merge, back to back on this stream (no events between them, so the
    # launches overlap as they do in serving)
    per_launch_ms = t_start.elapsed_time(t_end) / args.steps
    v_row = RB if args.v_fmt.startswith("q8_0") else 2 * D
    bytes_rank = decode_bytes(lens, hkv, hq, v_row)
    bytes_all = bytes_rank * world
    ms_per_step = total_ms / args.steps
    value = bytes_all / (ms_per_step * 1e-3) / 1e9
    hbm_peak, tf_peak, peak_kind = load_peaks()
    achieved = bytes_rank / (per_launch_ms * 1e-3) / 1e9

    # ---------------- end to end: host buffers through forward_paged --------
    # Two buffer sets, double-buffered as a serving loop would run it: step
    # i+1's inputs go up on a copy stream and step i-1's output comes down
    # on another while step i's kernels run.  Every step still copies its
    # inputs from pinned host memory and reads its output back, all inside
    # the timed region (the end event waits for the last download).
    NBUF = 2
    q_host = [q.cpu().pin_memory() for _ in range(NBUF)]
    out_host = [torch.empty(out.shape, dtype=out.dtype).pin_memory() for _ in range(NBUF)]
    sl_host = [sl.cpu().pin_memory() for _ in range(NBUF)]
    cu_host = [cu.cpu().pin_memory() for _ in range(NBUF)]
    bt_host = [bt.cpu().pin_memory() for _ in range(NBUF)]
    q_dev = [torch.empty_like(q) for _ in range(NBUF)]
    sl_dev = [torch.empty_like(sl) for _ in range(NBUF)]
    cu_dev = [torch.empty_like(cu) for _ in range(NBUF)]
    bt_dev = [torch.empty_like(bt) for _ in range(NBUF)]
    o_dev = [torch.empty_like(out) for _ in range(NBUF)]
    main = torch.cuda.current_stream()
    up, down = torch.cuda.Stream(), torch.cuda.Stream()
    ev_in = [torch.cuda.Event() for _ in range(NBUF)]      # inputs of buffer b uploaded
    ev_done = [torch.cuda.Event() for _ in range(NBUF)]    # kernels of buffer b finished
    ev_out = [torch.cuda.Event() for _ in range(NBUF)]     # output of buffer b downloaded
    for b in range(NBUF):
        ev_done[b].record(main)
        ev_out[b].record(main)

    def e2e_step(i):
        b = i % NBUF
        with torch.cuda.stream(up):
            up.wait_event(ev_done[b])                       # step i-2 no longer reads these
            q_dev[b].copy_(q_host[b], non_blocking=True)
            sl_dev[b].copy_(sl_host[b], non_blocking=True)
            cu_dev[b].copy_(cu_host[b], non_blocking=True)
            bt_dev[b].copy_(bt_host[b], non_blocking=True)
            ev_in[b].record(up)
        main.wait_event(ev_in[b])
        main.wait_event(ev_out[b])                          # step i-2's output is down
        forward_paged(q_dev[b], None, v_cache, bt_dev[b], sl_dev[b], cu_dev[b], 1, max_l, scale=scale,
                      key_cache_q8=k_cache, out=o_dev[b], query_lens_host=ones, seq_lens_host=lens_l)
        ev_done[b].record(main)
        with torch.cuda.stream(down):
            down.wait_event(ev_done[b])
            out_host[b].copy_(o_dev[b], non_blocking=True)
            ev_out[b].record(down)

    for i in range(3):
        e2e_step(i)
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(main)
    for i in range(args.steps):
        e2e_step(i)
    for b in range(NBUF):
        main.wait_event(ev_out[b])
    e1.record(main)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1)) / args.steps
    h2d = q_host[0].numel() * 2 + sl_host[0].numel() * 4 + cu_host[0].numel() * 4 + bt_host[0].numel() * 4
    d2h = out_host[0].numel() * 2
    e2e_value = bytes_all / (e2e_ms * 1e-3) / 1e9

    # ---------------- same decode with fp16 V (reference parity mode) -------
    fp16v = None
    if args.v_fmt != "fp16" and not args.no_fp16v:
        v_cache = None
        torch.cuda.empty_cache()
        k2, v2, bt2 = build_cache(lens, hkv, seed=3000 + rank, device=device, v_fmt="fp16")

        def decode_fp16v():
            gfx906_fa.paged_attention(q, k2, v2, bt2, sl, cu, 1, max_l, scale, out=out,
                                      query_lens_host=ones, seq_lens_host=lens_l)

        for _ in range(max(3, args.warmup)):
            decode_fp16v()
        barrier()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record()
        for _ in range(args.steps):
            decode_fp16v()
        f1.record()
        barrier()
        fms = max_over_ranks(f0.elapsed_time(f1)) / args.steps
        fb = decode_bytes(lens, hkv, hq, 2 * D)
        fp16v = {"value": fb * world / (fms * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": fms,
                 "frac_of_hbm": fb / (fms * 1e-3) / 1e9 / hbm_peak,
                 "workload": "config3 decode with fp16 V rows (the reference's V format)"}
        del k2, v2, bt2
        torch.cuda.empty_cache()

    # ---------------- prefill (config 4 at 32K, 64K, 130K) ---------------------
    def prefill_run(N, C=8192, psteps=3):
        """One sequence of N tokens prefilled in 8192-query chunks, each chunk
        one paged_attention call against every earlier key (causal inside the
        chunk).  Returns (ms per prefill, staging workspace bytes of the last
        chunk)."""
        kc, vc, btp = build_cache([N], hkv, seed=2000 + rank, device=device, v_fmt=args.v_fmt)
        qp = torch.randn((N, hq, D), generator=gq, device=device).to(torch.bfloat16)
        op = torch.empty_like(qp)
        chunks = []
        for s0 in range(0, N, C):
            n = min(C, N - s0)
            chunks.append((s0, n, torch.tensor([s0 + n], dtype=torch.int32, device=device),
                           torch.tensor([0, n], dtype=torch.int32, device=device)))

        def prefill_step():
            for s0, n, slc, cuc in chunks:
                gfx906_fa.paged_attention(qp[s0:s0 + n], kc, vc, btp, slc, cuc, n, s0 + n, scale,
                                          out=op[s0:s0 + n], query_lens_host=[n], seq_lens_host=[s0 + n])

        for _ in range(max(3, args.warmup // 2)):
            prefill_step()
        barrier()
        p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        psampler = ClockSampler(local_rank)
        with psampler:
            p0.record()
            for _ in range(psteps):
                prefill_step()
            p1.record()
            psampler.sample_until(p1)
            barrier()
        pms = max_over_ranks(p0.elapsed_time(p1)) / psteps
        prefill_clocks.append(psampler.summary())
        # staging: fp16 Q rows (row tiles padded to pairs), K rows and V^T tiles of every visible key
        s0, n = chunks[-1][0], chunks[-1][1]
        rt = 2 * ((n * (hq // hkv) + 255) // 256)
        kt = (s0 + n + 127) // 128
        ws = hkv * (rt + 2 * kt) * 128 * D * 2
        del kc, vc, btp, qp, op
        torch.cuda.empty_cache()
        return pms, ws, len(chunks)

    prefill = None
    prefill_clocks = []
    if not args.no_prefill:
        del k_cache, v_cache
        torch.cuda.empty_cache()
        N = args.prefill_tokens
        pms, ws, nch = prefill_run(N, psteps=max(3, args.steps // 4))
        fl_all = prefill_flops(N, 8192, HQ)
        ach = fl_all / world / (pms * 1e-3) / 1e12
        # back-to-back prefills of tens to hundreds of milliseconds of dense
        # tensor work can settle under the 1 kW cap: the denominator follows
        # the clocks seen during the region (sustained rate when power-capped,
        # else burst)
        pc = prefill_clocks[-1]
        tf_den, den_kind = tensor_peak(pc, tf_peak, peak_kind)
        prefill = {"value": fl_all / (pms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": pms,
                   "workload": f"config4: 1 seq x {N} tokens, 8192-query chunks, causal, GQA 48/8, "
                               f"{'Q8_0' if args.v_fmt.startswith('q8_0') else 'fp16'} V",
                   "workspace_bytes": ws, "clocks": pc,
                   "roofline": {"bound": "tensor", "achieved": ach, "peak": tf_den, "unit": "TFLOP/s",
                                "frac": ach / tf_den, "peak_kind": den_kind,
                                "frac_of_burst": ach / tf_peak, "burst_peak": tf_peak,
                                "traffic": (PREFILL_TRAFFIC_PER_FLOP * fl_all / world
                                            if PREFILL_TRAFFIC_PER_FLOP else None),
                                "traffic_note": PREFILL_TRAFFIC_NOTE},
                   "gpu_launches_per_step": 3 * nch}
        longer = []
        for NL in [int(x) for x in args.prefill_long.split(",") if x.strip()]:
            lms, lws, _ = prefill_run(NL, psteps=2)
            fl = prefill_flops(NL, 8192, HQ)
            lden, lkind = tensor_peak(prefill_clocks[-1], tf_peak, peak_kind)
            longer.append({"tokens": NL, "value": fl / (lms * 1e-3) / 1e12, "unit": "TFLOP/s",
                           "ms_per_step": lms, "tflop": fl / 1e12, "workspace_bytes": lws,
                           "frac": fl / world / (lms * 1e-3) / 1e12 / lden, "peak_kind": lkind,
                           "frac_of_burst": fl / world / (lms * 1e-3) / 1e12 / tf_peak,
                           "clocks": prefill_clocks[-1]})
        if longer:
            prefill["longer_contexts"] = longer

    # ---------------- mixed serving batch (config 5) -------------------------
    mixed = None
    if not args.no_mixed:
        torch.cuda.empty_cache()
        kv5, nq5 = config5_batch()
        k5, v5, bt5 = build_cache(kv5, hkv, seed=4000 + rank, device=device, v_fmt=args.v_fmt)
        T5 = int(np.sum(nq5))
        q5 = torch.randn((T5, hq, D), generator=gq, device=device).to(torch.bfloat16)
        o5 = torch.empty_like(q5)
        sl5 = torch.tensor(kv5, dtype=torch.int32, device=device)
        cu5 = torch.tensor(np.concatenate([[0], np.cumsum(nq5)]), dtype=torch.int32, device=device)
        nq5_l, kv5_l = [int(x) for x in nq5], [int(x) for x in kv5]

        def mixed_step():
            gfx906_fa.paged_attention(q5, k5, v5, bt5, sl5, cu5, max(nq5_l), max(kv5_l), scale, out=o5,
                                      query_lens_host=nq5_l, seq_lens_host=kv5_l)

        for _ in range(max(3, args.warmup)):
            mixed_step()
        barrier()
        m0, m1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        msteps = max(3, args.steps // 2)
        m0.record()
        for _ in range(msteps):
            mixed_step()
        m1.record()
        barrier()
        mms = max_over_ranks(m0.elapsed_time(m1)) / msteps
        v_row5 = RB if args.v_fmt.startswith("q8_0") else 2 * D
        b5, f5 = config5_work(kv5, nq5, hkv, hq, v_row5)
        t_lb = b5 / (hbm_peak * 1e9) + f5 / (tf_peak * 1e12)
        mixed = {"value": T5 / (mms * 1e-3), "unit": "query tokens/s (all heads)", "ms_per_step": mms,
                 "workload": "config5: 32 decode seqs x 4 speculative tokens (ctx U[16K,100K]) + 2 prefill "
                             "chunks of 4096 at offsets 0 and 24K, one paged_attention call",
                 "bytes_per_gpu": b5, "flops_per_gpu": f5,
                 "roofline": {"bound": "hbm+tensor (serial sum)", "lower_bound_ms": t_lb * 1e3,
                              "frac": t_lb / (mms * 1e-3)}}
        del k5, v5, bt5, q5, o5
        torch.cuda.empty_cache()

    # ---------------- config 2: Q8_0 KV store + paged gather ----------------
    kvio = None
    if not args.no_kv:
        torch.cuda.empty_cache()
        S2, L2, NB2 = 16, 4096, 70000
        T2 = S2 * L2
        g2 = torch.Generator(device=device).manual_seed(6 + rank)
        pool = torch.randperm(NB2, generator=g2, device=device).to(torch.int32)
        bt2 = pool[:S2 * (L2 // BS)].view(S2, L2 // BS).contiguous()
        tpos = torch.arange(L2, device=device)
        slots2 = (bt2[:, tpos // BS].to(torch.int64) * BS + tpos % BS).reshape(-1)
        def outl(x):   # 1% of the elements scaled x8
            m = torch.rand(x.shape, generator=g2, device=device) < 0.01
            return torch.where(m, x * 8, x)
        key2 = outl(torch.randn((T2, hkv, D), generator=g2, device=device, dtype=torch.float16))
        val2 = outl(torch.randn((T2, hkv, D), generator=g2, device=device, dtype=torch.float16))
        # the reference's layout for this path: a contiguous Q8_0 K cache beside the fp16 V cache
        k2v = torch.zeros((NB2, BS, hkv, RB), dtype=torch.uint8, device=device)
        v2v = torch.zeros((NB2, BS, hkv, D), dtype=torch.float16, device=device)
        sl2 = torch.full((S2,), L2, dtype=torch.int32, device=device)
        kout = torch.empty((S2, hkv, L2, RB), dtype=torch.uint8, device=device)
        vout = torch.empty((S2, hkv, L2, D), dtype=torch.float16, device=device)

        def timed(fn, n):
            for _ in range(3):
                fn()
            barrier()
            a, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for _ in range(n):
                fn()
            b_.record()
            barrier()
            return max_over_ranks(a.elapsed_time(b_)) / n

        st_ms = timed(lambda: gfx906_fa.store_kv(key2, val2, slots2, k2v, v2v, 1), max(5, args.steps))
        ga_ms = timed(lambda: gfx906_fa.gather_paged_kv_q8(k2v, v2v, bt2, sl2, L2, k_out=kout, v_out=vout),
                      max(5, args.steps))
        st_b = T2 * hkv * (2 * D * 2 + RB + 2 * D) + T2 * 8       # K, V in; Q8_0 K, V out; slots
        ga_b = 2 * T2 * hkv * (RB + 2 * D) + S2 * (L2 // BS) * 4  # pages in, dense rows out; block table
        kvio = {"workload": "config2: 16 seqs x 4096 tokens, 8 kv heads (per GPU share), d128, block 16, "
                            "fp16 K/V N(0,1) with 1% x8 outliers, pages drawn from a 70K-page pool",
                "kv_store": {"value": st_b * world / (st_ms * 1e-3) / 1e9, "unit": "GB/s", "ms": st_ms,
                             "frac_of_hbm": st_b / (st_ms * 1e-3) / 1e9 / hbm_peak,
                             "op": "store_kv (K -> Q8_0, V copied), fused"},
                "gather": {"value": ga_b * world / (ga_ms * 1e-3) / 1e9, "unit": "GB/s", "ms": ga_ms,
                           "frac_of_hbm": ga_b / (ga_ms * 1e-3) / 1e9 / hbm_peak,
                           "op": "gather_paged_kv_q8 (Q8_0 K + fp16 V pages -> dense BHSD)"}}
        del k2v, v2v, key2, val2, kout, vout
        torch.cuda.empty_cache()

    cpu = cpu_c = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu, _ = torch_cpu_baseline(seconds_target=10.0, v_fmt=args.v_fmt)
        cpu_c, _ = cpu_baseline(seconds_target=5.0, v_fmt=args.v_fmt)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16 Q / q8_0 K / "
            + {"q8_0": "q8_0 (page-transposed)", "q8_0rows": "q8_0 rows"}.get(args.v_fmt, "fp16")
            + " V, fp32 accumulate",
            "data": "synthetic",
            "config": {"workload": f"config3 decode: {B} seqs x 1 query, L~U[1K,32K] seed 3, GQA 48/8, d128, "
                                   "block 16, shuffled pages",
                       "kv_heads_per_gpu": hkv, "parallelism": f"kv-head groups x{world}",
                       "l2": "inputs (%.2f GB per GPU) larger than L2, no flush" % (bytes_rank / 1e9)},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                         "frac": achieved / hbm_peak,
                         "traffic": (bytes_rank * DECODE_TRAFFIC_RATIO[args.v_fmt]
                                     if args.v_fmt in DECODE_TRAFFIC_RATIO else None),
                         "traffic_note": "ncu dram read+write of decode_kernel on the 16-sequence prefix of "
                                         "this workload, scaled by the algorithmic bytes",
                         "peak_kind": f"{peak_kind} copy bandwidth"},
            "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "path": "gfx906_fa_paged.forward_paged (reference plugin API), pinned host Q / lengths / block table in, O out, double-buffered (uploads and downloads on copy streams overlap the neighbouring steps' kernels)"},
            "gpu_launches": 2 * args.steps,          # decode_kernel + decode_combine_kernel per step
            "clocks": sampler.summary(),
        }
        if fp16v:
            line["decode_fp16_v"] = fp16v
        if mixed:
            line["mixed_config5"] = mixed
        if kvio:
            line["kv_store_gather_config2"] = kvio
        if prefill:
            line["prefill"] = prefill
        if cpu:
            line["cpu_baseline"] = cpu
        if cpu_c:
            line["cpu_baseline_c_oracle"] = cpu_c
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
