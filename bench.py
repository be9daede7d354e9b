"""Benchmark of one absorbed-MLA QCAU decode layer step (B=128, ctx 32K).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    (N > 1: python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N)

Workload (the decode configuration the metric is quoted on): batch 128
sequences, one new token each, 128 heads split evenly across the N ranks,
32768 cached tokens per sequence in a paged bf16 latent cache (page 64,
65,536 physical pages of [64, 576], block tables a random permutation), FP8
wq_b [128*192, 1536] / wkv_b [128*256, 512] / wo [7168, 16384] with fp32
128x128 block scales, all-reduce of the bf16 [128, 7168] output over NCCL.
Synthetic seeded data (no checkpoint or dataset): q_lora ~N(0,1) RMS-normalised,
weights ~N(0, 0.02), cache rows ~N(0,1) RMS-normalised.

One step = the whole layer for all 128 tokens.  value = 128 * K / (max over
ranks of the device time of K steps).  The 4.83 GB cache is far larger than
L2 (126 MB), so no L2 flush is needed between steps.
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
import torch.distributed as dist

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "deepseek-v4-flash_b200"))

BATCH, HEADS, CTX, PAGE = 128, 128, 32768, 64
DC, DIM, WIDTH = 1536, 7168, 576
METRIC = "QCAU layer decode tok/s (B=128, ctx 32K)"
MEASURED = REPO / "MEASURED_PEAKS.json"


def peaks():
    try:
        p = json.loads(MEASURED.read_text())
        return p["hbm_gbs"], p["bf16_tflops"], "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.gpu)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.reader = threading.Thread(target=self._read, daemon=True)
            self.reader.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons, power = [], [], set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        under_load = [s for s, p in zip(sm, power) if p > 0.3 * max(power)] or sm
        return {"sm_mhz": statistics.median(under_load), "sm_max_mhz": max(mx),
                "reasons": sorted(reasons), "samples": len(sm)}


SAMPLE_HEADS = 8  # heads of one decode token each CPU thread runs per step


def cpu_reference(steps: int, warmup: int, threads: int):
    """The reference's qcau_c C++ (oracle/_ref) on this host.  One step = every
    thread runs a head-shard sample of one decode token of the same workload:
    SAMPLE_HEADS of the 128 heads (q-up rows, attention heads and o-proj input
    columns of that shard), i.e. SAMPLE_HEADS/128 of the token's work, so a
    step takes seconds instead of half a minute.  The inputs are generated
    before the clock starts; only quant_gemm and sparse_attention are timed.
    Returns (tok/s, sample)."""
    sys.path.insert(0, str(REPO / "oracle"))
    import oracle as O  # CPU checker / baseline only

    if not O.ref_available():
        return None, "oracle/_ref/qcau_ref not built"
    hs = SAMPLE_HEADS
    r = O.ref_bench_decode(threads, threads, hs, WIDTH, CTX, DC, hs * 192, DIM,
                           steps=steps, warmup=warmup)
    secs = r["seconds"]
    frac = hs / HEADS
    sample = (f"per step each of {threads} threads runs {hs} of the {HEADS} heads of one decode "
              f"token ({frac:g} of its work): qcau_c quant_gemm q-up [1,{DC}]x[{hs * 192},{DC}], "
              f"sparse_attention over {CTX} rows x {hs} heads x {WIDTH} (the C++ port has one "
              f"width for K and V), quant_gemm o-proj [1,{hs * 128}]x[{DIM},{hs * 128}]; "
              f"inputs generated before the clock; {warmup} untimed and {steps} timed steps; "
              f"tok/s = threads x {frac:g} / step time")
    return threads * frac * steps / secs, sample


def traffic_from_profiles():
    """dram bytes per launch of the decode attention kernel from the committed ncu
    summary (a line `traffic_bytes_per_launch: N`), or None."""
    for f in sorted((REPO / "profiles").glob("*.md")):
        for line in f.read_text().splitlines():
            if line.startswith("traffic_bytes_per_launch:") and "decode_attn" in f.name:
                try:
                    return float(line.split(":", 1)[1].strip().split()[0])
                except ValueError:
                    return None
    return None


def run_reference_arm(args, rank):
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    v, sample = cpu_reference(args.steps, args.warmup, threads)
    if v is None:
        print(json.dumps({"impl": "reference", "unavailable": sample}))
        return
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * threads * SAMPLE_HEADS / HEADS / v,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": "absorbed-MLA decode layer, batch 128, 128 heads, ctx 32768",
                   "global_batch": BATCH, "seq_len": CTX, "parallelism": "cpu"},
        "cpu_baseline": {"value": v, "unit": "tok/s", "cores": threads, "kind": "reference",
                         "sample": sample},
        "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))


def attn_only(batch: int, ctx: int, local: int):
    """A small decode-attention case for ncu: 128 heads, `ctx` tokens per
    sequence, the same paged layout; 2 warm-up launches then 3 launches."""
    from qcau_b200 import _lib
    from qcau_b200.mla import make_paged_cache

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    cache, table, seqlens = make_paged_cache(batch, ctx, PAGE, WIDTH, dev, seed=0)
    gen = torch.Generator(device=dev).manual_seed(1)
    q = torch.randn(batch, HEADS, WIDTH, device=dev, generator=gen).to(torch.bfloat16)
    o = torch.empty(batch, HEADS, 512, device=dev, dtype=torch.bfloat16)
    L = _lib.lib()
    need = L.qcau_decode_attn_workspace_size(batch, HEADS, 512, ctx)
    wsb = torch.empty(max(need, 1), device=dev, dtype=torch.uint8)
    for _ in range(5):
        _lib.check(L.qcau_decode_attn_paged(q.data_ptr(), cache.data_ptr(), table.data_ptr(),
                                            seqlens.data_ptr(), None, o.data_ptr(), batch, HEADS,
                                            WIDTH, 512, WIDTH, PAGE, table.size(1), cache.size(0),
                                            ctx, 192 ** -0.5, wsb.data_ptr(), need,
                                            _lib.stream_ptr(dev)), "attn")
    torch.cuda.synchronize(dev)
    assert _lib.device_error() == 0
    print(json.dumps({"attn_only": True, "batch": batch, "ctx": ctx}))


def attn_sustained(local: int, seconds: float):
    """The dominant kernel under sustained load: the decode attention of the
    bench's workload (batch 128, 128 heads, ctx 32768, split-KV + combine)
    launched back to back for `seconds`, timed with CUDA events on its
    stream, with the SM clock and throttle reasons sampled during the loop.
    time x clock compares it with the burst figure at another clock."""
    from qcau_b200 import _lib
    from qcau_b200.mla import make_paged_cache

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    cache, table, seqlens = make_paged_cache(BATCH, CTX, PAGE, WIDTH, dev, seed=0)
    gen = torch.Generator(device=dev).manual_seed(1)
    q = torch.randn(BATCH, HEADS, WIDTH, device=dev, generator=gen).to(torch.bfloat16)
    o = torch.empty(BATCH, HEADS, 512, device=dev, dtype=torch.bfloat16)
    L = _lib.lib()
    need = L.qcau_decode_attn_workspace_size(BATCH, HEADS, 512, CTX)
    wsb = torch.empty(max(need, 1), device=dev, dtype=torch.uint8)
    stream = _lib.stream_ptr(dev)

    def run():
        _lib.check(L.qcau_decode_attn_paged(q.data_ptr(), cache.data_ptr(), table.data_ptr(),
                                            seqlens.data_ptr(), None, o.data_ptr(), BATCH, HEADS,
                                            WIDTH, 512, WIDTH, PAGE, table.size(1), cache.size(0),
                                            CTX, 192 ** -0.5, wsb.data_ptr(), need, stream), "attn")

    for _ in range(5):
        run()
    torch.cuda.synchronize(dev)
    # launches per second, from a short burst: enough launches for `seconds`
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(10):
        run()
    e1.record()
    torch.cuda.synchronize(dev)
    n = max(10, int(seconds * 1000.0 / (e0.elapsed_time(e1) / 10)))
    clocks = ClockSampler(local)
    clocks.start()
    e0.record()
    for _ in range(n):
        run()
    e1.record()
    torch.cuda.synchronize(dev)
    clk = clocks.stop()
    assert _lib.device_error() == 0
    ms = e0.elapsed_time(e1) / n
    hbm, _, peak_kind = peaks()
    nbytes = 4867751936
    line = {"attn_sustained": True, "launches": n, "seconds": e0.elapsed_time(e1) / 1000.0,
            "ms_per_launch": ms, "GB/s": nbytes / ms / 1e6, "frac_of_hbm": nbytes / ms / 1e6 / hbm,
            "peak_source": peak_kind, "clocks": clk}
    if clk.get("sm_mhz"):
        line["ms_x_ghz"] = ms * clk["sm_mhz"] / 1000.0
    print(json.dumps(line))


def gemm_only(local: int, m_rows: int = 0):
    """A small FP8 GEMM case for ncu and tuning: the decode layer's q-up
    ([128,1536] x [24576,1536]) and o-proj ([128,16384] x [7168,16384]) with
    fp32 128x128 block scales; 3 warm-up and 5 timed launches of each.  The
    two weights (155 MB) exceed L2 and are read alternately.  m_rows > 0
    gives both GEMMs that many rows (the prefill's 16384, or a smaller
    profiling case)."""
    from qcau_b200 import _lib

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    gen = torch.Generator(device=dev).manual_seed(3)
    L = _lib.lib()
    m_ = m_rows if m_rows > 0 else BATCH
    shapes = {"q_up": (m_, HEADS * 192, DC), "o_proj": (m_, DIM, HEADS * 128)}
    ops = {}
    for name, (m, n, k) in shapes.items():
        a = torch.randn(m, k, device=dev, generator=gen).to(torch.float8_e4m3fn)
        b = torch.randn(n, k, device=dev, generator=gen).to(torch.float8_e4m3fn)
        sa = torch.rand(m, k // 128, device=dev, generator=gen) + 0.5
        sb = torch.rand(n // 128, k // 128, device=dev, generator=gen) + 0.5
        c = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
        ops[name] = (a, sa, b, sb, c, m, n, k)

    def run(name):
        a, sa, b, sb, c, m, n, k = ops[name]
        _lib.check(L.qcau_fp8_gemm(a.data_ptr(), sa.data_ptr(), b.data_ptr(), sb.data_ptr(),
                                   c.data_ptr(), m, n, k, _lib.SCALE_F32, _lib.OUT_BF16,
                                   _lib.stream_ptr(dev)), name)

    for _ in range(3):
        for name in ops:
            run(name)
    res = {}
    for name, (a, sa, b, sb, c, m, n, k) in ops.items():
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        times = []
        for _ in range(5):
            run("q_up" if name == "o_proj" else "o_proj")  # evict this weight from L2
            ev[0].record()
            run(name)
            ev[1].record()
            torch.cuda.synchronize(dev)
            times.append(ev[0].elapsed_time(ev[1]))
        t = sorted(times)[len(times) // 2] * 1e-3
        nbytes = n * k + m * k + m * n * 2 + (n // 128) * (k // 128) * 4 + m * (k // 128) * 4
        res[name] = {"us": t * 1e6, "GB/s": nbytes / t / 1e9, "frac_of_hbm": nbytes / t / 1e9 / peaks()[0],
                     "TFLOP/s": 2.0 * m * n * k / t / 1e12}
    assert _lib.device_error() == 0
    print(json.dumps({"gemm_only": True, **res}))


def _time_ms(fn, warmup=2, reps=5):
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    ev[0].record()
    for _ in range(reps):
        fn()
    ev[1].record()
    torch.cuda.synchronize()
    return ev[0].elapsed_time(ev[1]) / reps


def prefill_only(local: int):
    """Causal prefill attention, batch 4 x 4096 new tokens x 128 heads over the
    paged 576-wide cache (qcau_prefill_attn_paged); device time per call."""
    from qcau_b200 import _lib
    from qcau_b200.mla import make_paged_cache

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    B, S = 4, 4096
    cache, table, sl = make_paged_cache(B, S, PAGE, WIDTH, dev, seed=0)
    gen = torch.Generator(device=dev).manual_seed(1)
    q = torch.randn(B, S, HEADS, WIDTH, device=dev, generator=gen).to(torch.bfloat16)
    o = torch.empty(B, S, HEADS, 512, device=dev, dtype=torch.bfloat16)
    L = _lib.lib()
    need = L.qcau_prefill_attn_workspace_size(B, S, HEADS, 512, S)
    ws = torch.empty(max(need, 1), device=dev, dtype=torch.uint8)

    def run():
        _lib.check(L.qcau_prefill_attn_paged(q.data_ptr(), cache.data_ptr(), table.data_ptr(),
                                             sl.data_ptr(), None, o.data_ptr(), B, S, HEADS,
                                             WIDTH, 512, WIDTH, PAGE, table.size(1),
                                             cache.size(0), S, 192 ** -0.5, ws.data_ptr(), need,
                                             _lib.stream_ptr(dev)), "prefill")
    ms = _time_ms(run)
    assert _lib.device_error() == 0
    flops = 2.0 * B * HEADS * (S * (S + 1) / 2) * (WIDTH + 512)
    print(json.dumps({"prefill_only": True, "batch": B, "seq": S, "heads": HEADS, "ms": ms,
                      "TFLOP/s": flops / ms / 1e9, "workspace_bytes": need}))


def prefill_layer(local: int, B: int = 4, S: int = 4096):
    """The whole absorbed-MLA layer on a prefill: batch 4 x 4096 new tokens x
    128 heads (q-up FP8 GEMM at M = 16384, RoPE, absorb, causal attention
    over the paged cache, v-up, o-proj FP8 GEMM at M = 16384); device time of
    the step and of each stage (CUDA events), with each stage's FLOPs."""
    from qcau_b200 import _lib
    from qcau_b200.mla import MLAConfig, MLADecodeLayer, make_paged_cache, precompute_freqs_cis

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    cfg = MLAConfig(n_heads=HEADS, dc=DC, dim=DIM)
    layer = MLADecodeLayer(cfg, dev)
    layer.random_weights(seed=0)
    cache, table, sl = make_paged_cache(B, S, PAGE, WIDTH, dev, seed=0)
    freqs = precompute_freqs_cis(64, S + 1, cfg.rope_theta, dev)
    gen = torch.Generator(device=dev).manual_seed(1)
    q_lora = torch.randn(B, S, DC, device=dev, generator=gen)
    q_lora = (q_lora * torch.rsqrt(q_lora.square().mean(-1, keepdim=True))).to(torch.bfloat16)
    y = torch.empty(B, S, DIM, device=dev, dtype=torch.bfloat16)

    def run():
        layer.forward_prefill(q_lora, cache, table, sl, freqs, S, y)
    ms = _time_ms(run, warmup=2, reps=3)
    assert _lib.device_error() == 0
    rows = B * S
    fl = {"q_up_fp8": 2.0 * rows * HEADS * 192 * DC,
          "absorb": 2.0 * rows * HEADS * 128 * 512,
          "attention": 2.0 * B * HEADS * (S * (S + 1) / 2) * (WIDTH + 512),
          "v_up": 2.0 * rows * HEADS * 512 * 128,
          "o_proj_fp8": 2.0 * rows * DIM * HEADS * 128}
    # per stage: the same calls one at a time between events
    c = cfg
    d = layer.dims(rows, table.size(1), cache.size(0), 1, freqs.size(0))
    q2 = q_lora.reshape(rows, DC)
    pos = (sl.to(torch.int64).view(B, 1) - S + 1 +
           torch.arange(S, device=dev).view(1, S)).to(torch.int32).reshape(-1)
    q_abs = torch.empty(rows, HEADS, WIDTH, device=dev, dtype=torch.bfloat16)
    o_lat = torch.empty(rows, HEADS, 512, device=dev, dtype=torch.bfloat16)
    L = _lib.lib()
    need = L.qcau_prefill_attn_workspace_size(B, S, HEADS, 512, S)
    ws = torch.empty(max(need, 1), device=dev, dtype=torch.uint8)
    st = {"q_up_rope_absorb": lambda: layer._q_stage(d, q2, pos, freqs, q_abs),
          "attention": lambda: _lib.check(L.qcau_prefill_attn_paged(
              q_abs.data_ptr(), cache.data_ptr(), table.data_ptr(), sl.data_ptr(), None,
              o_lat.data_ptr(), B, S, HEADS, WIDTH, 512, WIDTH, PAGE, table.size(1),
              cache.size(0), S, c.softmax_scale, ws.data_ptr(), need, _lib.stream_ptr(dev)),
              "prefill"),
          "v_up_o_proj": lambda: layer._out_stage(d, o_lat, y.view(rows, DIM))}
    stages = {k: _time_ms(f, warmup=1, reps=3) for k, f in st.items()}
    total = sum(fl.values())
    _, tflops, kind = peaks()
    print(json.dumps({"prefill_layer": True, "batch": B, "seq": S, "heads": HEADS, "ms": ms,
                      "TFLOP/s": total / ms / 1e9, "flops": total, "stage_ms": stages,
                      "stage_flops": fl, "bf16_peak_tflops": tflops, "peak_source": kind,
                      "note": "FP8 GEMM FLOPs (q-up, o-proj) run at the FP8 rate, the rest bf16"}))


def sparse_fp8_only(local: int, heads: int, rows: int = 131072):
    """Long-context sparse decode over an FP8 latent cache: batch 64, `rows`
    rows per sequence (131072 by default; e4m3 latent + fp32 row scale + bf16
    rope), top-2048 indices, `heads` heads (16 = one rank of an 8-way head
    shard).  Fewer rows gather the same bytes from a smaller cache (a
    profiling case)."""
    from qcau_b200 import _lib

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    B, N, K = 64, rows, 2048
    gen = torch.Generator(device=dev).manual_seed(2)
    codes = torch.randint(0, 0x7F, (B, N, 512), device=dev, generator=gen, dtype=torch.uint8)
    scale = torch.rand(B, N, device=dev, generator=gen) * 0.01 + 1e-3
    rope = torch.randn(B, N, 64, device=dev, generator=gen).to(torch.bfloat16)
    idx = torch.stack([torch.randperm(N, device=dev, generator=gen)[:K] for _ in range(B)])
    idx = idx.to(torch.int32).view(B, 1, K).contiguous()
    q = torch.randn(B, 1, heads, WIDTH, device=dev, generator=gen).to(torch.bfloat16)
    o = torch.empty(B, 1, heads, 512, device=dev, dtype=torch.bfloat16)
    L = _lib.lib()
    need = L.qcau_sparse_attn_fp8_workspace_size(B, 1, heads, K)
    ws = torch.empty(max(need, 1), device=dev, dtype=torch.uint8)

    def run():
        _lib.check(L.qcau_sparse_attn_fp8(q.data_ptr(), codes.data_ptr(), scale.data_ptr(),
                                          rope.data_ptr(), None, idx.data_ptr(), o.data_ptr(), B,
                                          1, heads, N, K, 192 ** -0.5, ws.data_ptr(), need,
                                          _lib.stream_ptr(dev)), "sparse_fp8")
    ms = _time_ms(run)
    assert _lib.device_error() == 0
    nbytes = B * K * (512 + 4 + 128) + B * K * 4 + B * heads * (WIDTH + 512) * 2
    hbm, _, peak_kind = peaks()
    print(json.dumps({"sparse_fp8_only": True, "batch": B, "rows": N, "topk": K, "heads": heads,
                      "us": ms * 1e3, "GB/s": nbytes / ms / 1e6, "algorithmic_bytes": nbytes,
                      "frac_of_hbm": nbytes / ms / 1e6 / hbm, "peak_source": peak_kind}))


def _time_flushed_us(fn, flush, reps=7):
    """Median device time (us) of fn(), each launch timed alone with CUDA
    events after `flush` (a write larger than L2) evicted its inputs."""
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    fn()
    fn()
    times = []
    for _ in range(reps):
        flush.add_(1)
        ev[0].record()
        fn()
        ev[1].record()
        torch.cuda.synchronize()
        times.append(ev[0].elapsed_time(ev[1]) * 1e3)
    return sorted(times)[len(times) // 2]


def producers_only(local: int):
    """The producers either side of the decode attention, each at the model's
    widths (V4-Flash: 64 heads of 512, index heads 64 x 128, top-512, ratio 4)
    and a decode or prefill shape, timed per call with L2 flushed before it:

    - kv_build: RMSNorm + RoPE + FP8 round trip of new 512-wide KV rows,
      written into the cache by slot (decode: 128 rows; prefill: 4 x 4096);
    - compressor: gated pooling of ratio-4 overlapping windows of the fp32
      wkv / wgate projections, then kv_build into the cache (prefill 4 x 4096;
      decode: 128 sequences, a step that closes a group);
    - indexer: Hadamard + FP4 of the queries, q.k over the compressed keys,
      ReLU x head weights, head sum, top-512 (decode: 128 sequences at 32768
      tokens = 8192 compressed keys each);
    - GOPU: grouped wo_a (8 groups x 1024 x 4096 bf16), act_quant, FP8 wo_b
      [4096, 8192] (decode: 128 tokens).

    Algorithmic bytes are the inputs read once and the outputs written once
    (workspace round trips are not counted)."""
    from qcau_b200 import _lib
    from qcau_b200.cache import Compressor, kv_build
    from qcau_b200.gopu import GOPU
    from qcau_b200.indexer import Indexer
    from qcau_b200.mla import precompute_freqs_cis, quantize_weight_fp8

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    gen = torch.Generator(device=dev).manual_seed(5)
    flush = torch.zeros(64 << 20, device=dev, dtype=torch.float32)  # 256 MB > L2
    hbm, _, peak_kind = peaks()
    res = {}

    def rec(name, us, nbytes, **kw):
        res[name] = {"us": round(us, 2), "algorithmic_bytes": int(nbytes),
                     "GB/s": round(nbytes / us / 1e3, 1),
                     "frac_of_hbm": round(nbytes / us / 1e3 / hbm, 3), **kw}

    d, rd = 512, 64
    freqs = precompute_freqs_cis(rd, 32768 + 8, 10000.0, dev)
    normw = torch.ones(d, device=dev)
    for name, rows in (("kv_build_decode_b128", 128), ("kv_build_prefill_4x4096", 16384)):
        x = torch.randn(rows, d, device=dev, generator=gen).to(torch.bfloat16)
        pos = torch.arange(rows, device=dev, dtype=torch.int32) % 32768
        cache = torch.zeros(rows + 64, d, device=dev, dtype=torch.bfloat16)
        slots = torch.arange(rows, device=dev, dtype=torch.int32)
        us = _time_flushed_us(lambda: kv_build(x, normw, freqs, pos, rope_dim=rd, cache=cache,
                                               slots=slots, return_rows=False), flush)
        rec(name, us, rows * (d * 2 * 2 + 8), rows=rows)

    for name, b, s, sp in (("compressor_prefill_4x4096", 4, 4096, 0),
                           ("compressor_decode_b128", 128, 1, 4095)):
        comp = Compressor(d, 4, rd, max_batch=b, device=dev)
        comp.kv_cache = torch.zeros(b, 1024, d, device=dev, dtype=torch.bfloat16)
        comp.freqs_cis = torch.view_as_complex(freqs[:4104])
        kv = torch.randn(b, s, 2 * d, device=dev, generator=gen)
        sc = torch.randn(b, s, 2 * d, device=dev, generator=gen)
        n_out = b * max(s // 4, 1)
        us = _time_flushed_us(lambda: comp.forward(kv, sc, sp), flush)
        state = 0 if s > 1 else comp.kv_state[:b].numel() * 4 * 2 * 2
        rec(name, us, kv.numel() * 4 * 2 + n_out * d * 2 + state, batch=b, tokens=s)

    b, h, t, k = 128, 64, 8192, 512
    q = torch.randn(b, 1, h, 128, device=dev, generator=gen).to(torch.bfloat16)
    keys = torch.randn(b, t, 128, device=dev, generator=gen).to(torch.bfloat16)
    w = (torch.randn(b, 1, h, device=dev, generator=gen) * 0.01).to(torch.bfloat16)
    ix = Indexer(n_heads=h, head_dim=128, index_topk=k, compress_ratio=4, device=dev)
    us = _time_flushed_us(lambda: ix.forward(q, keys, w, 4 * t - 1, 0, rotate=True), flush)
    rec("indexer_decode_b128_t8192", us, keys.numel() * 2 + q.numel() * 2 + w.numel() * 2
        + b * k * 4, batch=b, heads=h, compressed_keys=t, topk=k,
        score_workspace_bytes=b * h * t * 2)

    rows, G, R, Dm = 128, 8, 1024, 4096
    o = torch.randn(rows, 64, d, device=dev, generator=gen).to(torch.bfloat16)
    wo_a = (torch.randn(G * R, 64 * d // G, device=dev, generator=gen) * 0.02).to(torch.bfloat16)
    wb, wbs = quantize_weight_fp8(torch.randn(Dm, G * R, device=dev, generator=gen) * 0.02, True)
    m = GOPU(device=dev)
    m.load_weights(wo_a, wb, wbs)
    us = _time_flushed_us(lambda: m.forward_local(o), flush)
    rec("gopu_decode_b128", us, wo_a.numel() * 2 + wb.numel() + wbs.numel() + o.numel() * 2
        + rows * Dm * 2, rows=rows)
    assert _lib.device_error() == 0
    print(json.dumps({"producers_only": True, "peak_gbs": hbm, "peak_source": peak_kind,
                      "l2": "flushed before each timed call", **res}))


def stage_times(layer, q_lora, cache, table, seqlens, positions, freqs, y, dev, ws, steps):
    """Per-stage device time (us, mean over `steps` steps, max over ranks) of
    the row-split decode step: CUDA events recorded between its stages on the
    compute stream.  NCCL collectives run on that stream too, so a collective's
    time includes waiting for the slowest rank to reach it."""
    layer.stage_events = []
    split = layer.attn_split
    layer.attn_split = "rows"
    try:
        for _ in range(2):
            layer.forward_rows(q_lora, cache, table, seqlens, positions, freqs, CTX, y)
        torch.cuda.synchronize(dev)
        if ws > 1:
            dist.barrier()
        layer.stage_events = []
        for _ in range(steps):
            layer.forward_rows(q_lora, cache, table, seqlens, positions, freqs, CTX, y)
        torch.cuda.synchronize(dev)
        evs = layer.stage_events
    finally:
        layer.stage_events = None
        layer.attn_split = split
    names, acc = [], {}
    for (n0, e0), (n1, e1) in zip(evs, evs[1:]):
        if n1 == "start":
            continue
        if n1 not in acc:
            names.append(n1)
            acc[n1] = 0.0
        acc[n1] += e0.elapsed_time(e1) * 1000.0 / steps
    t = torch.tensor([acc[n] for n in names], device=dev, dtype=torch.float64)
    if ws > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return {n: round(float(v), 2) for n, v in zip(names, t.tolist())}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--attn-only", action="store_true",
                    help="profiling case: only the decode attention, --batch x --ctx, 5 launches")
    ap.add_argument("--gemm-only", action="store_true",
                    help="profiling case: the layer's two FP8 GEMMs at batch 128")
    ap.add_argument("--prefill-only", action="store_true",
                    help="time the causal prefill attention, batch 4 x 4096 x 128 heads")
    ap.add_argument("--gemm-m", type=int, default=0,
                    help="rows of the --gemm-only GEMMs (default: the decode batch)")
    ap.add_argument("--prefill-layer", action="store_true",
                    help="time the whole layer on a prefill, batch 4 x 4096 x 128 heads, "
                         "with its stages")
    ap.add_argument("--sparse-fp8-only", type=int, default=0, metavar="HEADS",
                    help="time the FP8-cache top-k sparse decode (batch 64, 131072 rows) at HEADS")
    ap.add_argument("--producers", action="store_true",
                    help="time the KV build, compressor, indexer top-k and GOPU at decode "
                         "and prefill shapes, each with L2 flushed")
    ap.add_argument("--attn-split", default="rows", choices=["context", "rows", "heads"],
                    help="N > 1: split the attention of the head-sharded layer by context "
                         "(each rank 1/N of every sequence), by rows (each rank 1/N of the "
                         "sequences) or by heads (each rank streams the whole cache)")
    ap.add_argument("--exchange", default="nccl", choices=["nccl", "p2p"],
                    help="context split: partial states exchanged by an NCCL all-to-all, or "
                         "stored by the attention kernel into the owning rank's memory")
    ap.add_argument("--sparse-rows", type=int, default=131072,
                    help="rows per sequence of the --sparse-fp8-only cache")
    ap.add_argument("--sustained", type=float, default=0.0, metavar="SECONDS",
                    help="time the decode attention launched back to back for SECONDS, "
                         "with clocks sampled (the sustained figure)")
    ap.add_argument("--no-graphs", action="store_true",
                    help="run every decode step eagerly instead of replaying it from a CUDA graph")
    ap.add_argument("--stages", action="store_true",
                    help="after the timed steps, time the row-split step's stages (q-up, "
                         "all-to-alls, attention, out-projection, all-reduce) with CUDA "
                         "events, max over ranks, and add them to the line as stages_us")
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--ctx", type=int, default=4096)
    args = ap.parse_args()
    ws, rank, local = dist_env()
    if args.attn_only:
        attn_only(args.batch, args.ctx, local)
        return
    if args.sustained > 0:
        attn_sustained(local, args.sustained)
        return
    if args.gemm_only:
        gemm_only(local, args.gemm_m)
        return
    if args.prefill_only:
        prefill_only(local)
        return
    if args.prefill_layer:
        prefill_layer(local)
        return
    if args.producers:
        producers_only(local)
        return
    if args.sparse_fp8_only:
        sparse_fp8_only(local, args.sparse_fp8_only, args.sparse_rows)
        return
    if args.impl == "reference":
        run_reference_arm(args, rank)
        return

    import qcau_b200
    from qcau_b200 import _lib
    from qcau_b200.mla import MLAConfig, MLADecodeLayer, make_paged_cache, precompute_freqs_cis

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=dev)
    cfg = MLAConfig(n_heads=HEADS, dc=DC, dim=DIM)
    layer = MLADecodeLayer(cfg, dev, rank=rank, world_size=ws, attn_split=args.attn_split,
                           exchange=args.exchange, cuda_graphs=not args.no_graphs)
    cp = ws > 1 and args.attn_split == "context"
    rs = ws > 1 and args.attn_split == "rows"
    layer.random_weights(seed=0)
    cache, table, seqlens = make_paged_cache(BATCH, CTX, PAGE, WIDTH, dev, seed=0)
    positions = seqlens.clone()
    freqs = precompute_freqs_cis(64, CTX + 1, cfg.rope_theta, dev)
    gen = torch.Generator(device=dev).manual_seed(1)
    q_lora = torch.randn(BATCH, DC, device=dev, generator=gen)
    q_lora = (q_lora * torch.rsqrt(q_lora.square().mean(-1, keepdim=True))).to(torch.bfloat16)
    y = torch.empty(BATCH, DIM, device=dev, dtype=torch.bfloat16)
    stream = torch.cuda.current_stream(dev)

    def step():
        layer.forward(q_lora, cache, table, seqlens, positions, freqs, CTX, y)

    def barrier():
        if ws > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    for _ in range(max(args.warmup, 3)):
        step()
    barrier()
    assert _lib.device_error() == 0, "device error during warm-up"

    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    barrier()
    ms = e0.elapsed_time(e1)
    clk = clocks.stop()
    t = torch.tensor([ms], device=dev, dtype=torch.float64)
    if ws > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_total = float(t.item())
    ms_step = ms_total / args.steps
    value = BATCH * args.steps / (ms_total / 1000.0)

    stages = stage_times(layer, q_lora, cache, table, seqlens, positions, freqs, y, dev, ws,
                         args.steps) if args.stages else None

    # ---- dominant kernel alone: the decode attention, timed on its stream
    L = _lib.lib()
    H = layer.n_local
    if cp:
        # this rank's context-parallel attention: all heads over 1/N of every
        # sequence's tiles, partials for the exchange
        q_all = torch.randn(ws, BATCH, H, WIDTH, device=dev, generator=gen).to(torch.bfloat16)
        part_o = torch.empty(ws, BATCH, H, 512, device=dev, dtype=torch.float16)
        part_ml = torch.empty(ws, BATCH, H, 2, device=dev)

        def attn():
            _lib.check(L.qcau_decode_attn_paged_cp(
                q_all.data_ptr(), cache.data_ptr(), table.data_ptr(), seqlens.data_ptr(),
                part_o.data_ptr(), part_ml.data_ptr(), BATCH, HEADS, ws, rank, WIDTH, 512, WIDTH,
                PAGE, table.size(1), cache.size(0), CTX, cfg.softmax_scale, 1,
                _lib.stream_ptr(dev)), "attn_cp")
    elif rs:
        # this rank's sequences with all heads, q and o in the owners' head blocks
        Br = BATCH // ws
        q_rows = torch.randn(ws, Br, H, WIDTH, device=dev, generator=gen).to(torch.bfloat16)
        o_rows = torch.empty(ws, Br, H, 512, device=dev, dtype=torch.bfloat16)
        need = L.qcau_decode_attn_workspace_size(Br, HEADS, 512, CTX)
        wsb = torch.empty(max(need, 1), device=dev, dtype=torch.uint8)
        t_rows = table[rank * Br:(rank + 1) * Br]
        s_rows = seqlens[rank * Br:(rank + 1) * Br]

        def attn():
            _lib.check(L.qcau_decode_attn_paged_blocked(
                q_rows.data_ptr(), H, cache.data_ptr(), t_rows.data_ptr(), s_rows.data_ptr(),
                None, o_rows.data_ptr(), H, Br, HEADS, WIDTH, 512, WIDTH, PAGE, table.size(1),
                cache.size(0), CTX, cfg.softmax_scale, wsb.data_ptr(), need,
                _lib.stream_ptr(dev)), "attn_rows")
    else:
        q_abs = torch.randn(BATCH, H, WIDTH, device=dev, generator=gen).to(torch.bfloat16)
        o_lat = torch.empty(BATCH, H, 512, device=dev, dtype=torch.bfloat16)
        need = L.qcau_decode_attn_workspace_size(BATCH, H, 512, CTX)
        wsb = torch.empty(max(need, 1), device=dev, dtype=torch.uint8)

        def attn():
            _lib.check(L.qcau_decode_attn_paged(
                q_abs.data_ptr(), cache.data_ptr(), table.data_ptr(), seqlens.data_ptr(), None,
                o_lat.data_ptr(), BATCH, H, WIDTH, 512, WIDTH, PAGE, table.size(1),
                cache.size(0), CTX, cfg.softmax_scale, wsb.data_ptr(), need,
                _lib.stream_ptr(dev)), "attn")

    for _ in range(3):
        attn()
    torch.cuda.synchronize(dev)
    a0 = torch.cuda.Event(enable_timing=True)
    a1 = torch.cuda.Event(enable_timing=True)
    n_attn = max(5, args.steps)
    a0.record(stream)
    for _ in range(n_attn):
        attn()
    a1.record(stream)
    torch.cuda.synchronize(dev)
    attn_ms = a0.elapsed_time(a1) / n_attn
    cache_bytes = BATCH * CTX * WIDTH * 2
    full_bytes = cache_bytes + BATCH * HEADS * (WIDTH + 512) * 2 + table.numel() * 4
    if cp:
        # 1/N of the cache and block table (the ranks' tile ranges are equal
        # here: 256 tiles per sequence), q of all heads, partials out (fp16
        # O / sum, fp32 max and sum)
        attn_bytes = (cache_bytes + table.numel() * 4) // ws + BATCH * HEADS * WIDTH * 2 + \
            BATCH * HEADS * (512 * 2 + 2 * 4)
        attn_flops = 2.0 * BATCH * (CTX // ws) * HEADS * (WIDTH + 512)
    elif rs:
        # the pages, q and o of 1/N of the sequences, all heads
        attn_bytes = (cache_bytes + table.numel() * 4 + BATCH * HEADS * (WIDTH + 512) * 2) // ws
        attn_flops = 2.0 * (BATCH // ws) * CTX * HEADS * (WIDTH + 512)
    else:
        attn_bytes = cache_bytes + BATCH * H * (WIDTH + 512) * 2 + table.numel() * 4
        attn_flops = 2.0 * BATCH * CTX * H * (WIDTH + 512)
    hbm, tflops, peak_kind = peaks()
    t_bw = attn_bytes / (hbm * 1e9)
    t_tc = attn_flops / (tflops * 1e12)
    if t_bw >= t_tc:
        roof = {"bound": "hbm", "achieved": attn_bytes / (attn_ms * 1e-3) / 1e9, "peak": hbm,
                "unit": "GB/s"}
    else:
        roof = {"bound": "tensor", "achieved": attn_flops / (attn_ms * 1e-3) / 1e12,
                "peak": tflops, "unit": "TFLOP/s"}
    roof["frac"] = roof["achieved"] / roof["peak"]
    traffic = traffic_from_profiles()
    if rs:
        roof["traffic"] = traffic * attn_bytes / full_bytes if traffic else None
        roof["traffic_note"] = "scaled from the 1-GPU full-launch capture by algorithmic bytes"
        roof["kernel"] = ("decode attention of this rank's 1/N of the sequences, all heads "
                          "(split-KV + combine); per launch")
    elif cp:
        # the one-GPU capture's DRAM bytes per algorithmic byte, applied to this launch
        roof["traffic"] = traffic * attn_bytes / full_bytes if traffic else None
        roof["traffic_note"] = "scaled from the 1-GPU full-launch capture by algorithmic bytes"
        roof["kernel"] = ("context-parallel decode attention: all heads over this rank's 1/N "
                          "of the tiles, partials out; per launch")
    else:
        roof["traffic"] = traffic
        roof["kernel"] = "decode attention (split-KV + combine), per launch"
    roof["ms_per_launch"] = attn_ms
    roof["peak_source"] = f"{peak_kind} (MEASURED_PEAKS.json)" if peak_kind == "measured" else peak_kind
    roof["algorithmic_bytes"] = attn_bytes
    roof["algorithmic_flops"] = attn_flops

    # ---- end to end through the public API with host buffers: every step
    # copies its q_lora from pinned host memory to the device and its y back;
    # the copies run on a second stream with double buffers, so a step's input
    # arrives while the previous step computes and its output leaves while the
    # next one does (as a serving loop would pipeline them)
    q_host = q_lora.cpu().pin_memory()
    y_host = [torch.empty(BATCH, DIM, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    q_dev = [torch.empty_like(q_lora) for _ in range(2)]
    y_dev = [torch.empty_like(y) for _ in range(2)]
    copy = torch.cuda.Stream(dev)
    ev = {k: [torch.cuda.Event() for _ in range(2)] for k in ("h2d", "comp", "d2h")}

    def e2e_run(n):
        copy.wait_stream(stream)
        with torch.cuda.stream(copy):
            q_dev[0].copy_(q_host, non_blocking=True)
            ev["h2d"][0].record(copy)
        for k in range(n):
            s_ = k & 1
            if k + 1 < n:
                with torch.cuda.stream(copy):
                    if k >= 1:   # step k-1 is done reading that buffer
                        copy.wait_event(ev["comp"][1 - s_])
                    q_dev[1 - s_].copy_(q_host, non_blocking=True)
                    ev["h2d"][1 - s_].record(copy)
            stream.wait_event(ev["h2d"][s_])
            if k >= 2:           # y_dev[s_] of step k-2 has been read out
                stream.wait_event(ev["d2h"][s_])
            layer.forward(q_dev[s_], cache, table, seqlens, positions, freqs, CTX, y_dev[s_])
            ev["comp"][s_].record(stream)
            with torch.cuda.stream(copy):
                copy.wait_event(ev["comp"][s_])
                y_host[s_].copy_(y_dev[s_], non_blocking=True)
                ev["d2h"][s_].record(copy)
        stream.wait_stream(copy)

    e2e_run(3)
    barrier()
    b0 = torch.cuda.Event(enable_timing=True)
    b1 = torch.cuda.Event(enable_timing=True)
    b0.record(stream)
    e2e_run(args.steps)
    b1.record(stream)
    barrier()
    te = torch.tensor([b0.elapsed_time(b1)], device=dev, dtype=torch.float64)
    if ws > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_val = BATCH * args.steps / (float(te.item()) / 1000.0)
    assert _lib.device_error() == 0, "device error during the timed region"

    # act_quant, gemm, bmm (absorb, with the query's RoPE in its epilogue),
    # attention, combine, bmm (v-up, with the act_quant of its output), gemm
    launches_per_step = 7
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded random weights, cache and activations)",
            "config": {"workload": "absorbed-MLA QCAU decode layer: batch 128, 128 heads "
                                   "head-sharded over ranks, ctx 32768, paged bf16 latent "
                                   "cache page 64, FP8 block-scaled wq_b/wo, bf16 all-reduce "
                                   "[128,7168]",
                       "global_batch": BATCH, "seq_len": CTX, "heads_per_rank": H,
                       "parallelism": (f"head-shard tp{ws}, attention split by context "
                                       f"(q all-gather, partial exchange: {args.exchange})"
                                       if cp else
                                       f"head-shard tp{ws}, attention split by sequences "
                                       "(q and o all-to-all)" if rs else f"head-shard tp{ws}"),
                       "l2": "inputs (4.83 GB cache) larger than L2; no flush",
                       "launch": ("eager launches" if args.no_graphs else
                                  "each step replayed from a CUDA graph (kernels and "
                                  "collectives), captured after one eager step")},
            "roofline": roof,
            "e2e": {"value": e2e_val, "unit": "tok/s",
                    "h2d_bytes_per_step": q_lora.numel() * 2,
                    "d2h_bytes_per_step": y.numel() * 2,
                    "copies": "pinned host buffers, overlapped with the neighbouring steps "
                              "on a second stream"},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clk,
        }
        if stages is not None:
            line["stages_us"] = stages
        if ws == 1 and not args.no_cpu_baseline:
            threads = os.cpu_count() or 1
            v, sample = cpu_reference(3, 1, threads)
            line["cpu_baseline"] = ({"value": v, "unit": "tok/s", "cores": threads,
                                     "kind": "reference", "sample": sample}
                                    if v is not None else {"value": None, "unavailable": sample})
        print(json.dumps(line))
    if ws > 1:
        dist.barrier()
        layer.close()   # peer receive buffers of the p2p exchange, if any (collective)
        layer.release_graphs()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
