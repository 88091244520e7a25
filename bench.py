"""Benchmark: Q4_0 Llama-2-7B-shaped greedy decode, batch 1, KV context 4096.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

One process per GPU (torchrun for N > 1); the model is tensor-parallel over
the N GPUs (NCCL all-reduce after o_proj and down_proj), so the total work per
step is fixed (strong scaling).  A step = one decode token of every sequence.

  value  : tokens/s with the step loop resident on the device (token ids stay
           in HBM, K CUDA-graph launches back to back), timed with CUDA events
           on the library's stream, max over ranks;
  e2e    : the same metric through the public C ABI call (fg_llama_decode) with
           host buffers: each step copies the input id in and the next id out;
  roofline: the dominant kernel.  On one GPU a decode step is one launch of
           the persistent decode-step kernel (k_decode_step), so its
           algorithmic bytes per launch (all Q4_0 weights + the KV cache read
           at the mean timed position + norms and vectors) / its time per
           launch vs the measured HBM copy bandwidth.  Under tensor parallelism
           the dominant kernel is the fused dequant-GEMV, re-timed live on the
           rank's 7B layer shapes with cold L2;
  cpu_baseline: the CPU oracle (a port of the reference arithmetic) decoding
           a bounded sample of the same workload on the host cores.

Weights are seeded synthetic N(0, 0.02) quantized to GGUF Q4_0; the prompt is
4096 seeded random ids (no checkpoint or dataset is used).
"""
import argparse
import json
import os
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "ameva-forge_b200"))

import numpy as np  # noqa: E402
import torch  # noqa: E402  (plumbing: rendezvous, barriers, events on the library stream)
import torch.distributed as dist  # noqa: E402

METRIC = "Q4_0 decode tokens/s"
UNIT = "tokens/s"
CONTEXT = 4096
BATCH = 1
SEED = 20240601
SHAPE = dict(vocab_size=32000, hidden_size=4096, intermediate_size=11008, num_hidden_layers=32,
             num_attention_heads=32, num_key_value_heads=32, rms_norm_eps=1e-5, rope_theta=10000.0)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="forge_b200", choices=["forge_b200", "reference"])
    ap.add_argument("--cpu-baseline", type=int, default=1, help="time the CPU oracle sample (rank 0, N=1)")
    ap.add_argument("--roofline-only", action="store_true",
                    help="only time the dequant-GEMV on the layer shapes (the profiling case)")
    ap.add_argument("--gemm-table", action="store_true",
                    help="the Q4_0 dequant-GEMV/GEMM table: 4096x11008 and 11008x4096 at batch 1/8/32/128")
    ap.add_argument("--gemm-case", default="",
                    help="profiling case M,N,K: `warmup` + `steps` launches of one Q4_0 GEMM (x [M,K] fp32, "
                         "W [N,K]); prints its event-timed launch time")
    ap.add_argument("--attention-case", default="",
                    help="flash-attention prefill B,H,S,d[,f32] (causal, fp16 (or fp32) Q/K/V ~ N(0,1), scale 1/sqrt(d)): "
                         "`warmup` + `steps` calls; prints TFLOP/s and the tensor-core fraction")
    ap.add_argument("--decode-table", action="store_true",
                    help="decode rows of the scope table: TinyLlama-1.1B shape b1 ctx 2048 (256 tokens), "
                         "Llama-2-7B shape b1/16/64 ctx 4096; prints one line per row")
    ap.add_argument("--graph-decode", action="store_true",
                    help="the executeGraph path: forge-py's Llama graph (GraphLlama) over TinyLlama-1.1B-shaped "
                         "Q4_0 weights, a 128-token prompt, then `steps` cached greedy tokens, one graph each "
                         "(JSON build, parse, run, logits read and host argmax all inside the timing)")
    ap.add_argument("--profile-layers", type=int, default=0,
                    help="profiling case: a model of this many 7B layers at context 4096, `steps` decode steps; "
                         "prints no bench line")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    return rank, world, local


def config_block(n):
    return {"workload": "llama2-7b-shape q4_0 greedy decode", "model": "Llama-2-7B-shaped (random init)",
            "global_batch": BATCH, "context": CONTEXT, "seq_len": CONTEXT, "layers": 32, "hidden": 4096,
            "heads": 32, "head_dim": 128, "ffn": 11008, "vocab": 32000, "weights": "GGUF Q4_0",
            "kv_cache": "fp16", "parallelism": f"tp{n}",
            "l2": "inputs larger than L2: every step streams 3.7 GB of weights + 2.1 GB of KV"}


# ------------------------------------------------------------------ clocks
class Clocks:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.p = None

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "200"],
                                      stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.p = None
        return self

    def __exit__(self, *a):
        self.rows = []
        if self.p is None:
            return
        self.p.terminate()
        try:
            out, _ = self.p.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.p.kill()
            out, _ = self.p.communicate()
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) >= 9:
                self.rows.append(f)

    def summary(self):
        if not getattr(self, "rows", None):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


# ------------------------------------------------------------------ CPU oracle
class CpuDecoder:
    """The reference's decode arithmetic on the host cores: the oracle port
    (oracle/forge_oracle.c, the reference's dequant / GEMV / attention / norm
    arithmetic restated in C, OpenMP over all host threads) running greedy
    decode steps of the Llama-2-7B-shaped model -- `layers` of its layers,
    embedding, final norm and lm_head -- from a KV cache filled with seeded
    fp16 values to `context` positions (LlamaRef.synthesize_kv).  The
    reference itself runs this path only as WGSL through WebGPU in a browser,
    which this host does not have."""

    def __init__(self, layers, context=CONTEXT, extra=64):
        sys.path.insert(0, os.path.join(REPO, "oracle"))
        import oracle as O
        self.O = O
        self.layers = layers
        t0 = time.perf_counter()
        shp = O.LlamaShape(**{**SHAPE, "num_hidden_layers": layers})
        self.ref = O.LlamaRef(O.synth_llama(shp, SEED), max_seq=context + extra, kv_f16=True)
        self.ref.synthesize_kv(SEED + 1, context)
        self.setup_s = time.perf_counter() - t0
        self.tok = np.array([[1]], np.int32)

    def step(self):
        """One greedy decode token; returns its wall time in seconds."""
        t0 = time.perf_counter()
        lg = self.ref.forward(self.tok)
        self.tok = np.array([[self.O.argmax(lg[0, -1])]], np.int32)
        return time.perf_counter() - t0

    def head_time(self):
        """Final norm + lm_head GEMV alone (the part of a step that does not scale with layers)."""
        O, w = self.O, self.ref.w
        x = O.normal(1, 0, SHAPE["hidden_size"], 0.0, 1.0).reshape(1, -1)
        t0 = time.perf_counter()
        O.qmatmul(w.qtype, w.lm_head, SHAPE["vocab_size"], SHAPE["hidden_size"], O.rmsnorm(x, w.norm))
        return time.perf_counter() - t0


def cpu_sample(steps=2, layers=2):
    """cpu_baseline of the main arm: a bounded sample (about 10 s of CPU work)
    -- `steps` decode steps at context 4096 through `layers` of the 32 layers
    plus the head; tokens/s scaled to the full model."""
    dec = CpuDecoder(layers)
    dec.step()  # warm-up (first touch of the weights)
    t_step = sum(dec.step() for _ in range(steps)) / steps
    t_head = dec.head_time()
    per_tok = (t_step - t_head) * (SHAPE["num_hidden_layers"] / layers) + t_head
    return {"value": 1.0 / per_tok, "unit": UNIT, "cores": dec.O.num_threads(), "kind": "port",
            "sample": f"1 warm-up + {steps} timed decode steps at context {CONTEXT} through {layers} of 32 layers "
                      f"+ lm_head, layer time scaled x{SHAPE['num_hidden_layers'] // layers}; KV filled with seeded "
                      f"fp16 N(0,1)"}


def forge_py_recorded():
    """The reference's own CPU path (forge-py LlamaForCausalLM(device='cpu'),
    numpy fp32) timed beside the port by oracle/time_forge_py.py in the build
    container -- forge-py is not installed on this host, so the figure is a
    recorded one, labelled as such."""
    try:
        with open(os.path.join(REPO, "oracle", "forge_py_cpu_timing.json")) as f:
            return json.load(f)
    except (OSError, ValueError):
        return None


def run_reference(args, rank, world):
    """--impl reference: the full 32-layer model decoded on the host cores by
    the oracle port (CpuDecoder); `warmup` untimed and `steps` timed greedy
    steps at context 4096, all of them real.  Under torchrun only rank 0 runs;
    the other ranks exit without work."""
    if rank != 0:
        return
    layers = SHAPE["num_hidden_layers"]
    dec = CpuDecoder(layers, extra=args.warmup + args.steps + 8)
    for _ in range(args.warmup):
        dec.step()
    t0 = time.perf_counter()
    times = [dec.step() for _ in range(args.steps)]
    wall = time.perf_counter() - t0
    ms = 1000.0 * sum(times) / len(times)
    value = 1000.0 / ms
    sample = (f"the full model: {layers} Llama-2-7B-shaped layers + embedding + lm_head, batch 1, KV cache filled "
              f"with seeded fp16 N(0,1) to context {CONTEXT}; {args.warmup} warm-up + {args.steps} timed greedy steps")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "steps_timed": args.steps,
            "layers_timed": layers, "scaled_from_layers": False, "timed_region_s": wall,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp32 (double accumulate)",
            "data": "synthetic", "config": config_block(world),
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": dec.O.num_threads(), "kind": "port",
                             "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "setup_s": dec.setup_s, "forge_py_cpu_recorded": forge_py_recorded()}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ roofline
def gemv_roofline(ctx, world, reps=8, rounds=10):
    """Time the fused dequant-GEMV alone on this rank's 7B shard shapes with
    cold L2 (each replay rotates over `reps` distinct weight copies per shape,
    > 2x L2).  The launches are captured in a CUDA graph on the library's
    stream (fg_qmatmul_into allocates nothing), so the events measure device
    time only.  Returns (algorithmic bytes per launch, ms per launch, detail)."""
    H, I, d = 4096, 11008, 128
    shapes = [((3 * 32 // world) * d, H), (H, 32 // world * d), (2 * I // world, H), (H, I // world)]
    stream = torch.cuda.ExternalStream(ctx.stream_ptr())
    total_bytes, total_ms, launches, per_shape = 0, 0.0, 0, []
    for si, (N, K) in enumerate(shapes):
        ws = [ctx.synth_quant("Q4_0", N, K, seed=1000 * si + r, std=0.02) for r in range(reps)]
        x = ctx.synth_normal((1, K), np.float32, seed=K)
        out = ctx.empty((1, N), np.float32)
        for w in ws:  # warm-up outside capture (sets kernel attributes)
            ctx.qmatmul_into(x, w, out)
        ctx.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for w in ws:
                ctx.qmatmul_into(x, w, out)
        with torch.cuda.stream(stream):
            g.replay()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(rounds):
                g.replay()
            e1.record()
        e1.synchronize()
        ms = e0.elapsed_time(e1)
        n = rounds * reps
        b = n * (N * K // 32 * 18 + 4 * (K + N))
        per_shape.append({"N": N, "K": K, "us_per_launch": 1000 * ms / n, "GBps": b / (ms / 1e3) / 1e9})
        total_bytes += b
        total_ms += ms
        launches += n
        del g
        for w in ws:
            ctx.dispose(w)
        ctx.dispose(x)
        ctx.dispose(out)
        ctx.synchronize()
    return total_bytes / launches, total_ms / launches, per_shape


def gemm_table(ctx, reps=8, rounds=10):
    """Dequant-GEMV/GEMM rows of the scope table: Q4_0 W [N, K] in {4096 x
    11008, 11008 x 4096} at batch 1/8/32/128, the Q8_0 4096 x 4096 GEMV at
    batch 1 and Q4_K / Q6_K GEMVs; W from N(0, 0.02) (k-quants: random super-blocks),
    x ~ N(0, 1).  Cold L2: every replay rotates
    over `reps` weight copies (more than L2 together).  Graph-captured
    launches on the library stream, CUDA-event timed."""
    stream = torch.cuda.ExternalStream(ctx.stream_ptr())
    peak_bw, _ = measured_peak()
    with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
        peak_tf = float(json.load(f).get("bf16_tflops", 1590.0))
    rows = []
    for (qt, N, K, batches) in [("Q4_0", 4096, 11008, (1, 8, 32, 128)), ("Q4_0", 11008, 4096, (1, 8, 32, 128)),
                                ("Q8_0", 4096, 4096, (1,)), ("Q4_K", 4096, 11008, (1, 4)), ("Q4_K", 11008, 4096, (1,)),
                                ("Q6_K", 4096, 11008, (1,)), ("Q6_K", 11008, 4096, (1,))]:
        if qt in ("Q4_K", "Q6_K"):  # random super-blocks with finite fp16 scales
            ws = []
            bb = 144 if qt == "Q4_K" else 210
            for r in range(reps):
                rng = np.random.default_rng(77 + r)
                b = rng.integers(0, 256, size=(N * K // 256, bb), dtype=np.uint8)
                dd = (rng.random(N * K // 256) * 1e-3 + 1e-4).astype(np.float16).view(np.uint8).reshape(-1, 2)
                if qt == "Q4_K":
                    b[:, 0:2], b[:, 2:4] = dd, dd
                else:
                    b[:, 208:210] = dd
                ws.append(ctx.upload_quant(qt, b, N, K))
        else:
            ws = [ctx.synth_quant(qt, N, K, seed=77 + r, std=0.02) for r in range(reps)]
        for M in batches:
            x = ctx.synth_normal((M, K), np.float32, seed=K + M)
            out = ctx.empty((M, N), np.float32)
            for w in ws:
                ctx.qmatmul_into(x, w, out)
            ctx.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                for w in ws:
                    ctx.qmatmul_into(x, w, out)
            with torch.cuda.stream(stream):
                g.replay()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(rounds):
                    g.replay()
                e1.record()
            e1.synchronize()
            us = 1000 * e0.elapsed_time(e1) / (rounds * reps)
            kq = {"Q4_K": 144, "Q6_K": 210}
            byt = (N * (K // 256) * kq[qt] if qt in kq else N * (K // 32) * (18 if qt == "Q4_0" else 34)) + \
                4 * M * (K + N)
            fl = 2.0 * M * N * K
            if qt in kq:
                kern = ("k_gemv_" + qt.lower().replace("_", "")) if M <= 8 else "dequant + k_matmul_f32"
            else:
                kern = "k_qgemv" if M <= 4 else ("k_qgemm_tc (tcgen05)" if qt == "Q4_0" else "k_qgemm_simt")
            rows.append({"qtype": qt, "N": N, "K": K, "batch": M, "kernel": kern,
                         "us": us, "GBps": byt / us / 1e3, "TFLOPs": fl / us / 1e6,
                         "hbm_frac": byt / us / 1e3 / peak_bw, "tensor_frac": fl / us / 1e6 / peak_tf})
            del g
            ctx.dispose(x)
            ctx.dispose(out)
        for w in ws:
            ctx.dispose(w)
        ctx.synchronize()
    # fp32 matmul (the reference's matmul / matmul_tiled and fp32 nn.Linear): tcgen05 tf32 with the
    # three-term split (3 MMA passes); useful flops 2 M N K, event-timed per call incl. the split pass
    for (M, K, N) in [(2048, 4096, 4096), (512, 4096, 11008)]:
        a = ctx.synth_normal((M, K), np.float32, seed=5)
        b = ctx.synth_normal((K, N), np.float32, seed=6)
        for _ in range(2):
            ctx.dispose(ctx.matmul(a, b))
        ctx.synchronize()
        with torch.cuda.stream(stream):  # outputs go back to the pool per call (one reused block)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(rounds):
                ctx.dispose(ctx.matmul(a, b))
            e1.record()
        e1.synchronize()
        us = 1000 * e0.elapsed_time(e1) / rounds
        fl = 2.0 * M * N * K
        rows.append({"qtype": "F32", "N": N, "K": K, "batch": M, "kernel": "k_tf32_split + k_matmul_tc (tcgen05 tf32 x3)",
                     "us": us, "TFLOPs": fl / us / 1e6, "tensor_frac": fl / us / 1e6 / peak_tf})
        for h in (a, b):
            ctx.dispose(h)
        ctx.synchronize()
    return rows


def gemm_case(ctx, spec, warmup, steps):
    """One Q4_0 GEMM shape, launched warmup + steps times on the library stream
    (for ncu captures: the first `warmup` launches are the ones to skip)."""
    M, N, K = (int(v) for v in spec.split(","))
    stream = torch.cuda.ExternalStream(ctx.stream_ptr())
    w = ctx.synth_quant("Q4_0", N, K, seed=77, std=0.02)
    x = ctx.synth_normal((M, K), np.float32, seed=K + M)
    out = ctx.empty((M, N), np.float32)
    for _ in range(warmup):
        ctx.qmatmul_into(x, w, out)
    with torch.cuda.stream(stream):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            ctx.qmatmul_into(x, w, out)
        e1.record()
    e1.synchronize()
    us = 1000 * e0.elapsed_time(e1) / steps
    for h in (w, x, out):
        ctx.dispose(h)
    return {"gemm_case": {"M": M, "N": N, "K": K}, "launches": warmup + steps, "us_per_launch": us,
            "TFLOPs": 2.0 * M * N * K / us / 1e6, "note": "two kernels per launch: k_x_to_f16, k_qgemm_tc"}


def attention_case(ctx, spec, warmup, steps):
    """Causal flash-attention prefill on seeded fp16 inputs [B, H, S, d], timed
    with CUDA events on the library stream (FLOPs = 4 B H S^2 d / 2)."""
    parts = spec.split(",")
    B, H, S, d = (int(v) for v in parts[:4])
    dt = np.float32 if len(parts) > 4 and parts[4] == "f32" else np.float16  # f32: the executeGraph path
    stream = torch.cuda.ExternalStream(ctx.stream_ptr())
    q, k, v = (ctx.synth_normal((B, H, S, d), dt, seed=SEED + i) for i in range(3))
    for _ in range(warmup):
        ctx.dispose(ctx.flashAttention(q, k, v, isCausal=True))
    # each output goes back to the stream-ordered pool right after its call, so every call reuses one
    # block instead of growing the pool (mapping fresh memory) inside the timed region
    with torch.cuda.stream(stream):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            ctx.dispose(ctx.flashAttention(q, k, v, isCausal=True))
        e1.record()
    e1.synchronize()
    ms = e0.elapsed_time(e1) / steps
    for h in (q, k, v):
        ctx.dispose(h)
    flops = 4.0 * B * H * S * S * d / 2
    with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
        peak_tf = float(json.load(f).get("bf16_tflops", 1590.0))
    return {"attention_case": {"B": B, "H": H, "S": S, "d": d, "causal": True,
                               "dtype": ("fp32" if dt == np.float32 else "fp16") + " in, fp32 out"},
            "calls": warmup + steps, "ms_per_call": ms, "TFLOPs": flops / ms / 1e9,
            "tensor_frac": flops / ms / 1e9 / peak_tf, "peak_TFLOPs": peak_tf,
            "path": os.environ.get("FORGE_B200_ATTN", "tcgen05")}


def decode_bytes(shape, batch, pos_mean):
    """Algorithmic DRAM bytes of one decode step of `batch` sequences at mean
    cache length pos_mean: every Q4_0 weight once, each sequence's fp16 K/V of
    keys [0, pos] read once and the new key/value written, norms, embedding
    rows, and each GEMV's input and output vectors per sequence."""
    H, I, V, L = shape["hidden_size"], shape["intermediate_size"], shape["vocab_size"], shape["num_hidden_layers"]
    hq, hkv = shape["num_attention_heads"], shape["num_key_value_heads"]
    d = H // hq
    gemvs = [((hq + 2 * hkv) * d, H), (H, hq * d), (2 * I, H), (H, I)]
    per_layer = sum(q4_bytes(n, k) + 4 * batch * (n + k) for n, k in gemvs) + 2 * H * 4
    per_layer += batch * (2 * hkv * d * 2 * (pos_mean + 1) + 2 * hkv * d * 2)
    head = q4_bytes(V, H) + 4 * batch * (V + H) + H * 4 + batch * H * 2
    return L * per_layer + head


def decode_table(local, steps, warmup):
    """Decode throughput of the scope table's decode rows on one GPU: random-
    init Q4_0 weights, cache length set to the context without a prefill (the
    zero-filled cache is read exactly as a filled one), greedy steps timed with
    CUDA events on the library stream."""
    import forge_b200
    from forge_b200.llama import LLAMA2_7B, TINYLLAMA_1_1B
    peak, _ = measured_peak()
    rows = []
    # largest first: the batch-64 cache alone is ~140 GB
    for name, shape, batch, ctx_len, n_steps in [("llama2-7b", LLAMA2_7B, 64, 4096, steps),
                                                  ("llama2-7b", LLAMA2_7B, 16, 4096, steps),
                                                  ("llama2-7b", LLAMA2_7B, 1, 4096, steps),
                                                  ("tinyllama-1.1b", TINYLLAMA_1_1B, 1, 2048, 256)]:
        torch.cuda.synchronize(local)
        free, _ = torch.cuda.mem_get_info(local)
        ctx = forge_b200.Context(device=local, vram_limit_bytes=int(free * 0.98))
        stream = torch.cuda.ExternalStream(ctx.stream_ptr())
        cap = ctx_len + warmup + n_steps + 8
        m = forge_b200.LlamaForCausalLM(forge_b200.LlamaConfig(max_position_embeddings=cap, max_batch=batch,
                                                               qtype="Q4_0", **shape), ctx)
        m.synthesize(SEED)
        m.set_position(batch, ctx_len)
        ids = (np.arange(batch, dtype=np.int32) * 7919 + 11) % shape["vocab_size"]
        m.decode(ids)  # seeds the device-side ids
        m.generate_device(batch, warmup, read=False)
        ctx.synchronize()
        with torch.cuda.stream(stream):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
        m.generate_device(batch, n_steps, read=False)
        with torch.cuda.stream(stream):
            e1.record()
        ctx.synchronize()
        ms = e0.elapsed_time(e1)
        pos_mean = ctx_len + 1 + warmup + (n_steps - 1) / 2.0
        byt = decode_bytes(shape, batch, pos_mean)
        sec = ms / 1e3 / n_steps
        rows.append({"decode": name, "batch": batch, "context": ctx_len, "steps": n_steps,
                     "tokens_per_s": batch * n_steps / (ms / 1e3), "ms_per_step": ms / n_steps,
                     "GBps": byt / sec / 1e9, "hbm_frac": byt / sec / 1e9 / peak,
                     "path": "persistent step kernel" if batch == 1 else "layered kernels (CUDA graph)",
                     "kv": "cache length set without a prefill (zero-filled keys/values, read in full)"})
        m.close()
        ctx.shutdown()
    return rows


def graph_decode(local, steps, warmup):
    """Decode through fg_execute_graph, as forge-py's model drives the reference (llama.py:211-248):
    one instruction list per token built by GraphLlama, the present keys/values passed on as handles.
    Wall-clock per token (the loop is host-synchronous: every step reads its logits)."""
    import time

    import forge_b200
    from forge_b200.graph_llama import GraphLlama
    from forge_b200.llama import TINYLLAMA_1_1B
    shape = dict(TINYLLAMA_1_1B)
    ctx = forge_b200.Context(device=local)
    m = GraphLlama(ctx, **shape)
    w = {}
    for i, name in enumerate(m.weight_names()):
        shp = m.weight_shape(name)
        if name == "embed":
            w[name] = ctx.synth_normal(shp, np.float16, seed=SEED + i, std=0.02)
        elif len(shp) == 1:
            w[name] = ctx.synth_normal(shp, np.float32, seed=SEED + i, mean=1.0, std=0.1)
        else:
            w[name] = ctx.synth_quant("Q4_0", shp[0], shp[1], seed=SEED + i)
    m.weights = w
    prompt = [int(t) for t in (np.arange(128) * 7919 + 11) % shape["vocab_size"]]
    m.generate(prompt, 1 + warmup)  # prefill + warm-up steps (a run of its own)
    ctx.synchronize()
    t0 = time.perf_counter()
    toks = m.generate(prompt, 1)  # prefill alone, subtracted below
    ctx.synchronize()
    t_prefill = time.perf_counter() - t0
    t0 = time.perf_counter()
    toks = m.generate(prompt, 1 + steps)
    ctx.synchronize()
    dt = time.perf_counter() - t0 - t_prefill
    g = forge_b200.GraphBuilder()
    m.forward(g, {}, np.array([prompt]), 0)
    n_pre = len(g.nodes)
    g = forge_b200.GraphBuilder()
    m.forward(g, {}, np.array([[1]]), len(prompt), [(1, 2, len(prompt))] * m.L)  # node count only
    nodes_step = len(g.nodes)
    for h in w.values():
        ctx.dispose(h)
    ctx.shutdown()
    return {"decode": "tinyllama-1.1b via executeGraph", "batch": 1, "context": len(prompt), "steps": steps,
            "tokens_per_s": steps / dt, "ms_per_step": dt / steps * 1e3, "prefill_ms": t_prefill * 1e3,
            "graph_nodes_per_step": nodes_step, "graph_nodes_prefill": n_pre,
            "path": "forge-py Llama graph JSON -> fg_execute_graph (transpose fold, Q4_0 fused GEMV, native GQA, "
                    "in-place KV append); host argmax per token", "tokens": len(toks)}


def ctx_stream(ctx):
    import ctypes
    from forge_b200 import _capi as C
    s = ctypes.c_void_p()
    C.call("fg_get_stream", ctx.ptr, ctypes.byref(s))
    return s.value


def measured_peak():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def q4_bytes(n, k):
    return n * (k // 32) * 18


def step_bytes(layers, pos_mean, world=1):
    """Algorithmic DRAM bytes of one batch-1 decode step (this rank's shard):
    every Q4_0 weight once, the fp16 KV cache of keys [0, pos] read once and
    the new key/value written, the norms, the embedding row and the
    activation vectors (each GEMV's input and output once)."""
    H, I, d = SHAPE["hidden_size"], SHAPE["intermediate_size"] // world, H_D
    hq, hkv, V = SHAPE["num_attention_heads"] // world, SHAPE["num_key_value_heads"] // world, SHAPE["vocab_size"] // world
    gemvs = [((hq + 2 * hkv) * d, H), (H, hq * d), (2 * I, H), (H, I)]
    per_layer = sum(q4_bytes(n, k) + 4 * (n + k) for n, k in gemvs)
    per_layer += 2 * H * 4                          # attn / ffn norm weights
    per_layer += 2 * hkv * d * 2 * (pos_mean + 1)   # K and V of keys [0, pos]
    per_layer += 2 * hkv * d * 2                    # the new key / value
    head = q4_bytes(V, H) + 4 * (V + H) + H * 4 + H * 2
    return layers * per_layer + head


H_D = 128


def ncu_traffic():
    """DRAM bytes per decode-step launch from the committed ncu summary, if any."""
    p = os.path.join(REPO, "profiles", "decode_step_7b_traffic.json")
    try:
        with open(p) as f:
            return json.load(f)
    except (OSError, ValueError):
        return None


def profile_case(args, local):
    """A 7B-shaped model of --profile-layers layers at context 4096: W + K
    decode steps through the same graph as the bench (for ncu captures of the
    decode-step kernel on a case that holds well under a GB on the device)."""
    import forge_b200
    ctx = forge_b200.Context(device=local)
    L = args.profile_layers
    shape = {**SHAPE, "num_hidden_layers": L}
    cap = CONTEXT + args.warmup + args.steps + 8
    model = forge_b200.LlamaForCausalLM(forge_b200.LlamaConfig(max_position_embeddings=cap, max_batch=1, qtype="Q4_0",
                                                               **shape), ctx)
    model.synthesize(SEED)
    prompt = np.random.default_rng(SEED).integers(0, SHAPE["vocab_size"], (1, CONTEXT), dtype=np.int32)
    model.forward(prompt, return_logits=False)
    model.generate_device(1, args.warmup + args.steps)
    ctx.synchronize()
    pos_mean = CONTEXT + args.warmup + (args.steps - 1) / 2.0
    print(json.dumps({"profile_case": f"{L} of 32 Llama-2-7B layers, context {CONTEXT}, batch 1",
                      "decode_steps": args.warmup + args.steps, "first_profiled_launch": args.warmup,
                      "algorithmic_bytes_per_launch": step_bytes(L, pos_mean),
                      "full_model_bytes_per_launch": step_bytes(SHAPE["num_hidden_layers"], pos_mean)}), flush=True)
    model.close()
    ctx.shutdown()


def main():
    args = parse()
    rank, world, local = dist_env()
    if world > 1 and not dist.is_initialized():
        torch.cuda.set_device(local)
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    if args.impl == "reference":
        run_reference(args, rank, world)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return

    import forge_b200
    if args.gemm_table:
        ctx = forge_b200.Context(device=local)
        for r in gemm_table(ctx):
            print(json.dumps(r), flush=True)
        ctx.shutdown()
        return
    if args.decode_table:
        for r in decode_table(local, args.steps, args.warmup):
            print(json.dumps(r), flush=True)
        return
    if args.graph_decode:
        print(json.dumps(graph_decode(local, args.steps, args.warmup)), flush=True)
        return
    if args.attention_case:
        ctx = forge_b200.Context(device=local)
        print(json.dumps(attention_case(ctx, args.attention_case, args.warmup, args.steps)), flush=True)
        ctx.shutdown()
        return
    if args.gemm_case:
        ctx = forge_b200.Context(device=local)
        print(json.dumps(gemm_case(ctx, args.gemm_case, args.warmup, args.steps)), flush=True)
        ctx.shutdown()
        return
    if args.roofline_only:
        ctx = forge_b200.Context(device=local)
        b_launch, ms_launch, per_shape = gemv_roofline(ctx, world)
        peak, _ = measured_peak()
        print(json.dumps({"kernel": "k_qgemv", "GBps": b_launch / (ms_launch / 1e3) / 1e9, "peak": peak,
                          "per_shape": per_shape}), flush=True)
        ctx.shutdown()
        return
    if args.profile_layers:
        profile_case(args, local)
        return
    nid = None
    if world > 1:
        obj = [forge_b200.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        nid = obj[0]
    ctx = forge_b200.Context(device=local, tp_rank=rank, tp_size=world, nccl_id=nid)
    cap = CONTEXT + args.warmup + 2 * args.steps + 8
    cfg = forge_b200.LlamaConfig(max_position_embeddings=cap, max_batch=BATCH, qtype="Q4_0", **SHAPE)
    model = forge_b200.LlamaForCausalLM(cfg, ctx)
    t0 = time.perf_counter()
    model.synthesize(SEED)
    t_synth = time.perf_counter() - t0
    rng = np.random.default_rng(SEED)
    prompt = rng.integers(0, SHAPE["vocab_size"], (BATCH, CONTEXT), dtype=np.int32)
    t0 = time.perf_counter()
    _, nxt = model.forward(prompt, return_logits=False)
    t_prefill = time.perf_counter() - t0

    stream = torch.cuda.ExternalStream(ctx_stream(ctx))
    model.generate_device(BATCH, args.warmup)  # warm-up steps (graph capture + W launches)
    ctx.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()

    # ---- value: device-resident decode loop ----
    barrier()
    ctx.synchronize()
    with Clocks(local) as clk:
        with torch.cuda.stream(stream):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
        model.generate_device(BATCH, args.steps, read=False)  # enqueues K graph launches
        with torch.cuda.stream(stream):
            e1.record()
        ctx.synchronize()
        ms = e0.elapsed_time(e1)
    toks = model.read_tokens(BATCH, args.steps)
    barrier()
    t = torch.tensor([ms], dtype=torch.float64, device=f"cuda:{local}")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    value = args.steps * BATCH / (ms / 1e3)

    # ---- e2e: public API with host buffers, one call per step ----
    ids = np.asarray(toks[-1], np.int32).copy()
    barrier()
    ctx.synchronize()
    with torch.cuda.stream(stream):
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record()
    for _ in range(args.steps):
        ids = model.decode(ids)  # H2D of the ids, graph launch, D2H of the next ids
    with torch.cuda.stream(stream):
        f1.record()
    ctx.synchronize()
    ms_e2e = f0.elapsed_time(f1)
    t = torch.tensor([ms_e2e], dtype=torch.float64, device=f"cuda:{local}")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_value = args.steps * BATCH / (float(t.item()) / 1e3)

    # ---- roofline of the dominant kernel ----
    b_launch, ms_launch, per_shape = gemv_roofline(ctx, world)
    peak, peak_kind = measured_peak()
    step_kernel = world == 1 and os.environ.get("FORGE_B200_DECODE", "") != "layered"
    pos_mean = CONTEXT + args.warmup + (args.steps - 1) / 2.0
    if step_kernel:
        alg = step_bytes(SHAPE["num_hidden_layers"], pos_mean)
        roof = {"bound": "hbm", "kernel": "k_decode_step (persistent decode step: Q4_0 GEMVs + split-KV attention)",
                "achieved": alg / (ms / args.steps / 1e3) / 1e9, "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                "algorithmic_bytes_per_launch": alg, "us_per_launch": 1e3 * ms / args.steps,
                "launches_per_step": 1,
                "gemv_alone": {"GBps": b_launch / (ms_launch / 1e3) / 1e9, "per_shape": per_shape}}
    else:
        roof = {"bound": "hbm", "kernel": "k_qgemv (fused Q4_0 dequant-GEMV)",
                "achieved": b_launch / (ms_launch / 1e3) / 1e9, "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                "algorithmic_bytes_per_launch": b_launch, "us_per_launch": ms_launch * 1e3, "per_shape": per_shape}
    roof["frac"] = roof["achieved"] / peak
    traffic = ncu_traffic() if step_kernel else None
    # ncu dram bytes per launch: measured on a 2-layer launch, scaled by the bytes streamed
    roof["traffic"] = traffic["traffic_over_algorithmic"] * roof["algorithmic_bytes_per_launch"] if traffic else None

    model.close()
    ctx.shutdown()
    cpu = None
    if rank == 0 and world == 1 and args.cpu_baseline:
        cpu = cpu_sample()
    if rank == 0:
        L = SHAPE["num_hidden_layers"]
        launches = args.steps if step_kernel else (5 * L + 4 + (3 if world > 1 else 0)) * args.steps
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "q4_0 x int8-digit MMA, fp32 accumulate", "data": "synthetic",
            "config": config_block(world),
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": 4 * BATCH,
                    "d2h_bytes_per_step": 4 * BATCH},
            "roofline": roof,
            "cpu_baseline": cpu, "clocks": clk.summary(), "gpu_launches": launches,
            "setup": {"synthesize_s": t_synth, "prefill_s": t_prefill, "prefill_tokens": CONTEXT * BATCH},
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
