"""LLaMA-2-7B fp16 batch-1 decode benchmark of the vkllm-b200 C-ABI library.

Workload: LLaMA-2-7B architecture (dim 4096, 32 layers, 32 heads of 128, SwiGLU 11008, vocab 32000,
context 4096), fp16 weights random-initialised on the device (N(0, 0.02) counter-based generator;
no checkpoint or dataset exists here, the data is synthetic), a 512-token seeded prompt prefilled
through the drop-in API, then greedy decode. One bench "step" = one decode token at batch 1.

  value : decode tok/s with the token feedback on the device (CUDA-Graph replay of the fused step),
          timed with CUDA events on the library's stream; weights (13.2 GB) exceed L2, so every step
          streams them from HBM.
  e2e   : the same metric through the reference token loop of the C API
          (tests/vkllm_test_infer_gguf.c:181-272): per token a new mapped input tensor (host write),
          vkllm_graph_new / vkllm_models_llama2_build_graph / init / upload / run / post_run, read of
          the mapped output (device -> host), vkllm_graph_free.
  N > 1 : one process per GPU (torchrun), each decoding its own independent sequence (data
          parallel, weak scaling); value = total tokens / max-over-ranks time.

--impl reference runs the reference's algorithm on the host cores instead: the C++ oracle
(oracle/, the CPU restatement of the reference shaders) on the same weights, because the reference
itself (Vulkan) cannot run on these machines.
"""
import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "vkllm.c_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

CFG_7B = dict(block_count=32, context_length=4096, embedding_length=4096, head_count=32, ffn_length=11008,
              vocab_size=32000, rope_freq_base=10000.0, rms_eps=1e-5, init_std=0.02)
PROMPT_LEN = 512
SEED = 2024


def weight_bytes(cfg):
    D, F, V, L = cfg["embedding_length"], cfg["ffn_length"], cfg["vocab_size"], cfg["block_count"]
    per_layer = (4 * D * D + 3 * F * D) * 2 + 2 * D * 4
    return L * per_layer + V * D * 2 + D * 4 + D * 2  # layers + logits matrix + output norm + 1 embedding row


def kv_bytes(cfg, lk):
    D, L = cfg["embedding_length"], cfg["block_count"]
    return L * 2 * D * 2 * lk  # K and V rows read per layer


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d.get("hbm_gbs", 6650.0), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clock/throttle sampling during the timed region (a read-only query every 20 ms into a
    temporary file). Entering waits, up to 3 s, for the first sample, so that a timed region of a few
    tens of milliseconds is still covered."""

    def __init__(self, gpu):
        import tempfile

        self.gpu = gpu
        self.proc = None
        fd, self.path = tempfile.mkstemp(prefix=f"vkllm_clocks_gpu{gpu}_", suffix=".csv")
        os.close(fd)

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                          "-lms", "20"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
            return self
        t0 = time.time()
        while time.time() - t0 < 3.0 and os.path.getsize(self.path) == 0 and self.proc.poll() is None:
            time.sleep(0.01)
        return self

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.f.close()
        self.rows = []
        try:
            with open(self.path) as f:
                for line in f:
                    parts = [p.strip() for p in line.split(",")]
                    if len(parts) >= 9:
                        self.rows.append(parts)
            os.unlink(self.path)
        except OSError:
            pass

    def summary(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = self.rows
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(world, v):
    if world == 1:
        return v
    import torch
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def prompt_tokens(rank, n=PROMPT_LEN):
    import numpy as np

    return np.random.default_rng(SEED + 1000 * rank).integers(3, 32000, size=n, dtype=np.uint32)


def download_weights(vk, ctx, model, cfg):
    """Copies the model's weights to host numpy arrays (for the CPU oracle)."""
    import numpy as np

    w = {}
    m = model.m.weights
    w["token_embd.weight"] = vk.fetch(ctx, m.tok_embed_weights).reshape(cfg["vocab_size"], -1)
    w["output.weight"] = vk.fetch(ctx, m.output_weight).reshape(cfg["vocab_size"], -1)
    w["output_norm.weight"] = vk.fetch(ctx, m.output_norm_weight).reshape(-1)
    names = {"attn_norm_weight": "attn_norm", "ffn_norm_weight": "ffn_norm", "WQ": "attn_q", "WK": "attn_k",
             "WV": "attn_v", "WO": "attn_output", "WG": "ffn_gate", "WU": "ffn_up", "WD": "ffn_down"}
    for l in range(cfg["block_count"]):
        bw = model.block(l)
        for f, n in names.items():
            a = vk.fetch(ctx, getattr(bw, f))
            w[f"blk.{l}.{n}.weight"] = a.reshape(-1) if "norm" in n else a.reshape(a.shape[2], a.shape[3])
    return w


def cpu_decode_sample(weights, cfg, n_steps=3, threads=0, prompt=None):
    """Times n single-token decode steps of the oracle (reference algorithm on the CPU). With a
    prompt, the steps run at positions len(prompt) .. len(prompt)+n-1 after an untimed prefill of
    it (the GPU arm's configuration); without one, at positions 1..n. Returns (tok/s, threads used,
    prefill seconds or None, the greedy tokens: the prefill's prediction then one per step)."""
    import oracle

    used = oracle.threads(threads or os.cpu_count() or 1)
    start = len(prompt) if prompt is not None else 1
    ctx = start + n_steps + 8
    ocfg = dict(D=cfg["embedding_length"], H=cfg["head_count"], F=cfg["ffn_length"], V=cfg["vocab_size"],
                L=cfg["block_count"], ctx=ctx, eps=cfg["rms_eps"], rope_base=cfg["rope_freq_base"])
    m = oracle.Llama2(ocfg, weights, ctx=ctx)
    prefill_s = None
    if prompt is not None:
        t0 = time.perf_counter()
        _, out = m.step(list(prompt), 0)
        prefill_s = time.perf_counter() - t0
        tok = int(out[-1])
    else:
        tok = 1
        m.step([tok], 0)  # warm-up (page-in)
    toks = [tok]
    t0 = time.perf_counter()
    for i in range(n_steps):
        _, out = m.step([tok], start + i)
        tok = int(out[-1])
        toks.append(tok)
    dt = time.perf_counter() - t0
    m.close()
    return n_steps / dt, used, prefill_s, toks


def prefill_gemm_roofline(vk, l, model, cfg, stream):
    """Times the prefill GEMM shapes (M = prompt length) of one layer and the logits on the tensor-core
    GEMM (vkllm_b200_gemm_f16) with the model's weights as B; TF/s against MEASURED_PEAKS bf16 burst."""
    import torch

    D, F, V = cfg["embedding_length"], cfg["ffn_length"], cfg["vocab_size"]
    bw = model.block(0)
    # The fused prefill runs Q/K/V and up/gate as one grouped GEMM each (N = 3 D and 2 F); a
    # contiguous seeded B of that height stands in for the three (two) weight blocks, same tiles.
    shapes = {"qkv grouped (12288x4096)": (None, 3 * D, D), "wo (4096x4096)": (bw.WO, D, D),
              "up/gate grouped (22016x4096)": (None, 2 * F, D), "down (4096x11008)": (bw.WD, D, F),
              "logits (32000x4096)": (model.m.weights.output_weight, V, D)}
    peak = 1656.1
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            peak = json.load(f).get("bf16_tflops", peak)
    out = {}
    M = PROMPT_LEN
    g = torch.Generator(device="cuda").manual_seed(11)
    for name, (w, N, K) in shapes.items():
        A = (torch.rand((M, K), generator=g, device="cuda") * 0.2 - 0.1).half()
        Cm = torch.empty((M, N), device="cuda", dtype=torch.float16)
        Bt = (torch.randn((N, K), generator=g, device="cuda") * 0.02).half() if w is None else None
        B = Bt.data_ptr() if w is None else w.contents.data.dev
        args = (A.data_ptr(), B, Cm.data_ptr(), M, N, K, K, K, N, 1.0, 0, stream.cuda_stream)
        for _ in range(3):
            vk.check(l.vkllm_b200_gemm_f16(*args), "gemm")
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n = 10
        e0.record(stream)
        for _ in range(n):
            l.vkllm_b200_gemm_f16(*args)
        e1.record(stream)
        e1.synchronize()
        us = e0.elapsed_time(e1) * 1000.0 / n
        tf = 2.0 * M * N * K / (us * 1e-6) / 1e12
        out[name] = {"M": M, "N": N, "K": K, "us": round(us, 2), "tflops": round(tf, 1), "frac": round(tf / peak, 4)}
    if l.vkllm_b200_gemm_f16_error() != 0:
        raise RuntimeError("tensor-core GEMM reported a timed-out wait")
    out["peak_tflops"] = peak
    out["peak_source"] = "MEASURED_PEAKS.json bf16_tflops (burst)"
    return out


def host_graph_cost(vk, ctx, model, pos, n=200):
    """Host time per token of the reference loop's graph handling (tests/vkllm_test_infer_gguf.c:181-272)
    without the device step: input tensor_new + graph_new + build_graph + graph_init, then graph_free,
    with the structural graph cache on and off. Microseconds per token (median of 5 blocks of n),
    measured around the ctypes calls (each adds ~0.1-0.3 us of Python overhead)."""
    import ctypes as C

    l = vk.lib()
    out = {}
    for on in (True, False):
        ctx.set_graph_cache(on)
        blocks = []
        for _ in range(6):
            t_build = t_free = 0
            for i in range(n):
                t0 = time.perf_counter_ns()
                inp = vk.tensor_new(ctx, "input_toks", (1, 1, 1, 1), vk.U32, mapped=True)
                g = C.POINTER(vk.Graph)()
                vk.check(l.vkllm_graph_new(ctx.ptr, C.byref(g)), "graph_new")
                vk.check(l.vkllm_models_llama2_build_graph(ctx.ptr, C.byref(model.m), inp, g, pos + i % 64),
                         "build_graph")
                vk.check(l.vkllm_graph_init(ctx.ptr, g), "graph_init")
                t1 = time.perf_counter_ns()
                l.vkllm_graph_free(ctx.ptr, g)
                t2 = time.perf_counter_ns()
                t_build += t1 - t0
                t_free += t2 - t1
            blocks.append((t_build / n / 1e3, t_free / n / 1e3))
        blocks = sorted(blocks[1:], key=lambda b: b[0] + b[1])  # the first block warms the cache
        b, f = blocks[len(blocks) // 2]
        out["cache_on" if on else "cache_off"] = {"build_init_us": round(b, 2), "free_us": round(f, 2),
                                                  "total_us": round(b + f, 2)}
    ctx.set_graph_cache(True)
    return out


def batched_decode_leg(vk, model, args, world, rank, stream):
    """64 independent sequences with their own 128-token seeded prompts, greedy
    decode on the tensor-core GEMM path, sequences split evenly over the ranks (data parallel).
    Returns aggregate tokens/s over all ranks (max-over-ranks device time)."""
    import numpy as np
    import torch

    n_local = max(1, args.batch_seqs // world)
    P, cap = 128, 384
    rng = np.random.default_rng(SEED + 7)
    prompts = [rng.integers(3, 32000, size=P, dtype=np.uint32) for _ in range(args.batch_seqs)]
    mine = prompts[rank * n_local:(rank + 1) * n_local]
    b = vk.Batch(model, len(mine), cap)
    try:
        for i, p in enumerate(mine):
            b.add_prompt(i, p)
        b.decode(3)  # warm-up (graph capture) at positions 128..130
        K = args.batch_steps
        barrier(world)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if args.profile_batched:  # a profiler started with --profile-from-start off sees the timed steps only
            torch.cuda.profiler.start()
        e0.record(stream)
        b.decode(K)
        e1.record(stream)
        e1.synchronize()
        if args.profile_batched:
            torch.cuda.profiler.stop()
        ms = max_over_ranks(world, e0.elapsed_time(e1))
    finally:
        b.free()
    cfg = dict(CFG_7B)
    if args.layers:  # profiling case with fewer layers
        cfg["block_count"] = args.layers
    D, L = cfg["embedding_length"], cfg["block_count"]
    mean_lk = P + 3 + (K + 1) / 2.0
    step_bytes = weight_bytes(cfg) + n_local * L * 2 * D * 2 * mean_lk
    peak, _ = measured_peaks()
    return {"sequences": n_local * world, "per_rank": n_local, "steps": K, "prompt": P, "kv_rows": cap,
            "tok_s": round(n_local * world * K / (ms / 1000.0), 1), "ms_per_step": round(ms / K, 4),
            "hbm_frac_per_rank": round(step_bytes / (ms / K * 1e-3) / 1e9 / peak, 4),
            "path": "tcgen05 GEMMs (M = sequences per rank) on tile-order weight copies ([Wq;Wk;Wv], [Wup;Wgate], Wo, "
                    "Wdown, output), launched as programmatic dependents; split-K partials summed by the consumer "
                    "kernels (RoPE/KV rows, gate, residual + RMSNORM); bulk-copy staged attention; CUDA graph per step"}


def ops_microbench(vk, local, seed):
    """the operator microbenchmarks, each op run through the reference's op API
    (tensor_new -> upload -> op init -> run on a commands object -> submit/wait), timed by the
    per-launch CUDA events of the op executor (VKLLM_NODE_TIMING=1 on a context of its own). L2 is
    flushed before every timed run: a 256 MB write, then a 256 MB read of another buffer that evicts
    the written lines (so their write-back is not charged to the op), both on the op's stream and
    queued just before it;
    the median of 5 runs is reported. Bytes are the
    algorithmic bytes of the call (inputs read once, outputs written once); MATMUL at M = 512 is
    reported in TF/s against the tensor-core peak, everything else in GB/s against the HBM peak."""
    import ctypes as C

    import numpy as np
    import torch

    os.environ["VKLLM_NODE_TIMING"] = "1"
    try:
        ctx = vk.Context(local)
    finally:
        os.environ.pop("VKLLM_NODE_TIMING", None)
    hbm, _ = measured_peaks()
    tc = tc_peak()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=torch.device("cuda", local))
    flush_rd = torch.ones(64 << 20, dtype=torch.float32, device=torch.device("cuda", local))
    cstream = torch.cuda.ExternalStream(ctx.stream, device=torch.device("cuda", local))
    rng = np.random.default_rng(seed + 11)
    lib = vk.lib()
    out = {}
    live = []

    def tensor(name, arr, dt):
        t = vk.tensor_new(ctx, name, arr.shape, dt)
        vk.put(ctx, t, arr)
        live.append(t)
        return t

    def node(name, shape, dt, op, srcs, params):
        t = vk.tensor_new(ctx, name, shape, dt, op=op, srcs=srcs, params=params)
        live.append(t)
        return t

    def timed(n, op):
        init_fn, run_fn = f"vkllm_op_{op}_init", f"vkllm_op_{op}_run"
        vk.run_op(ctx, n, init_fn, run_fn)  # init + a first run (GEMM tuning happens here)
        cmd = vk.Commands(ctx)
        ts = []
        try:
            for _ in range(5):
                # the flush runs on the op's own (the context's) stream with no host wait, so the GPU
                # is still busy with it while the op's events and kernels are enqueued: the event pair
                # then brackets the op's kernels only, not the host's launch latency
                with torch.cuda.stream(cstream):
                    flush.zero_()
                    flush_rd.sum()
                cmd.begin()
                vk.check(getattr(lib, run_fn)(ctx.ptr, cmd.ptr, n), run_fn)
                cmd.end()
                cmd.submit_wait()
                ns = C.c_uint64()
                vk.check(lib.vkllm_pipeline_query_exec_time(ctx.ptr, n.contents.pipeline, C.byref(ns)), "exec_time")
                ts.append(ns.value / 1e3)
        finally:
            cmd.close()
        return float(np.median(ts))

    def report(key, us, nbytes, flops=None):
        r = {"us": round(us, 2), "GBps": round(nbytes / (us * 1e-6) / 1e9, 1),
             "hbm_frac": round(nbytes / (us * 1e-6) / 1e9 / hbm, 4)}
        if flops is not None:
            r["tflops"] = round(flops / (us * 1e-6) / 1e12, 1)
            r["tc_frac"] = round(flops / (us * 1e-6) / 1e12 / tc, 4)
        out[key] = r

    try:
        for M in (1, 8, 64, 512):
            for N, K in ((4096, 4096), (11008, 4096), (4096, 11008)):
                a = rng.uniform(-1, 1, (1, 1, M, K)).astype(np.float16)
                b = rng.uniform(-1, 1, (1, 1, N, K)).astype(np.float16)
                A, B = tensor("A", a, vk.F16), tensor("B", b, vk.F16)
                n = node("C", (1, 1, M, N), vk.F16, vk.OP_MATMUL, [A, B], bytes(C.c_float(1.0)) + bytes(C.c_int32(0)))
                report(f"matmul_M{M}_N{N}_K{K}", timed(n, "matmul"), 2 * (N * K + M * K + M * N),
                       2.0 * M * N * K if M == 512 else None)
                for t in (n, A, B):
                    vk.tensor_free(ctx, t)
                    live.remove(t)
        x = rng.uniform(-1, 1, (1, 1, 512, 4096)).astype(np.float16)
        g = rng.uniform(0.5, 1.5, (1, 1, 1, 4096)).astype(np.float32)
        X, G = tensor("x", x, vk.F16), tensor("g", g, vk.F32)
        n = node("y", x.shape, vk.F16, vk.OP_RMSNORM, [X, G], bytes(C.c_float(2.0)) + bytes(C.c_float(1e-5)))
        report("rmsnorm_512x4096", timed(n, "rmsnorm"), 2 * x.nbytes + g.nbytes)
        q = rng.uniform(-1, 1, (1, 32, 512, 128)).astype(np.float16)
        Q = tensor("q", q, vk.F16)
        rope = bytes(C.c_uint32(0)) + bytes(C.c_float(10000.0)) + bytes(C.c_bool(False)) + bytes(3)
        n = node("rq", q.shape, vk.F16, vk.OP_ROPE, [Q], rope)
        report("rope_1x32x512x128", timed(n, "rope"), 2 * q.nbytes)
        sc = rng.uniform(-4, 4, (1, 32, 1, 4096)).astype(np.float16)
        S = tensor("s", sc, vk.F16)
        n = node("p", sc.shape, vk.F16, vk.OP_SOFTMAX, [S], bytes(C.c_int32(1)) + bytes(C.c_uint32(4095)))
        report("softmax_32x1x4096", timed(n, "softmax"), 2 * sc.nbytes)
        src = rng.uniform(-1, 1, (1, 32, 1, 128)).astype(np.float16)
        Sr = tensor("src", src, vk.F16)
        n = node("cache", (1, 32, 4096, 128), vk.F16, vk.OP_UPDATE_ROWS, [Sr], bytes(C.c_uint32(100)))
        report("update_rows_1_into_32x4096x128", timed(n, "update_rows"), 2 * src.nbytes)
        table = rng.uniform(-1, 1, (1, 1, 32000, 4096)).astype(np.float16)
        ids = rng.integers(0, 32000, size=(1, 1, 1, 512), dtype=np.uint32)
        T, I = tensor("E", table, vk.F16), tensor("ids", ids, vk.U32)
        n = node("emb", (1, 1, 512, 4096), vk.F16, vk.OP_EMBEDDING, [I, T], bytes(C.c_uint32(0)))
        report("embedding_512_of_32000x4096", timed(n, "embedding"), 2 * 512 * 4096 * 2 + ids.nbytes)
        lg = rng.uniform(-8, 8, (1, 1, 1, 32000)).astype(np.float32)
        Lg = tensor("l", lg, vk.F32)
        n = node("am", (1, 1, 1, 1), vk.U32, vk.OP_ARG_MAX, [Lg], None)
        report("arg_max_32000_f32", timed(n, "arg_max"), lg.nbytes + 4)
    finally:
        for t in live:
            vk.tensor_free(ctx, t)
        del flush, flush_rd
        ctx.close()
    return out


def tc_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"])
    except Exception:
        return 1590.0


CFG_13B = dict(block_count=40, context_length=4096, embedding_length=5120, head_count=40, ffn_length=13824,
               vocab_size=32000, rope_freq_base=10000.0, rms_eps=1e-5, init_std=0.02)


def tp13b_leg(vk, ctx, args, world, rank, stream, exchange="peer"):
    """LLaMA-2-13B, tensor parallel over the ranks (heads / FFN rows / vocabulary
    sharded; the Wo and down partial sums exchanged inside the persistent decode kernel over peer
    memory). Batch-1 greedy decode at positions 2048.. (the prompt length of the config); the KV rows
    before 2048 are the zeroed cache, since only decode throughput is measured here (a 2048-token TP
    prefill is not part of this leg). Returns tokens/s (max-over-ranks device time)."""
    import ctypes as C

    import numpy as np
    import torch
    import torch.distributed as dist

    cfg = dict(CFG_13B)
    l = vk.lib()
    m = vk.Model(ctx)
    if world > 1:
        m.init_random_tp(cfg, SEED, rank, world)

        def gather(b):
            got = [None] * world
            dist.all_gather_object(got, b)
            return got

        if exchange == "nccl":
            m.tp_connect_nccl(gather)
        else:
            m.tp_connect(gather)
    else:
        m.init_random(cfg, SEED)
    try:
        P, K, W = 2048, args.tp_steps, 3
        vk.check(l.vkllm_b200_engine_set_state(ctx.ptr, C.byref(m.m), 1, P), "set_state")
        vk.check(l.vkllm_b200_engine_decode_steps(ctx.ptr, C.byref(m.m), W), "warmup")
        torch.cuda.synchronize()
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        vk.check(l.vkllm_b200_engine_decode_steps(ctx.ptr, C.byref(m.m), K), "decode")
        e1.record(stream)
        e1.synchronize()
        toks = np.zeros(W + K, dtype=np.uint32)
        vk.check(l.vkllm_b200_engine_read_tokens(ctx.ptr, C.byref(m.m), toks.ctypes.data, W + K), "tokens")
        ms = max_over_ranks(world, e0.elapsed_time(e1))
        persistent = bool(l.vkllm_b200_engine_is_persistent(ctx.ptr, C.byref(m.m)))
    finally:
        m.free()
    D, F, V, L = cfg["embedding_length"], cfg["ffn_length"], cfg["vocab_size"], cfg["block_count"]
    w_rank = (L * ((4 * D * D + 3 * F * D) * 2) + V * D * 2) / world + L * 2 * D * 4 + D * 4 + D * 2
    mean_lk = P + W + (K + 1) / 2.0
    kv_rank = L * 2 * D * 2 * mean_lk / world
    peak, _ = measured_peaks()
    ms_tok = ms / K
    return {"model": "llama2-13b-arch", "tp": world, "tok_s": round(K / (ms / 1000.0), 2),
            "ms_per_token": round(ms_tok, 4), "positions": [P + W, P + W + K],
            "bytes_per_token_per_rank": int(w_rank + kv_rank),
            "hbm_frac_per_rank": round((w_rank + kv_rank) / (ms_tok * 1e-3) / 1e9 / peak, 4),
            "exchange": exchange if world > 1 else "none",
            "allreduce": ("none (1 GPU)" if world == 1 else
                          "fused in the decode kernel: per layer 2 x D fp32 row partials over NVLink peer memory"
                          if exchange == "peer" else
                          "ncclAllReduce (fp32 sum, D rows) after Wo and after down, ncclAllGather of the argmax "
                          "candidates, between the per-op kernels of a CUDA-graph step"),
            "path": "persistent kernel" if persistent else "graph", "kv": "zeroed cache below position 2048 (decode-only leg)"}


def run_ours(args, world, rank, local):
    import numpy as np
    import torch

    import vkllm_b200 as vk

    if args.profile_tp:
        ctx = vk.Context(local)
        stream = torch.cuda.ExternalStream(ctx.stream, device=torch.device("cuda", local))
        for exchange in (("peer", "nccl") if world > 1 else ("peer",)):
            tp = tp13b_leg(vk, ctx, args, world, rank, stream, exchange)
            if rank == 0:
                print(json.dumps({"profile_case": "tp13b", **tp}), flush=True)
        ctx.close()
        return None
    cfg = dict(CFG_7B)
    if args.layers:
        cfg["block_count"] = args.layers
    ctx = vk.Context(local)
    model = vk.Model(ctx).init_random(cfg, SEED)
    l = vk.lib()
    stream = torch.cuda.ExternalStream(ctx.stream, device=torch.device("cuda", local))
    prompt = prompt_tokens(rank)
    if args.profile_prefill:
        times = []
        for _ in range(3):
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            tok = model.step(list(prompt), 0)
            e1.record(stream)
            e1.synchronize()
            times.append(e0.elapsed_time(e1))
        if rank == 0:
            print(json.dumps({"profile_case": "prefill", "layers": cfg["block_count"], "tokens": PROMPT_LEN,
                              "ms": [round(t, 3) for t in times], "token": tok}), flush=True)
        model.free()
        ctx.close()
        return None
    if args.profile_batched:
        batched = batched_decode_leg(vk, model, args, world, rank, stream)
        if rank == 0:
            print(json.dumps({"profile_case": "batched", "layers": cfg["block_count"], **batched}), flush=True)
        model.free()
        ctx.close()
        return None

    # Prefill through the drop-in API (timed separately, reported as prefill tok/s): one untimed
    # warm-up prefill (first-use costs: kernel attributes, tensor maps, allocator growth), then the
    # timed one over the same prompt and positions (it rewrites the same KV rows).
    if args.no_extras:  # profiling case: skip the prefill graph; decode starts at position PROMPT_LEN anyway
        first, prefill_s = int(prompt[-1]), float("nan")
    else:
        model.step(list(prompt), 0)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        first = model.step(list(prompt), 0)
        torch.cuda.synchronize()
        prefill_s = time.perf_counter() - t0
    model.engine_prepare()
    kps = l.vkllm_b200_engine_kernels_per_step(ctx.ptr, C.byref(model.m))

    # ---- value: device-resident decode loop --------------------------------------------------
    W, K = args.warmup, args.steps
    vk.check(l.vkllm_b200_engine_set_state(ctx.ptr, C.byref(model.m), first, PROMPT_LEN), "set_state")
    vk.check(l.vkllm_b200_engine_decode_steps(ctx.ptr, C.byref(model.m), W), "warmup")
    torch.cuda.synchronize()
    barrier(world)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        torch.cuda.synchronize()
        ev0.record(stream)
        vk.check(l.vkllm_b200_engine_decode_steps(ctx.ptr, C.byref(model.m), K), "decode_steps")
        ev1.record(stream)
        ev1.synchronize()
        torch.cuda.synchronize()
    dev_ms = ev0.elapsed_time(ev1)
    persistent = bool(l.vkllm_b200_engine_is_persistent(ctx.ptr, C.byref(model.m)))
    launches = int(l.vkllm_b200_engine_last_launches(ctx.ptr, C.byref(model.m)))
    toks = np.zeros(W + K, dtype=np.uint32)
    vk.check(l.vkllm_b200_engine_read_tokens(ctx.ptr, C.byref(model.m), toks.ctypes.data, W + K), "read_tokens")
    barrier(world)
    t_max = max_over_ranks(world, dev_ms)
    value = world * K / (t_max / 1000.0)

    if args.no_extras:
        if rank == 0:
            print(json.dumps({"profile_case": True, "layers": cfg["block_count"], "steps": K, "warmup": W,
                              "ms_per_step": round(t_max / K, 4), "persistent": persistent, "launches": launches}),
                  flush=True)
        model.free()
        ctx.close()
        return None

    # ---- dominant-kernel roofline (FFN up/gate GEMV, the largest weight stream of a step) --------
    us, nbytes = C.c_float(), C.c_uint64()
    vk.check(l.vkllm_b200_engine_bench_kernel(ctx.ptr, C.byref(model.m), b"upgate", 64, C.byref(us),
                                              C.byref(nbytes)), "bench_kernel")
    kern = {}
    for name in (b"qkv", b"wo", b"down", b"logits"):
        u2, b2 = C.c_float(), C.c_uint64()
        vk.check(l.vkllm_b200_engine_bench_kernel(ctx.ptr, C.byref(model.m), name, 32, C.byref(u2), C.byref(b2)), "k")
        kern[name.decode()] = {"us": round(u2.value, 2), "GBps": round(b2.value / (u2.value * 1e-6) / 1e9, 1)}

    # ---- prefill GEMMs on the tensor cores (tcgen05), on the model's own weights --------------------
    prefill_gemms = prefill_gemm_roofline(vk, l, model, cfg, stream)

    # ---- batched decode: 64 sequences split over the ranks -------------------
    batched = None
    if args.batch_seqs > 0:
        batched = batched_decode_leg(vk, model, args, world, rank, stream)

    # ---- host cost of the per-token graph rebuild (no device work) ---------------------------------
    host_cost = host_graph_cost(vk, ctx, model, PROMPT_LEN + W + K)

    # ---- e2e: reference token loop through the C API, host buffers --------------------------------
    pos = PROMPT_LEN + W + K
    tok = int(toks[-1])
    n_e2e = max(2, min(K, 64))
    for _ in range(2):  # warm the per-step allocations
        tok = model.step([tok], pos)
        pos += 1
    # (1) the loop in native code (vkllm_b200_token_loop: the reference loop's calls, one graph per
    # token); (2) the same calls made one by one from Python through ctypes (Model.step)
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    w0 = time.perf_counter()
    e0.record(stream)
    toks_native, host_us = model.token_loop([tok], pos, n_e2e)
    e1.record(stream)
    e1.synchronize()
    wall_e2e = time.perf_counter() - w0
    pos += n_e2e
    tok = toks_native[-1]
    e2e_ms = max(e0.elapsed_time(e1), wall_e2e * 1000.0)
    e2e_max = max_over_ranks(world, e2e_ms)
    e2e_value = world * n_e2e / (e2e_max / 1000.0)
    torch.cuda.synchronize()
    barrier(world)
    w0 = time.perf_counter()
    for _ in range(n_e2e):
        tok = model.step([tok], pos)
        pos += 1
    torch.cuda.synchronize()
    e2e_py_max = max_over_ranks(world, (time.perf_counter() - w0) * 1000.0)
    e2e_py_value = world * n_e2e / (e2e_py_max / 1000.0)

    result = None
    if rank == 0:
        peak, peak_kind = measured_peaks()
        mean_lk = PROMPT_LEN + W + (K + 1) / 2.0
        step_bytes = weight_bytes(cfg) + kv_bytes(cfg, mean_lk)
        ms_step = t_max / K
        if persistent:
            # The dominant kernel is the persistent decode kernel itself: one launch runs K / launches
            # whole decode steps (all weights + the KV rows of every step).
            steps_per_launch = K / max(launches, 1)
            rl_bytes = step_bytes * steps_per_launch
            rl_us = t_max * 1000.0 / max(launches, 1)
            rl_kernel = "k_decode_persistent (whole decode steps: rmsnorm, QKV+RoPE+KV write, attention, Wo, up/gate+SiLU, down, logits, argmax)"
            prof = os.path.join(ROOT, "profiles", "decode_persistent_7b.traffic.json")
        else:
            rl_bytes, rl_us = nbytes.value, us.value
            rl_kernel = "k_dec_upgate (ffn_norm + up/gate GEMV + SiLU gating)"
            prof = os.path.join(ROOT, "profiles", "decode_upgate_gemv_7b.traffic.json")
        achieved = rl_bytes / (rl_us * 1e-6) / 1e9
        traffic = None
        if os.path.exists(prof):
            with open(prof) as f:
                tj = json.load(f)
            traffic = tj.get("bytes_per_step", 0) * (K / max(launches, 1)) if persistent else tj.get("bytes_per_launch")
            traffic = int(traffic) if traffic else None
        result = {
            "metric": "LLaMA2-7B fp16 decode tok/s (batch 1)",
            "value": round(value, 2),
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": K,
            "warmup": W,
            "ms_per_step": round(ms_step, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "f16",
            "data": "synthetic (random-init weights on device, seeded prompt ids)",
            "config": {"workload": "llama2-7b fp16 batch-1 greedy decode after a 512-token prefill (BASELINE configs[2])",
                       "model": "llama2-7b-arch", "global_batch": world, "seq_len": PROMPT_LEN,
                       "positions": [PROMPT_LEN + W, PROMPT_LEN + W + K],
                       "parallelism": f"dp{world}" if world > 1 else "single",
                       "l2": "inputs larger than L2 (13.2 GB of weights streamed per step)"},
            "step_roofline": {"bytes_per_token": int(step_bytes), "achieved_GBps": round(step_bytes / (ms_step * 1e-3) / 1e9, 1),
                              "frac": round(step_bytes / (ms_step * 1e-3) / 1e9 / peak, 4),
                              "ideal_tok_s": round(peak * 1e9 / step_bytes, 1)},
            "roofline": {"kernel": rl_kernel, "bound": "hbm",
                         "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic,
                         "bytes_per_launch": int(rl_bytes), "us_per_launch": round(rl_us, 3),
                         "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback 6650 GB/s"},
            "decode_path": "persistent cooperative kernel" if persistent else "CUDA-graph of per-op kernels",
            "graph_path_kernels": kern,
            "prefill": {"tokens": PROMPT_LEN, "seconds": round(prefill_s, 4),
                        "tok_s": round(PROMPT_LEN / prefill_s, 1), "path": "drop-in API (graph of op kernels, tcgen05 GEMMs)",
                        "gemms": prefill_gemms},
            "batched": batched,
            "e2e": {"value": round(e2e_value, 2), "unit": "tokens/s", "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 4,
                    "steps": n_e2e,
                    "path": "reference token loop through the C API in native code (vkllm_b200_token_loop: "
                            "tensor_new, graph_new, build_graph, init, upload, run, post_run, read, graph_free per token)",
                    "host_us_per_token": round(host_us / n_e2e, 2),
                    "python_ctypes_loop": {"value": round(e2e_py_value, 2), "unit": "tokens/s",
                                           "path": "the same calls one by one from Python (ctypes)"},
                    "host_graph_us_per_token": host_cost},
            "gpu_launches": int(launches if persistent else kps * K),
            "clocks": clk.summary(),
        }
    # ---- cpu baseline (rank 0, N == 1 only) ---------------------------------------------------
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            w = download_weights(vk, ctx, model, cfg)
            tps, thr, cpu_prefill_s, ref_toks = cpu_decode_sample(w, cfg, n_steps=args.cpu_steps, prompt=prompt)
            result["cpu_baseline"] = {"value": round(tps, 4), "unit": "tokens/s", "cores": thr, "kind": "port",
                                      "sample": f"{args.cpu_steps} single-token decode steps of the same 7B weights at "
                                                f"positions {PROMPT_LEN}..{PROMPT_LEN + args.cpu_steps - 1}, after an untimed "
                                                f"prefill of the same {PROMPT_LEN}-token prompt ({cpu_prefill_s:.1f} s) "
                                                f"(oracle/ C++ restatement of the reference shaders, OpenMP)"}
            # The same run is the parity check of the benchmarked configuration: the oracle's prefill
            # prediction and greedy tokens against the GPU's (API prefill, then the device loop).
            gpu_toks = [first] + [int(t) for t in toks[:args.cpu_steps]]
            result["parity"] = {"config": "llama2-7b, this run's weights and prompt", "tokens_gpu": gpu_toks,
                                "tokens_oracle": ref_toks, "match": gpu_toks == ref_toks}
            del w
        except Exception as e:  # the baseline must not void the GPU measurement
            result["cpu_baseline"] = {"value": None, "error": str(e)[:200]}
    model.free()
    # ---- operator microbenchmarks, rank 0 of a 1-GPU run ----------------------
    if args.ops and world == 1 and result is not None:
        try:
            result["ops"] = ops_microbench(vk, local, SEED)
        except Exception as e:  # a failing microbenchmark must not void the decode measurement
            result["ops"] = {"error": str(e)[:200]}
    # ---- 13B tensor parallel ---------------------------------------------------
    if args.tp_steps > 0:
        tp = tp13b_leg(vk, ctx, args, world, rank, stream)
        if result is not None:
            result["tp13b"] = tp
        if world > 1:  # the NCCL exchange on the same shards, for comparison
            try:
                tp = tp13b_leg(vk, ctx, args, world, rank, stream, "nccl")
            except Exception as e:  # the comparison arm must not void the line
                tp = {"error": str(e)[:200]}
            if result is not None:
                result["tp13b_nccl"] = tp
    ctx.close()
    return result


def run_reference(args, world, rank, local):
    """The reference's algorithm on the host cores (the oracle port; the Vulkan reference cannot run
    here). Weights are the same generator's bits, rebuilt on the CPU."""
    import numpy as np

    import oracle

    if rank != 0:
        return None
    cfg = dict(CFG_7B)
    D, F, V, L = cfg["embedding_length"], cfg["ffn_length"], cfg["vocab_size"], cfg["block_count"]
    oracle.threads(os.cpu_count() or 1)
    w, tid = {}, 0

    def mat(name, r, c):
        nonlocal tid
        w[name] = oracle.random_f16(SEED, tid, 0.02, 0, r * c).reshape(r, c)
        tid += 1

    def ones(name, n):
        nonlocal tid
        w[name] = np.ones(n, dtype=np.float32)
        tid += 1

    t_gen = time.perf_counter()
    mat("token_embd.weight", V, D)
    for l in range(L):
        ones(f"blk.{l}.attn_norm.weight", D)
        ones(f"blk.{l}.ffn_norm.weight", D)
        for n in ("attn_q", "attn_k", "attn_v", "attn_output"):
            mat(f"blk.{l}.{n}.weight", D, D)
        mat(f"blk.{l}.ffn_gate.weight", F, D)
        mat(f"blk.{l}.ffn_up.weight", F, D)
        mat(f"blk.{l}.ffn_down.weight", D, F)
    ones("output_norm.weight", D)
    mat("output.weight", V, D)
    gen_s = time.perf_counter() - t_gen
    steps = max(1, min(args.steps, 4))
    prompt = prompt_tokens(0)
    tps, thr, prefill_s, _ = cpu_decode_sample(w, cfg, n_steps=steps, prompt=prompt)
    return {
        "impl": "reference",
        "metric": "LLaMA2-7B fp16 decode tok/s (batch 1)",
        "value": round(tps, 4),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": steps,
        "warmup": 1,
        "ms_per_step": round(1000.0 / tps, 2),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f16",
        "data": "synthetic (same generator bits as the GPU arm)",
        "config": {"workload": "llama2-7b fp16 batch-1 greedy decode (BASELINE configs[2])", "model": "llama2-7b-arch"},
        "cpu_baseline": {"value": round(tps, 4), "unit": "tokens/s", "cores": thr, "kind": "port",
                         "sample": f"{steps} single-token decode steps at positions {PROMPT_LEN}..{PROMPT_LEN + steps - 1} "
                                   f"after an untimed prefill of the GPU arm's {PROMPT_LEN}-token prompt "
                                   f"({prefill_s:.1f} s); weights regenerated on the CPU in {gen_s:.1f} s (not timed)"},
        "e2e": {"value": round(tps, 4), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "vkllm.c itself needs Vulkan, absent on this box; this is its algorithm restated in C++ (oracle/)",
    }


def profile_gemm(args):
    """Profiling case: the tensor-core GEMM (vkllm_b200_gemm_f16) on seeded fp16 operands A [M, K] and
    B [N, K], launched 4 times on one stream; prints the event-timed mean of the last 2 launches."""
    import torch

    import vkllm_b200 as vk

    M, N, K = (int(v) for v in args.profile_gemm.split(","))
    l = vk.lib()
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    A = (torch.rand((M, K), generator=g, device="cuda") * 2 - 1).half()
    B = (torch.rand((N, K), generator=g, device="cuda") * 2 - 1).half()
    Cm = torch.empty((M, N), device="cuda", dtype=torch.float16)
    s = torch.cuda.current_stream()
    launch = lambda: vk.check(l.vkllm_b200_gemm_f16(A.data_ptr(), B.data_ptr(), Cm.data_ptr(), M, N, K, K, K, N,
                                                     1.0, 0, s.cuda_stream), "gemm")
    launch()
    launch()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    launch()
    launch()
    e1.record(s)
    e1.synchronize()
    us = e0.elapsed_time(e1) * 1000.0 / 2
    print(json.dumps({"profile_case": "gemm", "M": M, "N": N, "K": K, "us": round(us, 2),
                      "tflops": round(2.0 * M * N * K / (us * 1e-6) / 1e12, 1),
                      "error_word": int(l.vkllm_b200_gemm_f16_error())}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-steps", type=int, default=3)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch-seqs", type=int, default=64)
    ap.add_argument("--batch-steps", type=int, default=32)
    ap.add_argument("--tp-steps", type=int, default=32, help="13B tensor-parallel decode leg (0: skip)")
    # Profiling case only (ncu): fewer layers, no prefill / e2e / per-kernel extras, no JSON result line.
    ap.add_argument("--layers", type=int, default=0)
    ap.add_argument("--no-extras", action="store_true")
    ap.add_argument("--profile-batched", action="store_true",
                    help="profiling case: only the batched decode leg (with --layers), no JSON result line")
    ap.add_argument("--profile-gemm", default="",
                    help="profiling case: M,N,K - only the tensor-core GEMM on seeded operands, 4 launches")
    ap.add_argument("--profile-prefill", action="store_true",
                    help="profiling case: only the prompt prefill through the drop-in API (with --layers), 3 runs")
    ap.add_argument("--profile-tp", action="store_true",
                    help="profiling case: only the 13B tensor-parallel decode leg over the ranks")
    ap.add_argument("--ops", type=int, default=1, help="operator microbenchmark leg (0: skip)")
    args = ap.parse_args()
    if args.profile_gemm:
        profile_gemm(args)
        return
    args.warmup = max(3, args.warmup)
    world, rank, local = dist_setup() if args.impl == "ours" else (int(os.environ.get("WORLD_SIZE", "1")),
                                                                    int(os.environ.get("RANK", "0")),
                                                                    int(os.environ.get("LOCAL_RANK", "0")))
    res = run_ours(args, world, rank, local) if args.impl == "ours" else run_reference(args, world, rank, local)
    if rank == 0 and res is not None:
        print(json.dumps(res), flush=True)
    if args.impl == "ours" and world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
