"""Benchmark: 8B-class Q4_K decode at batch 1 through the B200 provider.

Workload: a Llama-style decoder with 32 layers, d_model
4096, 32 query / 8 KV heads of 128, SwiGLU FFN 14336, vocabulary 128256,
RMSNorm eps 1e-5, RoPE theta 500000; projections Q4_K, token embedding and
output Q6_K; fp16 KV cache. Random-init weights from the seeded synthetic
generator (no checkpoint), a 512-token prompt of random ids, then greedy
decoding. One bench step = 256 greedy decode tokens at positions 512..767.

value  tokens/s with everything resident in HBM: each step replays the
       captured decode graph 256 times, the argmax feeding the next token on
       the device; CUDA events on the provider's stream.
e2e    tokens/s through the engine-facing vtable (plan_token with a host
       logits buffer): every token is a kernel-argument upload of
       {token, position}, the graph replay, the 513 KB logits download into
       pinned host memory and the host greedy argmax.

--impl reference times the Fyodor engine's own CPU path (compiled from the
reference sources into oracle/_ref) on this host's cores for the same
workload and metric: the same model bytes (oracle/libsynth.so, the seeded
generator built on its own), the same 512-token prompt prefilled by the
engine's batched CPU prefill, then greedy decode tokens at positions 512 and
up. It loads no library of this provider.
"""
import argparse
import hashlib
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PROMPT = 512
DECODE = 256
CFG8B = dict(layers=32, embedding=4096, heads=32, kv_heads=8, feed_forward=14336, vocabulary=128256, context=1024,
             rope_base=500000.0, epsilon=1e-5, seed=1234, norm_mode=1)
# algorithmic bytes per token: every weight byte once + the fp16 KV rows read
# (Q4_K linears 3,925,868,544 + Q6_K output 430,940,160 + F32 norms
# 1,064,960 + one Q6_K embedding row 3,360)
WEIGHT_BYTES_8B = 4_357_877_024


METRIC = "8B Q4_K decode tok/s (bs1)"
CONFIG8B = {"workload": "8B-class Llama decode: prompt 512 then 256 greedy tokens per step, batch 1",
            "layers": 32, "d_model": 4096, "heads": "32/8", "ffn": 14336, "vocab": 128256,
            "weights": "Q4_K projections, Q6_K embedding/output", "kv": "fp16",
            "l2": "inputs larger than L2 (4.36 GB of weights per token)"}


def kv_bytes(position):  # fp16 K+V of every layer at attention length position+1
    return 131_072 * (position + 1)


def mean_bytes_per_token():
    return WEIGHT_BYTES_8B + sum(kv_bytes(p) for p in range(PROMPT, PROMPT + DECODE)) / DECODE


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f), "measured"
    except OSError:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.samples = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), "--query-gpu=" + self.QUERY,
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append([x.strip() for x in line.split(",")])

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4) if len(s) > 5 + i and s[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples)}


def dist_env():
    return int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("LOCAL_RANK", "0"))


def init_dist(world):
    if world <= 1:
        return None
    import datetime
    import torch.distributed as dist
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
    return dist


def max_over_ranks(dist, value):
    if dist is None:
        return value
    import torch
    t = torch.tensor([value], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(dist):
    if dist is not None:
        dist.barrier()


# ----------------------------------------------------------------------------- CPU reference
def cpu_reference_session(model_ptr, vocabulary):
    """The engine's CPU provider (its SIMD kernels and worker pool, as
    fyodor-bench -b cpu) on all host threads, with the bench prompt prefilled
    by the engine's batched CPU prefill. Returns (session, first greedy token,
    threads)."""
    import oracle as O
    from tests.patterns import bench_tokens
    threads = os.cpu_count() or 1
    os.environ["NYA_CPU_THREADS"] = str(threads)
    s = O.RefSession(model_ptr, PROMPT + DECODE, vocabulary, provider="cpu")
    s.run(bench_tokens(PROMPT, vocabulary), each=False)
    return s, int(np.argmax(s.logits())), threads


def cpu_greedy(s, token, count):
    """count greedy decode steps on an engine session; the last token."""
    for _ in range(count):
        s.run(np.array([token], np.uint32))
        token = int(np.argmax(s.logits()))
    return token


def cpu_reference_rate(model_ptr, vocabulary, sample_seconds, max_tokens=64):
    """Greedy decode on the engine's CPU provider at positions PROMPT.. (the
    GPU's positions); returns (tok/s, tokens, threads)."""
    s, t, threads = cpu_reference_session(model_ptr, vocabulary)
    t = cpu_greedy(s, t, 1)  # warm the worker pool
    n, t0 = 0, time.perf_counter()
    while n < max_tokens - 1 and (time.perf_counter() - t0 < sample_seconds or n < 2):
        t = cpu_greedy(s, t, 1)
        n += 1
    rate = n / (time.perf_counter() - t0)
    s.close()
    return rate, n, threads


# ----------------------------------------------------------------------------- provider arm
def batch_decode(nseq, steps=3, warmup=1, plan=None, model=None, model_name="8b", prompt=PROMPT, decode=DECODE):
    """Batched decode (fyb_batch_*): nseq sequences of the 8B (or, with
    model_name "70b", the 70B) model, each
    with its own random 512-token prompt (prefilled by batched steps, one
    token of every sequence per step), then greedy decode of DECODE tokens per
    sequence at positions 512.., timed with CUDA events over graph replays.
    Returns tok/s over all sequences, ms per step, the weight bytes per step
    and the GB/s those bytes make at that step time."""
    import fyodor_b200 as F
    from tests.patterns import bench_tokens
    own = plan is None  # else: the bench's 8B plan (capacity PROMPT + DECODE), its weights shared
    wbytes, name = WEIGHT_BYTES_8B, "8B"
    if own and model_name == "70b":  # C5 geometry on one GPU, fp16 KV for 8192 positions per sequence
        path = "/dev/shm/fyb_bench_70b_%d.bin" % CFG70B["seed"]
        model = F.SynthModel(matrix_type=F.Q4_K, embed_type=F.Q6_K, output_type=F.Q4_K, path=path, **CFG70B)
        if os.path.exists(path):
            os.unlink(path)
        provider = F.Provider()
        plan = provider.plan(model, CAPACITY_70B)
        wbytes, name = int(bytes_per_token_70b(1, [-1])), "70B"  # position -1: no KV term
    elif own:
        model = F.SynthModel(matrix_type=F.Q4_K, embed_type=F.Q6_K, output_type=F.Q6_K, **CFG8B)
        provider = F.Provider()
        plan = provider.plan(model, PROMPT + DECODE)
    if plan is None:
        raise SystemExit("the provider declined the %s plan" % name)
    batch = F.Batch(plan, nseq)
    prompts = np.stack([bench_tokens(prompt, model.vocabulary, start=997 * b) for b in range(nseq)])
    for i in range(prompt):
        _, am = batch.step(prompts[:, i], np.full(nseq, i, np.uint32), logits=False)
    first, start = am.astype(np.uint32), np.full(nseq, prompt, np.uint32)
    for _ in range(warmup):
        batch.time_greedy(first, start, decode)
    ms = [batch.time_greedy(first, start, decode) for _ in range(steps)]
    if min(ms) < 0:
        raise SystemExit("batched decode failed")
    step_ms = sum(ms) / len(ms)
    out = {"sequences": nseq, "tok_s": round(nseq * 1000.0 / step_ms, 1), "ms_per_step": round(step_ms, 4),
           "weight_bytes_per_step": wbytes,
           "weights_gb_s": round(wbytes / step_ms / 1e6, 1),
           "launches_per_step": int(batch.launches_per_step()),
           "workload": "%s, %d sequences x (%d-token prompt + %d greedy tokens), positions %d..%d"
                       % (name, nseq, prompt, decode, prompt, prompt + decode - 1)}
    batch.close()
    if own:
        plan.close()
        model.close()
        provider.close()
    return out


def run_provider(args):
    import torch
    import fyodor_b200 as F
    from tests.patterns import bench_tokens
    rank, world, local = dist_env()
    os.environ["NYA_CUDA_DEVICE"] = str(local)
    if world > 1:  # tensor parallelism: this rank holds one shard of every layer
        os.environ["NYA_CUDA_TP_SIZE"] = str(world)
        os.environ["NYA_CUDA_TP_RANK"] = str(rank)
    torch.cuda.set_device(local)
    dist = init_dist(world)
    t_setup = time.perf_counter()
    model = F.SynthModel(matrix_type=F.Q4_K, embed_type=F.Q6_K, output_type=F.Q6_K, **CFG8B)
    provider = F.Provider()
    capacity = PROMPT + DECODE
    plan = provider.plan(model, capacity)
    if plan is None:
        raise SystemExit("the provider declined the 8B plan")
    if world > 1:
        if not F.tp_connect_all(plan):
            raise SystemExit("connecting the tensor-parallel ranks failed")
        barrier(dist)
    prompt = bench_tokens(PROMPT, model.vocabulary)
    if plan.prefill(prompt, 0) != 0:
        raise SystemExit("prefill failed")
    first = int(np.argmax(plan.logits))
    setup_s = time.perf_counter() - t_setup
    # the same prompt again (rewrites the same cache rows): plan_prefill with a
    # host logits buffer, wall clock (the first call also built the chunker)
    barrier(dist)
    t0 = time.perf_counter()
    if plan.prefill(prompt, 0) != 0 or int(np.argmax(plan.logits)) != first:
        raise SystemExit("second prefill failed")
    prefill_s = max_over_ranks(dist, time.perf_counter() - t0)
    prefill = {"tokens": PROMPT, "ms": round(prefill_s * 1e3, 2), "tok_s": round(PROMPT / prefill_s, 1),
               "chunk_tokens": int(plan.stats()["prefill_batch"]),
               "how": "plan_prefill through the vtable, host logits of the last token, wall clock"}

    for _ in range(args.warmup):
        if plan.time_greedy(first, PROMPT, DECODE) < 0:
            raise SystemExit("warm-up failed")
    barrier(dist)
    torch.cuda.synchronize()
    launches_before = plan.stats()["kernel_launches"]
    with ClockSampler(local) as clocks:
        total_ms = 0.0
        for _ in range(args.steps):
            ms = plan.time_greedy(first, PROMPT, DECODE)
            if ms < 0:
                raise SystemExit("timed step failed")
            total_ms += ms
    torch.cuda.synchronize()
    launches = plan.stats()["kernel_launches"] - launches_before  # counted by the plan, graph nodes included
    # the first 64 greedy tokens of the timed decode (same start, same positions),
    # comparable across GPU counts
    digest_tokens = plan.decode_greedy(first, PROMPT, 64)
    if digest_tokens is None:
        raise SystemExit("greedy digest run failed")
    digest = {"tokens": 64, "sha1": hashlib.sha1(np.asarray(digest_tokens, np.uint32).tobytes()).hexdigest()[:16],
              "first8": [int(x) for x in digest_tokens[:8]]}
    barrier(dist)
    total_ms = max_over_ranks(dist, total_ms)
    tokens = args.steps * DECODE
    value = tokens / (total_ms / 1000.0)  # one sequence: with tensor parallelism all ranks decode it together

    # e2e through the vtable with host buffers (pinned logits buffer)
    pinned = torch.empty(model.vocabulary, dtype=torch.float32, pin_memory=True)
    plan.logits = pinned.numpy()
    e2e_steps = max(1, min(args.steps, 3))
    barrier(dist)
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        t = first
        for i in range(DECODE):
            if plan.token(t, PROMPT + i) != 0:
                raise SystemExit("e2e token failed")
            t = int(np.argmax(plan.logits))
    e2e_s = max_over_ranks(dist, time.perf_counter() - t0)
    e2e_value = e2e_steps * DECODE / e2e_s

    # stand-alone GEMV kernels (the matvec/matmul entry points), for reference
    gate_ms, gate_bytes = plan.time_projection(0, 2, 20)
    qkv_ms, qkv_bytes = plan.time_projection(0, 0, 20)
    down_ms, down_bytes = plan.time_projection(0, 3, 20)
    o_ms, o_bytes = plan.time_projection(0, 1, 20)
    lg_ms, lg_bytes = plan.time_projection(0, 4, 10)
    phases = trace_summary(plan, first, PROMPT, model.config.layers)
    peaks, peak_kind = measured_peaks()
    hbm = peaks.get("hbm_gbs", 6650.0)
    # the dominant kernel is the persistent decode kernel, one launch per token:
    # algorithmic bytes per launch = weights + the KV cache read at that step
    bpt = mean_bytes_per_token() / world  # with tensor parallelism each GPU streams its shard
    per_launch_ms = total_ms / (args.steps * DECODE)
    achieved = bpt / (per_launch_ms / 1000.0) / 1e9
    traffic = None  # ncu DRAM bytes per launch of the single-GPU kernel (no capture of a shard)
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            traffic = json.load(f).get("decode_kernel_8b") if world == 1 else None
    except (OSError, ValueError):
        pass

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rate, n, threads = cpu_reference_rate(model.ptr, model.vocabulary, args.cpu_seconds)
        cpu = {"value": rate, "unit": "tok/s", "cores": threads, "kind": "reference",
               "sample": "%d greedy decode tokens of the same 8B model at positions 513.. through the Fyodor "
                         "engine's CPU provider (nya_llm_session_run, NYA_CPU_THREADS=%d), after the same "
                         "512-token prompt prefilled by its batched CPU prefill" % (n, threads)}
    attn_c4 = attention_c4() if rank == 0 and world == 1 else None
    with_cpu = not args.no_cpu_baseline
    mv_c2 = matvec_c2(cpu=with_cpu) if rank == 0 and world == 1 else None
    mv_c1 = matvec_c1(cpu=with_cpu) if rank == 0 and world == 1 else None
    batch16 = batch_decode(16, steps=2, plan=plan, model=model) if rank == 0 and world == 1 else None
    verify = None
    if world == 1:  # speculative verification of an 8-token draft at position 512 (one pass, all logits to the host)
        draft = bench_tokens(8, model.vocabulary, 77)
        plan.verify(draft, PROMPT)
        t0 = time.perf_counter()
        for _ in range(5):
            if plan.verify(draft, PROMPT) is None:
                raise SystemExit("draft verification failed")
        vs = (time.perf_counter() - t0) / 5
        verify = {"draft_tokens": 8, "ms": round(vs * 1e3, 3), "tok_s": round(8 / vs, 1),
                  "how": "fyb_plan_verify at positions 512..519 with [8][V] host logits, wall clock; "
                         "one decode step per draft token would take 8 x %.3f ms" % (per_launch_ms,)}
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "tok/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(total_ms / args.steps, 3),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "q4_k weights, s8 limb x u8/s8 int MMA, fp32 accumulate, fp16 KV",
        "data": "synthetic (seeded random-init weights, random prompt ids)",
        "config": dict(CONFIG8B, parallelism="tp%d" % world if world > 1 else "single-gpu"),
        "greedy_digest": digest,
        "e2e": {"value": round(e2e_value, 2), "unit": "tok/s", "h2d_bytes_per_step": 8 * DECODE,
                "d2h_bytes_per_step": 4 * model.vocabulary * DECODE},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 4), "traffic": traffic,
                     "kernel": "decode_kernel (persistent, one launch per token; %d B per launch%s)"
                               % (int(bpt), ", per GPU" if world > 1 else ""),
                     "us_per_launch": round(per_launch_ms * 1000, 2), "peak_source": peak_kind,
                     "tok_s_at_peak": round(hbm * 1e9 / bpt, 1)},
        "decode_phases_us": phases,
        "kernels": {"qkv": [round(qkv_ms * 1e3, 2), round(qkv_bytes / qkv_ms / 1e6, 1)],
                    "o": [round(o_ms * 1e3, 2), round(o_bytes / o_ms / 1e6, 1)],
                    "gateup": [round(gate_ms * 1e3, 2), round(gate_bytes / gate_ms / 1e6, 1)],
                    "down": [round(down_ms * 1e3, 2), round(down_bytes / down_ms / 1e6, 1)],
                    "logits": [round(lg_ms * 1e3, 2), round(lg_bytes / lg_ms / 1e6, 1)],
                    "units": "stand-alone GEMV launches (matvec/matmul path): [us per launch, GB/s]"},
        "attention_c4": attn_c4,
        "matvec_c2": mv_c2,
        "matvec_c1": mv_c1,
        "batch_decode": batch16,
        "verify_draft": verify,
        "gpu_launches": int(launches),
        "clocks": clocks.summary(),
        "cpu_baseline": cpu,
        "prefill": prefill,
        "setup_s": round(setup_s, 1),
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    plan.close()
    provider.close()
    model.close()
    if dist is not None:
        dist.destroy_process_group()


# ----------------------------------------------------------------------------- 70B tensor parallel
CFG70B = dict(layers=80, embedding=8192, heads=64, kv_heads=8, feed_forward=28672, vocabulary=128256, context=8192,
              rope_base=500000.0, epsilon=1e-5, seed=4321, norm_mode=1)
CAPACITY_70B = 8192  # fp16 KV cache sized for the 8192-token context


def bytes_per_token_70b(world, positions):
    """Algorithmic bytes one GPU streams per token of the 70B configuration at
    the given attention positions: its 1/world of the projection and output
    weights (Q4_K), the replicated norms and one Q6_K embedding row, and its
    KV heads' fp16 rows at each position (mean over `positions`)."""
    L, d, ffn, V, hd, kvh = 80, 8192, 28672, 128256, 128, 8
    q4 = lambda r, c: r * c // 256 * 144
    layer = q4(d, d) + 2 * q4(kvh * hd, d) + q4(d, d) + 3 * q4(ffn, d)
    weights = (L * layer + q4(V, d)) / world + L * 2 * d * 4 + d * 4 + d // 256 * 210
    kv = sum(L * (kvh // world) * hd * 2 * 2 * (p + 1) for p in positions) / len(positions)
    return weights + kv


def run_provider_70b(args):
    """The 70B-class configuration (80 layers, d 8192, 64 / 8 heads of 128,
    FFN 28672, vocabulary 128256; Q4_K projections and output head, Q6_K
    embedding; fp16 KV cache for 8192 positions), tensor parallel over the
    launch's ranks (one process per GPU; 1 = a single GPU). All ranks map one
    copy of the model in /dev/shm (the first creates it), as processes on a
    host map one GGUF file. Prompt 512 then 256 greedy tokens per step, batch
    1 (batches of up to 16 sequences on one GPU: --batch 16 --model 70b)."""
    import torch
    import fyodor_b200 as F
    from tests.patterns import bench_tokens
    rank, world, local = dist_env()
    os.environ["NYA_CUDA_DEVICE"] = str(local)
    if world > 1:
        os.environ["NYA_CUDA_TP_SIZE"] = str(world)
        os.environ["NYA_CUDA_TP_RANK"] = str(rank)
    torch.cuda.set_device(local)
    dist = init_dist(world)
    t_setup = time.perf_counter()
    path = "/dev/shm/fyb_bench_70b_%d.bin" % CFG70B["seed"]
    model = F.SynthModel(matrix_type=F.Q4_K, embed_type=F.Q6_K, output_type=F.Q4_K, path=path, **CFG70B)
    provider = F.Provider()
    plan = provider.plan(model, CAPACITY_70B)
    if plan is None:
        raise SystemExit("the provider declined the 70B plan")
    barrier(dist)
    if rank == 0 and os.path.exists(path):
        os.unlink(path)  # every rank holds its mapping; the file goes with the last one
    if world > 1 and not F.tp_connect_all(plan):
        raise SystemExit("connecting the tensor-parallel ranks failed")
    barrier(dist)
    prompt = bench_tokens(PROMPT, model.vocabulary)
    if plan.prefill(prompt, 0) != 0:
        raise SystemExit("prefill failed")
    first = int(np.argmax(plan.logits))
    setup_s = time.perf_counter() - t_setup
    barrier(dist)
    t0 = time.perf_counter()  # the same prompt again, as in the 8B line
    if plan.prefill(prompt, 0) != 0 or int(np.argmax(plan.logits)) != first:
        raise SystemExit("second prefill failed")
    prefill_s = max_over_ranks(dist, time.perf_counter() - t0)
    prefill = {"tokens": PROMPT, "ms": round(prefill_s * 1e3, 2), "tok_s": round(PROMPT / prefill_s, 1),
               "chunk_tokens": int(plan.stats()["prefill_batch"])}
    for _ in range(args.warmup):
        if plan.time_greedy(first, PROMPT, DECODE) < 0:
            raise SystemExit("warm-up failed")
    barrier(dist)
    torch.cuda.synchronize()
    launches_before = plan.stats()["kernel_launches"]
    with ClockSampler(local) as clocks:
        total_ms = 0.0
        for _ in range(args.steps):
            ms = plan.time_greedy(first, PROMPT, DECODE)
            if ms < 0:
                raise SystemExit("timed step failed")
            total_ms += ms
    torch.cuda.synchronize()
    launches = plan.stats()["kernel_launches"] - launches_before
    digest_tokens = plan.decode_greedy(first, PROMPT, 64)
    barrier(dist)
    total_ms = max_over_ranks(dist, total_ms)
    value = args.steps * DECODE / (total_ms / 1000.0)
    peaks, peak_kind = measured_peaks()
    hbm = peaks.get("hbm_gbs", 6650.0)
    bpt = bytes_per_token_70b(world, range(PROMPT, PROMPT + DECODE))
    per_launch_ms = total_ms / (args.steps * DECODE)
    achieved = bpt / (per_launch_ms / 1000.0) / 1e9
    line = {
        "metric": "70B Q4_K decode tok/s (bs1)", "value": round(value, 2), "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(total_ms / args.steps, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "q4_k weights, s8 limb x u8/s8 int MMA, fp32 accumulate, fp16 KV",
        "data": "synthetic (seeded random-init weights, random prompt ids)",
        "config": {"workload": "70B-class Llama decode: prompt 512 then 256 greedy tokens per step, batch 1",
                   "layers": 80, "d_model": 8192, "heads": "64/8", "ffn": 28672, "vocab": 128256,
                   "weights": "Q4_K projections and output, Q6_K embedding", "kv": "fp16, 8192 positions",
                   "parallelism": "tp%d" % world if world > 1 else "single-gpu",
                   "l2": "inputs larger than L2 (%.1f GB of weights per GPU per token)" % (bpt / 1e9)},
        "greedy_digest": {"tokens": 64, "first8": [int(x) for x in digest_tokens[:8]],
                          "sha1": hashlib.sha1(np.asarray(digest_tokens, np.uint32).tobytes()).hexdigest()[:16]},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 4), "traffic": None,
                     "kernel": "decode_kernel (persistent, one launch per token; %d B per launch per GPU)" % int(bpt),
                     "us_per_launch": round(per_launch_ms * 1000, 2), "peak_source": peak_kind,
                     "tok_s_at_peak": round(hbm * 1e9 / bpt, 1)},
        "gpu_launches": int(launches), "clocks": clocks.summary(), "prefill": prefill, "setup_s": round(setup_s, 1),
        "cpu_baseline": None,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    plan.close()
    provider.close()
    model.close()
    if dist is not None:
        dist.destroy_process_group()


# ----------------------------------------------------------------------------- reference arm
def run_reference(args):
    """The engine's own CPU path on this host's cores: the bench model's bytes
    from oracle/libsynth.so, the same prompt prefilled by the engine's batched
    CPU prefill (untimed), then each step = ref_tokens greedy decode tokens at
    the GPU arm's positions. No library of this provider is loaded."""
    import oracle as O
    from oracle.synth import SynthModel, Q4_K, Q6_K
    rank, world, _ = dist_env()
    if rank != 0:
        return
    if not O.reference_available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libnya_ref.so was not built"}))
        return
    model = SynthModel(matrix_type=Q4_K, embed_type=Q6_K, output_type=Q6_K, **CFG8B)
    per_step = max(1, args.ref_tokens)
    s, t, threads = cpu_reference_session(model.ptr, model.vocabulary)
    for _ in range(args.warmup):
        t = cpu_greedy(s, t, per_step)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        t = cpu_greedy(s, t, per_step)
    elapsed = time.perf_counter() - t0
    value = args.steps * per_step / elapsed
    last = PROMPT + (args.warmup + args.steps) * per_step
    s.close()
    model.close()
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "tok/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(elapsed * 1000 / args.steps, 2), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "q4_k weights, fp32 (engine CPU provider)",
            "data": "synthetic (seeded random-init weights, random prompt ids)",
            "config": dict(CONFIG8B, parallelism="tp%d" % world if world > 1 else "single-gpu"),
            "cpu_baseline": {"value": round(value, 3), "unit": "tok/s", "cores": threads, "kind": "reference",
                             "sample": "%d greedy decode tokens per step through nya_llm_session_run with the "
                                       "engine's cpu provider at positions %d..%d, after the 512-token prompt "
                                       "(batched CPU prefill, untimed)" % (per_step, PROMPT + 1, last)},
            "e2e": {"value": round(value, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def attention_c4(reps=20, warmup=3, splits_decode=16, splits_verify=8, nseq=32):
    """The ragged-batch attention configuration: 32 sequences with context
    lengths uniform in [128, 32768] (seeded), 32 query / 8 KV heads, head_dim
    128, fp16 K/V; decode (one query per sequence) and speculative
    verification (8 draft queries per sequence, causal within the draft).
    [us per launch, GB/s] with GB/s = unique K/V bytes (4096 B per position
    and KV-head group) plus q and out, over CUDA-event time."""
    import ctypes as C
    import torch
    import fyodor_b200 as F
    heads, kvh, hd, cap = 32, 8, 128, 32768
    rng = np.random.default_rng(1234)
    lengths = rng.integers(128, cap + 1, size=nseq).astype(np.int32)
    g = torch.Generator(device="cuda").manual_seed(1234)
    k = torch.randn((nseq, kvh, cap, hd), generator=g, device="cuda", dtype=torch.float16)
    v = torch.randn((nseq, kvh, cap, hd), generator=g, device="cuda", dtype=torch.float16)
    dl = torch.from_numpy(lengths).cuda()
    P = lambda t: C.c_void_p(t.data_ptr())
    kv_bytes = int(lengths.sum()) * kvh * hd * 2 * 2
    res = {}
    for name, queries, splits in (("decode", 1, splits_decode), ("verify8", 8, splits_verify)):
        q = torch.randn((nseq, queries, heads, hd), generator=g, device="cuda")
        out = torch.empty_like(q)
        wsb = F.lib.fyb_attention_workspace(nseq * queries, heads, kvh, hd, splits)
        ws = torch.zeros(wsb, dtype=torch.uint8, device="cuda")
        call = lambda: F.lib.fyb_attention_verify(P(q), P(k), P(v), kvh * cap * hd, P(dl), nseq, queries, heads,
                                                  kvh, hd, cap, C.c_float(1 / np.sqrt(hd)), P(out), splits, P(ws),
                                                  wsb, C.c_void_p(torch.cuda.current_stream().cuda_stream))
        for _ in range(warmup):
            assert call() == 0
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            call()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        nbytes = kv_bytes + 2 * q.numel() * 4
        res[name] = [round(ms * 1e3, 1), round(nbytes / ms / 1e6, 1)]
    del k, v
    torch.cuda.empty_cache()
    res["units"] = "[us per launch, GB/s of unique K/V + q + out]; 32 sequences, lengths U[128, 32768]"
    return res


def _cpu_compute():
    """The engine's "cpu" compute provider on all host threads, or None when
    oracle/_ref was not built."""
    import oracle as O
    if not O.reference_available():
        return None, 0
    threads = os.cpu_count() or 1
    os.environ["NYA_CPU_THREADS"] = str(threads)
    return O.RefCompute(), threads


def _time_device(call, copies, reps, warmup):
    """Milliseconds per call(copy) of device time, rotating over `copies`:
    the `reps` calls are captured once in a CUDA graph and the graph replay
    is timed with CUDA events, so the host's per-call cost (ctypes, argument
    checks, launch API) does not pace the GPU for kernels of a few us."""
    import torch
    reps = max(reps, len(copies))  # every copy once per replay: the replays stream more than L2 holds
    for i in range(warmup):
        assert call(copies[i % len(copies)]) == 0
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for i in range(reps):
            assert call(copies[i % len(copies)]) == 0
    graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    graph.replay()
    e1.record()
    torch.cuda.synchronize()
    del graph
    return e0.elapsed_time(e1) / reps


def matvec_c2(reps=10, warmup=3, cpu=False):
    """The matvec / small-batch GEMM sweep: Q4_K and Q6_K weights of the four
    projection shapes (out x in) at batches 1, 2, 4, 8, 16, repacked once
    (fyb_quant_repack) and multiplied with fyb_quant_matmul_prepared. Consecutive
    timed launches rotate over copies of the weights totalling at least 512 MB
    (more than L2). Values: {shape: {type: {batch: [us, GB/s]}}}, GB/s =
    (GGUF weight bytes once + 4 B x batch x (in + out)) / time. With cpu=True
    the same weights (host copies) also go through the engine's CPU provider
    at batches 1 and 16 (nya_compute_matvec_typed / matmul_typed on a "cpu"
    context): values under "cpu"."""
    import ctypes as C
    import torch
    import fyodor_b200 as F
    P = lambda t: C.c_void_p(t.data_ptr())
    stream = lambda: C.c_void_p(torch.cuda.current_stream().cuda_stream)
    ref, threads = _cpu_compute() if cpu else (None, 0)
    out, cpu_out = {}, {}
    for rows, cols in ((4096, 4096), (14336, 4096), (4096, 14336), (128256, 4096)):
        shape = "%dx%d" % (rows, cols)
        out[shape], cpu_out[shape] = {}, {}
        for tname, t in (("q4_k", F.Q4_K), ("q6_k", F.Q6_K)):
            nbytes = rows * F.row_bytes(t, cols)
            data = np.empty(nbytes, np.uint8)
            F.lib.fyb_synth_fill(C.c_void_p(data.ctypes.data), rows, cols, t, 2024, rows * 7 + cols)
            wsb = F.lib.fyb_quant_matmul_workspace(rows, cols, t, 16)
            ws0 = torch.zeros(wsb, dtype=torch.uint8, device="cuda")
            dw = torch.from_numpy(data).cuda()
            assert F.lib.fyb_quant_repack(P(dw), rows, cols, t, P(ws0), wsb, stream()) == 0
            del dw
            copies = [ws0] + [ws0.clone() for _ in range(max(0, -(-(512 << 20) // wsb) - 1))]
            x = torch.randn((16, cols), device="cuda")
            y = torch.empty((16, rows), device="cuda")
            res = {}
            for batch in (1, 2, 4, 8, 16):
                ms = _time_device(lambda ws: F.lib.fyb_quant_matmul_prepared(rows, cols, t, P(x), P(y), batch, P(ws),
                                                                             wsb, stream()), copies, reps, warmup)
                res[batch] = [round(ms * 1e3, 2), round((nbytes + 4 * batch * (rows + cols)) / ms / 1e6, 1)]
            out[shape][tname] = res
            del copies, ws0
            torch.cuda.empty_cache()
            if ref is not None:
                xs = x.cpu().numpy()
                cres = {}
                for batch in (1, 16):
                    us = ref.time(data, rows, cols, t, xs[:batch], batch)
                    cres[batch] = [round(us, 1), round((nbytes + 4 * batch * (rows + cols)) / us / 1e3, 1)]
                cpu_out[shape][tname] = cres
    out["units"] = "[us per call, GB/s of GGUF weight bytes once + x + y]; batches of 3..16 run the small-batch GEMM (every weight unit read once)"
    if ref is not None:
        cpu_out["units"] = ("[us per call, GB/s] through the Fyodor engine's CPU provider (nya_compute_matvec_typed / "
                            "nya_compute_matmul_typed on a \"cpu\" context, NYA_CPU_THREADS=%d), weights in host memory"
                            % threads)
        out["cpu"] = cpu_out
        ref.close()
    return out


def matvec_c1(reps=200, warmup=5, cpu=False):
    """C1: Q8_0 4096x4096 (int8 uniform in [-127, 127], d = |N(0,1)| * 0.01,
    seeded) times an fp32 N(0,1) vector, through fyb_quant_matmul (the
    bulk-staged Q8_0 kernel; batch 8 as well), rotating over copies of the
    weights totalling at least 512 MB. With cpu=True the engine's CPU provider
    times the same product from host memory."""
    import ctypes as C
    import torch
    import fyodor_b200 as F
    rows = cols = 4096
    P = lambda t: C.c_void_p(t.data_ptr())
    stream = lambda: C.c_void_p(torch.cuda.current_stream().cuda_stream)
    nbytes = rows * F.row_bytes(F.Q8_0, cols)
    data = np.empty(nbytes, np.uint8)
    F.lib.fyb_synth_fill(C.c_void_p(data.ctypes.data), rows, cols, F.Q8_0, 2024, rows * 7 + cols)
    dw = torch.from_numpy(data).cuda()
    copies = [dw] + [dw.clone() for _ in range(-(-(512 << 20) // nbytes) - 1)]
    x = torch.randn((8, cols), device="cuda")
    y = torch.empty((8, rows), device="cuda")
    res = {}
    for batch in (1, 8):
        ms = _time_device(lambda w: F.lib.fyb_quant_matmul(P(w), rows, cols, F.Q8_0, P(x), P(y), batch, None, 0,
                                                           stream()), copies, reps, warmup)
        res[batch] = [round(ms * 1e3, 2), round((nbytes + 4 * batch * (rows + cols)) / ms / 1e6, 1)]
    del copies, dw
    torch.cuda.empty_cache()
    out = {"q8_0_4096x4096": res,
           "units": "[us per call, GB/s of GGUF weight bytes once + x + y]"}
    ref, threads = _cpu_compute() if cpu else (None, 0)
    if ref is not None:
        us = ref.time(data, rows, cols, F.Q8_0, x[:1].cpu().numpy(), 1, seconds=1.0, max_calls=2000)
        out["cpu"] = {"1": [round(us, 1), round((nbytes + 4 * (rows + cols)) / us / 1e3, 1)],
                      "threads": threads, "kind": "reference",
                      "sample": "nya_compute_matvec_typed on a \"cpu\" context, weights in host memory"}
        ref.close()
    return out


def run_gemm_case(case, reps):
    """One prepared Q4_K/Q6_K product (fyb_quant_matmul_prepared) or one Q8_0
    product (fyb_quant_matmul) of the C1/C2
    sweep, `reps` launches after 3 warm-up launches on one weight copy: the
    small case an ncu capture of the small-batch GEMM or GEMV runs on."""
    import ctypes as C
    import torch
    import fyodor_b200 as F
    shape, tname, batch = case.split(":")
    rows, cols = (int(v) for v in shape.split("x"))
    t, batch = {"q4_k": F.Q4_K, "q6_k": F.Q6_K, "q8_0": F.Q8_0}[tname], int(batch)
    P = lambda v: C.c_void_p(v.data_ptr())
    stream = lambda: C.c_void_p(torch.cuda.current_stream().cuda_stream)
    nbytes = rows * F.row_bytes(t, cols)
    data = np.empty(nbytes, np.uint8)
    F.lib.fyb_synth_fill(C.c_void_p(data.ctypes.data), rows, cols, t, 2024, rows * 7 + cols)
    x = torch.randn((batch, cols), device="cuda")
    y = torch.empty((batch, rows), device="cuda")
    if t == F.Q8_0:  # no repack: the Q8_0 kernel reads the GGUF rows
        dw = torch.from_numpy(data).cuda()
        ms = _time_device(lambda w: F.lib.fyb_quant_matmul(P(w), rows, cols, t, P(x), P(y), batch, None, 0, stream()),
                          [dw], reps, 3)
        return {"gemm_case": case, "us_per_call": round(ms * 1e3, 2), "weight_bytes": nbytes,
                "gb_s": round(nbytes / ms / 1e6, 1)}
    wsb = F.lib.fyb_quant_matmul_workspace(rows, cols, t, batch)
    ws = torch.zeros(wsb, dtype=torch.uint8, device="cuda")
    dw = torch.from_numpy(data).cuda()
    assert F.lib.fyb_quant_repack(P(dw), rows, cols, t, P(ws), wsb, stream()) == 0
    ms = _time_device(lambda w: F.lib.fyb_quant_matmul_prepared(rows, cols, t, P(x), P(y), batch, P(w), wsb, stream()),
                      [ws], reps, 3)
    return {"gemm_case": case, "us_per_call": round(ms * 1e3, 2), "weight_bytes": nbytes,
            "gb_s": round(nbytes / ms / 1e6, 1)}


def run_allreduce_probe(args):
    """The exchange of the reference design for tensor parallelism (one NCCL
    all-reduce of the d-wide residual per attention block and per MLP block,
    64 per 8B token): under torchrun, every rank times `--reps` all-reduces
    of 4096 fp32 values captured in a CUDA graph, max over ranks. Prints us
    per all-reduce and the exchange time alone per 8B token."""
    import datetime
    import torch
    import torch.distributed as dist
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    x = torch.ones(CFG8B["embedding"], device="cuda")
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        for _ in range(5):
            dist.all_reduce(x)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for _ in range(args.reps):
            dist.all_reduce(x)
    graph.replay()
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record()
        graph.replay()
        e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / args.reps
    t = torch.tensor([us], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    del graph
    if rank == 0:
        print(json.dumps({"allreduce_probe": {"ranks": world, "bytes": 4 * CFG8B["embedding"], "us": round(float(t.item()), 2),
                                              "per_8b_token_us": round(float(t.item()) * 2 * CFG8B["layers"], 1)}}))
    dist.barrier()
    dist.destroy_process_group()


# ----------------------------------------------------------------------------- profiling modes
KERNELS = {"qkv": 0, "o": 1, "gateup": 2, "down": 3, "logits": 4}


def run_kernel_mode(args):
    """One 8B-shaped layer (plus the output head): time `--reps` stand-alone
    launches of one fused projection kernel. Small enough (about 1 GB on the
    device) for a full ncu capture of a single launch."""
    import fyodor_b200 as F
    model = F.SynthModel(matrix_type=F.Q4_K, embed_type=F.Q6_K, output_type=F.Q6_K,
                         **dict(CFG8B, layers=1, context=64))
    provider = F.Provider()
    plan = provider.plan(model, 64)
    ms, nbytes = plan.time_projection(0, KERNELS[args.kernel], args.reps)
    print(json.dumps({"kernel": args.kernel, "reps": args.reps, "us_per_launch": round(ms * 1000, 3),
                      "bytes_per_launch": nbytes, "gb_s": round(nbytes / ms / 1e6, 1)}))


def run_steps_mode(args):
    """A few 8B decode steps launched eagerly (one launch per kernel, graphs
    off) so an ncu launch list shows every kernel of a step."""
    os.environ["NYA_CUDA_GRAPHS"] = "0"
    import fyodor_b200 as F
    layers = args.layers or CFG8B["layers"]
    model = F.SynthModel(matrix_type=F.Q4_K, embed_type=F.Q6_K, output_type=F.Q6_K,
                         **dict(CFG8B, context=64, layers=layers))
    provider = F.Provider()
    plan = provider.plan(model, 64)
    for i in range(args.eager_steps):
        if plan.token(17 + i, i) != 0:
            raise SystemExit("decode step failed")
    print(json.dumps({"eager_steps": args.eager_steps, "kernel_launches": plan.stats()["kernel_launches"]}))


PHASE_KINDS = ["qkv", "attention", "o", "gateup", "down"]


def summarize_trace(tr, layers):
    """Per phase kind: the CTA-median microseconds from the end of the
    previous phase to the end of this one (waiting for its input, preparing
    it, the units and the tile outputs), summed over the layers of one step."""
    t = tr.astype(np.int64) - int(tr[0].min())
    out = {k: 0.0 for k in PHASE_KINDS + ["logits"]}
    for l in range(layers):
        for k in range(5):
            i = 1 + 5 * l + k
            out[PHASE_KINDS[k]] += float(np.median(t[i] - t[i - 1])) / 1e3
    lb = 1 + 5 * layers
    out["logits"] = float(np.median(t[lb] - t[lb - 1])) / 1e3
    res = {k: round(v, 1) for k, v in out.items()}
    res["exit"] = round(float(np.median(t[lb + 1] - t[lb])) / 1e3, 1)
    res["step_us"] = round(float(t[-1].max()) / 1e3, 1)
    return res


def trace_summary(plan, token, position, layers):
    """One traced persistent decode step (None when the plan does not run the
    persistent kernel)."""
    if plan.decode_form() != 1:
        return None
    tr = plan.trace(token, position)
    return None if tr is None else summarize_trace(tr, layers)


def run_trace_mode(args):
    """Where one persistent decode step spends its time: the 8B model after a
    PROMPT-token prefill, one step traced per CTA (globaltimer), reported per
    phase kind as the CTA-median time from the end of the previous phase to
    the end of this one, summed over layers, in microseconds."""
    import fyodor_b200 as F
    from tests.patterns import bench_tokens
    model = F.SynthModel(matrix_type=F.Q4_K, embed_type=F.Q6_K, output_type=F.Q6_K, **CFG8B)
    plan = F.Provider().plan(model, PROMPT + 8)
    if plan is None or plan.prefill(bench_tokens(PROMPT, model.vocabulary), 0) != 0:
        raise SystemExit("8B plan or prefill failed")
    tr = None
    for i in range(args.trace_step):  # the last traced step is reported (earlier ones warm up)
        res = plan.trace(17 + i, PROMPT + i, detail=bool(args.trace_raw))
        if res is None:
            raise SystemExit("trace failed (persistent kernel not in use?)")
        tr = res[0] if args.trace_raw else res
    if args.trace_raw:
        np.save(args.trace_raw, tr)
        np.save(args.trace_raw.replace(".npy", "") + "_detail.npy", res[1])
    res = summarize_trace(tr, model.config.layers)
    step = res.pop("step_us")
    print(json.dumps({"trace_us": res, "step_us": step, "grid": int(tr.shape[1]), "points": int(tr.shape[0])}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--kernel", choices=sorted(KERNELS), help="time one fused kernel of an 8B layer")
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--eager-steps", type=int, default=0, help="run N eager 8B decode steps (profiling)")
    ap.add_argument("--trace-step", type=int, default=0,
                    help="trace N persistent 8B decode steps per CTA and report the last (profiling)")
    ap.add_argument("--trace-raw", default="", help="with --trace-step: also save the raw trace (.npy)")
    ap.add_argument("--layers", type=int, default=0, help="with --eager-steps: layers of the model (small ncu cases)")
    ap.add_argument("--attention", action="store_true", help="time the ragged-batch attention configuration only")
    ap.add_argument("--matvec", action="store_true", help="time the matvec / small-batch GEMM sweep only")
    ap.add_argument("--gemm-case", default="",
                    help="ROWSxCOLS:TYPE:BATCH (TYPE q4_k, q6_k or q8_0): time one product (small ncu cases)")
    ap.add_argument("--seqs", type=int, default=32, help="with --attention: sequences of the ragged batch")
    ap.add_argument("--allreduce-probe", action="store_true",
                    help="under torchrun: time the reference design's NCCL all-reduce of the residual")
    ap.add_argument("--batch", type=int, default=0, help="time batched decode of this many sequences (1..16)")
    ap.add_argument("--batch-prompt", type=int, default=PROMPT, help="with --batch: prompt tokens per sequence")
    ap.add_argument("--batch-decode", type=int, default=DECODE, help="with --batch: greedy tokens per timed step")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--model", default="8b", choices=["8b", "70b"], help="70b: the tensor-parallel 70B configuration")
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="fyodor", choices=["fyodor", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--ref-tokens", type=int, default=2)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.kernel:
        run_kernel_mode(args)
    elif args.matvec:
        print(json.dumps({"matvec_c1": matvec_c1(cpu=not args.no_cpu_baseline),
                          "matvec_c2": matvec_c2(cpu=not args.no_cpu_baseline)}))
    elif args.batch:
        print(json.dumps({"batch_decode": batch_decode(args.batch, steps=args.steps, warmup=min(args.warmup, 1),
                                                       model_name=args.model, prompt=args.batch_prompt,
                                                       decode=args.batch_decode)}))
    elif args.allreduce_probe:
        run_allreduce_probe(args)
    elif args.gemm_case:
        print(json.dumps(run_gemm_case(args.gemm_case, args.reps)))
    elif args.attention:
        print(json.dumps({"attention_c4": attention_c4(reps=args.reps, warmup=3, nseq=args.seqs)}))
    elif args.eager_steps:
        run_steps_mode(args)
    elif args.trace_step:
        run_trace_mode(args)
    elif args.impl == "reference":
        run_reference(args)
    elif args.model == "70b":
        run_provider_70b(args)
    else:
        run_provider(args)


if __name__ == "__main__":
    main()
