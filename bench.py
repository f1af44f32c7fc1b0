"""Benchmark of the speculative-decode hot path (BASELINE metric: decode tok/s,
greedy MTP k=3; verify-step HBM GB/s vs peak).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload ("C3"): the synthetic 64-layer hybrid decoder
(hidden 5120, FFN 17408, vocab 248320, 48 Gated DeltaNet + 16 gated GQA
layers, IQ4_XS projections, Q6_K embedding/head, Q8_0 eh_proj) plus the
blk.64 MTP layer; 128-token random prompt; speculative decode with k = 3
drafts and a verify width of 4, accept length forced per cycle from a
seeded uniform{0..3} schedule.  One step = one speculative cycle (3 MTP
drafts, batched verify, acceptance, rollback, MTP anchor); the default
W + K = 5 + 200 cycles emit ~512 tokens.  Weights are random (no checkpoint
is available); the GGUF is written by the seeded generator before timing.

Multi-GPU: one process per GPU (torchrun).  --parallel tp (the default): the
ranks decode ONE sequence together; each holds 1/N of the DeltaNet /
attention heads and FFN columns, the residual projections exchange partial
sums over NVLink, the output head is split over the vocabulary; value = that
sequence's tokens / max rank time (strong scaling).  --parallel replicas: each
rank a full model decoding its own sequence; value = tokens of all ranks /
max rank time (weak scaling, no data-path collective).

Parity: the line's "parity" object compares the stream just timed (from the
first cycle after prefill) with the compiled reference's stream for the same
workload, committed in tests/golden/full_spec.npz, and, at N = 1, with the
reference run live on the host cores in the cpu_baseline leg; under tensor
parallelism every rank's stream must also equal rank 0's.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "tests"))


def _load(name, path):
    import importlib.util
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


qb = _load("qwen_b200", os.path.join(ROOT, "qwen3.8-27b-in-c_b200", "qwen_b200.py"))

METRIC = "decode tok/s (greedy, MTP k=3)"
WORKLOAD = "C3: 64-layer hybrid + MTP, k=3, verify width 4, forced accept U{0..3}"
PROMPT_LEN = 128
SEED = 0


_RESULT_FD = None


def emit(obj):
    """The one JSON line of the run, on the process's real standard output; everything
    else a library prints (NCCL's banner, warnings) goes to standard error."""
    os.write(_RESULT_FD if _RESULT_FD is not None else 1, (json.dumps(obj) + "\n").encode())


def log(msg):
    try:
        rss = int(open("/proc/self/statm").read().split()[1]) * os.sysconf("SC_PAGE_SIZE") / 1e9
    except Exception:
        rss = -1
    print(f"[bench {time.strftime('%H:%M:%S')}] {msg} (rss {rss:.1f} GB)", file=sys.stderr, flush=True)


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def profiled_traffic():
    """DRAM bytes (read + write) of one FFN gate+up launch from an ncu capture,
    kept as data in profiles/roofline_traffic.json (same launch shape in the
    4-layer capture and the full model)."""
    try:
        with open(os.path.join(ROOT, "profiles", "roofline_traffic.json")) as f:
            return float(json.load(f)["dram_bytes_per_launch"])
    except (OSError, KeyError, ValueError):
        return None


def golden_full():
    """The compiled reference's output on this exact workload (prompt, forced
    schedule, FULL seed-0 model), committed as tests/golden/full_spec.npz."""
    try:
        return np.load(os.path.join(ROOT, "tests", "golden", "full_spec.npz"))
    except OSError:
        return None


def golden_long():
    """The compiled reference's output on C4 (2048-token prompt, then MTP
    speculation): tests/golden/full_long.npz, or None when absent."""
    f = os.path.join(ROOT, "tests", "golden", "full_long.npz")
    return np.load(f) if os.path.exists(f) else None


def rel_l2(a, b):
    a, b = np.float64(a), np.float64(b)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def stream_parity(toks, js, ref_toks, ref_js):
    """Compare two speculative streams over their common prefix."""
    n = min(len(toks), len(ref_toks))
    nj = min(len(js), len(ref_js))
    diff = next((i for i in range(n) if toks[i] != ref_toks[i]), None)
    return {"tokens_equal": diff is None and n > 0, "n_tokens": int(n), "first_diff": diff,
            "accept_equal": bool(nj > 0 and np.array_equal(js[:nj], ref_js[:nj])), "n_cycles": int(nj)}


def gguf_path(rank, world):
    d = "/dev/shm" if os.path.isdir("/dev/shm") else "/tmp"
    path = os.path.join(d, f"qb_bench_full_seed{SEED}.gguf")
    if rank == 0 and not os.path.exists(path):
        tmp = path + f".tmp{os.getpid()}"
        t0 = time.time()
        qb.write_synth_gguf(tmp, qb.FULL, seed=SEED)
        os.replace(tmp, path)
        print(f"[bench] wrote {path} ({os.path.getsize(path) / 1e9:.2f} GB) in {time.time() - t0:.1f}s",
              file=sys.stderr, flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    return path


def prompt_tokens(rank):
    return np.random.default_rng(1000 + rank).integers(0, qb.FULL["vocab"], PROMPT_LEN).astype(np.uint32)


def forced_schedule(n=4096):
    return np.random.default_rng(SEED).integers(0, 4, n).astype(np.uint32)


class Clocks:
    """nvidia-smi sampling during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.p = None

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "200"],
                                      stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.p = None
        return self

    def __exit__(self, *a):
        self.rows = []
        if self.p:
            self.p.terminate()
            try:
                out, _ = self.p.communicate(timeout=5)
            except Exception:
                out = ""
            for line in out.strip().splitlines():
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9:
                    self.rows.append(parts)

    def summary(self):
        rows = getattr(self, "rows", [])
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def cpu_reference_run(path, n_threads, warmup, steps, time_budget=None):
    """The reference engine (oracle/_ref, compiled from its own sources) on the
    host cores: prefill 128, then speculative cycles.  Returns (tok/s, sample
    description, stream) where stream holds the emitted tokens and accept lengths
    from the first cycle on and the prefill logits, for the parity check."""
    orc = _load("qb_oracle", os.path.join(ROOT, "oracle", "ref.py"))
    if not orc.available():
        return None, "oracle/_ref not built", None
    n_ctx = PROMPT_LEN + 4 * (warmup + steps) + 64
    m = orc.RefModel(path, n_ctx, n_threads)
    log("reference model_init")
    tp0 = time.perf_counter()
    m.prefill(prompt_tokens(0), 1)
    prefill_tps = PROMPT_LEN / (time.perf_counter() - tp0)
    prefill_logits = m.logits()
    log("reference prefill")
    forced = forced_schedule()
    all_t, all_j = [], []
    if warmup:
        t, j = m.spec_generate(10 ** 6, 3, forced=forced, max_cycles=warmup)
        all_t.append(t)
        all_j.append(j)
    toks = 0
    cycles = 0
    t0 = time.perf_counter()
    while cycles < steps:
        # the forced schedule continues where the warmup left off
        t, j = m.spec_generate(10 ** 6, 3, forced=np.roll(forced, -(warmup + cycles)), max_cycles=1)
        toks += len(t)
        cycles += 1
        all_t.append(t)
        all_j.append(j)
        if time_budget and time.perf_counter() - t0 > time_budget:
            break
    dt = time.perf_counter() - t0
    # C2's rate: plain greedy decode from where the cycles left off (one forward per token)
    tg = time.perf_counter()
    g = m.greedy_generate(4)
    greedy_tps = (len(g) - 1) / (time.perf_counter() - tg)
    m.close()
    stream = {"tokens": np.concatenate(all_t), "accept": np.concatenate(all_j), "prefill_logits": prefill_logits,
              "greedy_tok_s": greedy_tps, "prefill_tok_s": prefill_tps}
    return toks / dt, f"{cycles} cycles ({toks} tokens) after {warmup} warm-up cycles, prompt {PROMPT_LEN}", stream


def cpu_micro_c1(n_threads, reps=3):
    """C1 on the reference's own gemv_batch (host cores): the 17408 x 5120
    IQ4_XS matrix of the seeded generator, N = 1, 2, 4, GB/s of weight bytes
    (page-cache warm: one untimed call first)."""
    orc = _load("qb_oracle", os.path.join(ROOT, "oracle", "ref.py"))
    if not orc.available():
        return None
    rows, K = 17408, 5120
    raw = qb.synth_matrix(qb.GGML_IQ4_XS, rows, K, seed=0, d_sigma=0.02)
    out = {}
    for n in (1, 2, 4):
        x = np.random.default_rng(n).standard_normal((n, K)).astype(np.float32)
        orc.ref_gemv_batch(raw, qb.GGML_IQ4_XS, K, rows, x, n_threads)
        t0 = time.perf_counter()
        for _ in range(reps):
            orc.ref_gemv_batch(raw, qb.GGML_IQ4_XS, K, rows, x, n_threads)
        t = (time.perf_counter() - t0) / reps
        out[f"n{n}"] = {"ms": t * 1e3, "GB/s": raw.nbytes / t / 1e9}
    return out


C4_PROMPT, C4_DECODE = 2048, 1024


def run_c4(args, model, open_model, close_model, seq_rank, ms_ver_short):
    """C4: a 2048-token prompt (63 prefill chunks of 32 and 4 of 8, device-timed), then MTP
    speculation (k = 3, forced schedule) for 1024 tokens at that context, then
    the verify step re-timed at the context reached (about 3072), against the
    verify step at the short context of C3.  The model is re-opened with a
    context of 3200 positions; the new model is returned under "_model"."""
    close_model(model)
    model = open_model(C4_PROMPT + C4_DECODE + 128)
    if not args.parallel == "tp" or int(os.environ.get("WORLD_SIZE", "1")) == 1:
        model.enable_wide()   # 32-token prefill chunks: IQ4_XS on the wide tcgen05 GEMM
    prompt = np.random.default_rng(2000 + seq_rank).integers(0, qb.FULL["vocab"], C4_PROMPT).astype(np.uint32)
    forced = forced_schedule()
    model.prefill(prompt, 1)   # warm: captures the chunk graph
    model.reset()
    model.prefill(prompt, 1)
    ms_pf = model.last_loop_ms()
    lg = model.logits()
    log(f"C4 prefill {ms_pf:.1f} ms")
    toks, js = model.spec_generate(C4_DECODE, 3, forced=forced, max_cycles=4096)
    ms_dec = model.last_loop_ms()
    log(f"C4 decode {len(toks)} tokens {ms_dec:.1f} ms")
    ms_v, b_v = model.bench(0, 4, 10)
    c4 = {"prefill_tok/s": C4_PROMPT / (ms_pf / 1e3), "prefill_ms": ms_pf,
          "prefill_chunks": "63 x 32 + 4 x 8 tokens (32-token chunks: IQ4_XS on the wide tcgen05 GEMM)",
          "decode_tok/s": len(toks) / (ms_dec / 1e3), "decode_tokens": int(len(toks)),
          "decode_context": [C4_PROMPT, int(model.pos)],
          "verify_ms_at_context": ms_v, "verify_context": int(model.pos), "verify_bytes": b_v,
          "verify_ms_short_context": ms_ver_short,
          "attention_share_of_verify": (ms_v - ms_ver_short) / ms_v,
          "kv_bytes_per_verify": 16 * model.pos * 2 * 1024 * 4}
    gold = golden_long()
    if gold is not None and seq_rank == 0:
        n = min(len(toks), len(gold["tokens"]))
        c4["parity_golden"] = {
            "prefill_logits_rel_l2": rel_l2(lg[:: int(gold["sub_stride"])], gold["prefill_sub"]),
            "tokens_equal": bool(np.array_equal(toks[:n], gold["tokens"][:n])),
            "accept_equal": bool(np.array_equal(js[:len(gold["accept"])], gold["accept"])),
            "n_tokens": int(n)}
    c4["_model"] = model
    return c4


C5_SEQ, C5_CTX = 8, (256, 4096)


def run_c5(args, model, open_model, close_model):
    """C5: 8 sequences at seeded contexts U{256..4096} (each prefilled alone),
    then MTP speculation (k = 3, forced schedule) of all of them at once: the
    verify runs 8 x 4 = 32 rows per weight sweep (8-row GEMV chunks), the drafts
    8 rows.  Device-timed over the timed cycles; sequence 0 is then re-run alone
    from the same prompt and must emit the same tokens.  Returns (dict, model)."""
    close_model(model)
    model = open_model(C5_CTX[1] + 4 * (args.warmup + args.c5_steps) + 64)
    rng = np.random.default_rng(5000)
    lens = rng.integers(C5_CTX[0], C5_CTX[1] + 1, C5_SEQ)
    prompts = [rng.integers(0, qb.FULL["vocab"], int(n)).astype(np.uint32) for n in lens]
    forced = forced_schedule()
    model.seq_init(C5_SEQ)
    t0 = time.time()
    for s, p in enumerate(prompts):
        model.seq_prefill(s, p)
    log(f"C5 prefill of {int(lens.sum())} tokens {time.time() - t0:.1f}s")
    w_t, w_j = model.seq_generate(args.warmup, 3, forced=forced)
    toks, js = model.seq_generate(args.c5_steps, 3, forced=np.roll(forced, -args.warmup))
    ms = model.last_loop_ms()
    n_tok = int(sum(len(t) for t in toks))
    log(f"C5 {args.c5_steps} cycles, {n_tok} tokens, {ms:.1f} ms")
    seq0 = np.concatenate([w_t[0], toks[0]])
    model.seq_init(1)   # sequence 0 alone, same prompt and schedule
    model.prefill(prompts[0], 1)
    alone, _ = model.spec_generate(10 ** 6, 3, forced=forced, max_cycles=args.warmup + args.c5_steps)
    c5 = {"tok/s": n_tok / (ms / 1e3), "ms_per_cycle": ms / args.c5_steps, "sequences": C5_SEQ,
          "contexts": [int(n) for n in lens], "cycles_timed": args.c5_steps, "tokens_timed": n_tok,
          "verify_rows": C5_SEQ * 4, "draft_rows": C5_SEQ,
          "gemv_path": "IQ4_XS: all 32 rows in one sweep on tcgen05 (qb_qmv_tcw); Q6_K head / Q8_0 in 8-row "
                       "mma.sync chunks",
          "seq0_tokens_equal_single": bool(np.array_equal(seq0, alone))}
    return c5, model


def shards_of(world, tp):
    """GPUs the weights are split over (each streams 1/shards of them)."""
    return world if tp else 1


def aggregate(ms, n_tok, tp, dist=None, device="cpu"):
    """Whole-job throughput from this rank's (device ms, tokens) and, under
    torch.distributed, every other rank's: the slowest rank's time over the tokens
    of all ranks (replicas), or of the one sequence they share (tensor
    parallelism).  Returns (tok/s, max ms, tokens counted).  device: where the
    collective's tensor lives (cuda for NCCL, cpu for gloo)."""
    import torch
    if dist is None:
        return float(n_tok) / (ms / 1e3), float(ms), float(n_tok)
    t = torch.tensor([ms, float(n_tok)], dtype=torch.float64, device=device)
    mx = t.clone()
    dist.all_reduce(mx[:1], op=dist.ReduceOp.MAX)
    dist.all_reduce(t[1:], op=dist.ReduceOp.SUM)
    ms_max, tok_sum = float(mx[0]), float(t[1])
    if tp:
        tok_sum = float(n_tok)   # the ranks decoded the same tokens
    return tok_sum / (ms_max / 1e3), ms_max, tok_sum


def bench_config(args, world, tp):
    """The `config` object both arms print (the same workload)."""
    return {"workload": WORKLOAD, "prompt": PROMPT_LEN, "cycles_timed": args.steps,
            "l2": "weights 15 GB per cycle >> 126 MB L2 (no flush needed)",
            "parallelism": f"tp x{world}" if tp else f"replicas x{world}"}


def run_reference(args, rank, world):
    if rank != 0:
        return
    path = gguf_path(0, 1)
    n_threads = os.cpu_count()
    v, sample, _ = cpu_reference_run(path, n_threads, args.warmup, args.steps)
    if v is None:
        emit({"impl": "reference", "unavailable": sample})
        return
    cfg = bench_config(args, world, world > 1 and args.parallel == "tp")
    line = {"impl": "reference", "platform": "host CPU, reference AVX2 engine", "metric": METRIC, "value": v,
            "unit": "tok/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp32", "data": "synthetic (seeded random weights, random prompt)",
            "config": cfg,
            "cpu_baseline": {"value": v, "unit": "tok/s", "cores": n_threads, "kind": "reference", "sample": sample},
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    emit(line)


def run_ours(args, rank, world, local_rank):
    import torch
    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import torch.distributed as dist
    tp = world > 1 and args.parallel == "tp"
    seq_rank = 0 if tp else rank   # tensor parallelism: one sequence for all ranks
    path = gguf_path(rank, world)
    n_ctx = max(1024, PROMPT_LEN + 4 * (args.warmup + args.steps) + 64)

    def open_model(n_ctx):
        t0 = time.time()
        if tp:
            m = qb.Model(path, n_ctx, rank, world)
            handles = [None] * world
            dist.all_gather_object(handles, m.tp_handle())
            m.tp_connect(handles)
            dist.barrier()
        else:
            m = qb.Model(path, n_ctx)
        print(f"[bench r{rank}] model_init {time.time() - t0:.1f}s", file=sys.stderr, flush=True)
        return m

    def close_model(m):
        torch.cuda.synchronize()
        if dist:
            dist.barrier()   # tensor parallelism: no rank still writes into a peer's buffers
        m.close()
        if dist:
            dist.barrier()

    model = open_model(n_ctx)
    if not tp:
        model.enable_wide()   # prompts in 32-token chunks, IQ4_XS on the wide tcgen05 GEMM
    forced = forced_schedule()

    # ---- device-timed value: K speculative cycles ----
    model.prefill(prompt_tokens(seq_rank), 1)
    prefill_logits = model.logits()
    log("prefill done")
    warm_t, warm_j = model.spec_generate(10 ** 6, 3, forced=forced, max_cycles=args.warmup)
    log("warmup done")
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    with Clocks(local_rank) as clk:
        toks, js = model.spec_generate(10 ** 6, 3, forced=np.roll(forced, -args.warmup), max_cycles=args.steps)
        ms = model.last_loop_ms()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    n_tok = len(toks)
    log(f"timed: {args.steps} cycles {n_tok} tokens {ms:.1f} ms")
    value, ms_max, tok_sum = aggregate(ms, n_tok, tp, dist, "cuda")

    # ---- parity of the stream just timed (from the first cycle after prefill) ----
    stream_t, stream_j = np.concatenate([warm_t, toks]), np.concatenate([warm_j, js])
    parity = {}
    gold = golden_full()
    if gold is not None and seq_rank == 0:
        parity["golden"] = stream_parity(stream_t, stream_j, gold["tokens"], gold["accept"])
        parity["golden"]["prefill_logits_rel_l2"] = rel_l2(prefill_logits[:: int(gold["sub_stride"])],
                                                           gold["prefill_sub"])
    if tp:   # every rank decoded the one sequence: all streams must be rank 0's
        mine = (stream_t.tobytes(), stream_j.tobytes())
        every = [None] * world
        dist.all_gather_object(every, mine)
        parity["ranks_agree"] = all(e == every[0] for e in every)

    # ---- end to end through the public C ABI: one request = reset + prefill(128)
    #      + decode 512 tokens, host buffers in and out, wall clock ----
    e2e_runs = []
    h2d = d2h = 0
    for rep in range(2):
        prompt = prompt_tokens(seq_rank)
        torch.cuda.synchronize()
        t1 = time.perf_counter()
        model.reset()
        model.prefill(prompt, 1)
        out, jj = model.spec_generate(512, 3, forced=forced, max_cycles=4096)
        t2 = time.perf_counter()
        e2e_runs.append(len(out) / (t2 - t1))
        h2d = prompt.nbytes + forced.nbytes + 4 * model.E + 64
        d2h = out.nbytes + jj.nbytes + 4 * (model.V + model.E) * 2
    e2e = max(e2e_runs[1:]) if len(e2e_runs) > 1 else e2e_runs[0]
    log(f"e2e {e2e_runs}")

    # ---- components (device events on the model's stream) ----
    hbm, peak_kind = peaks()
    kernels_per_cycle, _ = model.bench(4, 0, 1)
    ms_gemv, b_gemv = model.bench(1, 4, 3)        # FFN gate+up, N=4, over all 64 layers
    ms_head, b_head = model.bench(3, 4, 20)
    ms_draft, b_draft = model.bench(2, 1, 10)
    ms_ver, b_ver = model.bench(0, 4, 10)        # verify step (64 layers + head, B=4)
    ms_tok, b_tok = model.bench(0, 1, 10)        # one-token forward (64 layers + head): C2's bytes per token
    c1 = {}
    for n in (1, 2, 4):                          # C1: one 17408 x 5120 IQ4_XS matrix, rotated over 64 copies
        ms_c1, b_c1 = model.bench(8, n, 5)
        gbs = b_c1 / shards_of(world, tp) / (ms_c1 / 1e3) / 1e9
        c1[f"n{n}"] = {"us": ms_c1 * 1e3, "GB/s": gbs, "frac": gbs / peaks()[0]}
    if not tp:   # the prefill / multi-stream width: 16 vectors per sweep on tcgen05, beside 2 x 8 on mma.sync
        ms_8, _ = model.bench(8, 8, 5)
        for nw in (16, 32):   # one sweep on the scale-folded tcgen05 GEMM
            ms_w, b_w = model.bench(10, nw, 5)
            c1[f"n{nw}_tcgen05"] = {"us": ms_w * 1e3, "GB/s": b_w / (ms_w / 1e3) / 1e9,
                                   "frac": b_w / (ms_w / 1e3) / 1e9 / peaks()[0],
                                   f"us_as_{nw // 8}x8_mma_sync": nw // 8 * ms_8 * 1e3}
    # C2: 128-token prompt (plain prefill), then 256 greedy tokens on the device
    gold = golden_full()
    model.reset()
    model.prefill(prompt_tokens(seq_rank), 0)
    g_toks = model.greedy_generate(256)
    ms_g = model.last_loop_ms()
    c2_tps = (len(g_toks) - 1) / (ms_g / 1e3)
    c2_gbs = b_tok / shards_of(world, tp) * c2_tps / 1e9
    c2 = {"tok/s": c2_tps, "ms_per_token": ms_g / max(len(g_toks) - 1, 1), "GB/s": c2_gbs,
          "frac": c2_gbs / peaks()[0], "bytes_per_token": b_tok,
          "tokens_equal_golden": bool(gold is not None and seq_rank == 0 and
                                      np.array_equal(g_toks[:len(gold["greedy"])], gold["greedy"]))}
    c4 = run_c4(args, model, open_model, close_model, seq_rank, ms_ver) if not args.no_c4 else None
    if c4 is not None:
        model = c4.pop("_model")
    c5 = None
    if not tp and not args.no_c5:   # multi-sequence decode runs on one GPU (replicas: one set per GPU)
        c5, model = run_c5(args, model, open_model, close_model)
    log(f"components gemv {ms_gemv:.4f} head {ms_head:.4f} draft {ms_draft:.3f} verify {ms_ver:.3f} ms")
    shards = world if tp else 1   # each GPU streams 1/shards of the weights
    gemv_gbs = b_gemv / shards / (ms_gemv / 1e3) / 1e9
    ver_gbs = b_ver / shards / (ms_ver / 1e3) / 1e9

    line = None
    if rank == 0:
        cpu_v, cpu_sample = (None, None)
        if world == 1 and not args.no_cpu:
            log("cpu reference sample")
            cpu_v, cpu_sample, ref = cpu_reference_run(path, os.cpu_count(), 1, 400, time_budget=args.cpu_seconds)
            if ref is not None:   # the reference's own stream on the same box, same inputs
                parity["reference_live"] = stream_parity(stream_t, stream_j, ref["tokens"], ref["accept"])
                parity["reference_live"]["prefill_logits_rel_l2"] = rel_l2(prefill_logits, ref["prefill_logits"])
                c2["reference_cpu_tok/s"] = ref["greedy_tok_s"]
                if c4 is not None:   # prefill rate of the reference on the 128-token prompt (8-token chunks)
                    c4["reference_cpu_prefill_tok/s"] = ref["prefill_tok_s"]
            log("cpu reference C1 micro")
            c1["reference_cpu"] = cpu_micro_c1(os.cpu_count())
        checks = [v for v in parity.values() if isinstance(v, dict)]
        parity["tokens_equal"] = bool(checks) and all(c["tokens_equal"] for c in checks) and \
            parity.get("ranks_agree", True)
        parity["accept_equal"] = bool(checks) and all(c["accept_equal"] for c in checks)
        parity["logits_rel_l2"] = max((c["prefill_logits_rel_l2"] for c in checks), default=None)
        parity["n_tokens"] = max((c["n_tokens"] for c in checks), default=0)
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
            "scaling": "strong" if tp else "weak", "vs_baseline": None, "dtype": "fp32",
            "data": "synthetic (seeded random weights, random prompt)",
            "config": bench_config(args, world, tp),
            "run": {"tokens_timed": int(tok_sum), "mean_accept": float(np.mean(js)) if len(js) else None},
            "parity": parity,
            "gpu_launches": int(kernels_per_cycle) * args.steps,
            "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "step": "one request: reset + prefill 128 + decode 512 tokens"},
            "roofline": {"bound": "hbm", "kernel": "qmv IQ4_XS (FFN gate+up fused, N=4)", "achieved": gemv_gbs,
                         "peak": hbm, "unit": "GB/s", "frac": gemv_gbs / hbm,
                         "traffic": (profiled_traffic() / shards) if profiled_traffic() else None,
                         "algorithmic_bytes": b_gemv / shards,
                         "peak_kind": peak_kind},
            "verify_step": {"ms": ms_ver, "bytes": b_ver, "bytes_per_gpu": b_ver / shards, "GB/s": ver_gbs,
                            "frac": ver_gbs / hbm},
            "configs": {"C1 IQ4_XS 17408x5120 GEMV (64 rotated copies)": c1,
                        "C2 greedy decode, prompt 128 + 256 tokens": c2,
                        "C4 long context, prompt 2048 + 1024 speculative tokens": c4,
                        "C5 multi-sequence, 8 sequences x (k=3 -> 4) = 32 verify rows": c5},
            "draft_ms": ms_draft, "head_ms": ms_head,
            "head_GB/s": b_head / shards / (ms_head / 1e3) / 1e9,
            "clocks": clk.summary(),
        }
        if cpu_v is not None:
            line["cpu_baseline"] = {"value": cpu_v, "unit": "tok/s", "cores": os.cpu_count(), "kind": "reference",
                                    "sample": cpu_sample}
    close_model(model)
    if line:
        emit(line)


def run_components(args):
    """Component timings only (used for ncu captures on a small model): shape
    wide4 = the benchmark widths with 4 layers (~3 GB on the device)."""
    import torch
    torch.cuda.set_device(0)
    shape = {"full": qb.FULL, "wide4": qb.WIDE4}[args.shape]
    d = "/dev/shm" if os.path.isdir("/dev/shm") else "/tmp"
    path = os.path.join(d, f"qb_bench_{args.shape}_seed{SEED}.gguf")
    if not os.path.exists(path):
        qb.write_synth_gguf(path + ".tmp", shape, seed=SEED)
        os.replace(path + ".tmp", path)
    model = qb.Model(path, 1024)
    model.prefill(prompt_tokens(0), 1)
    out = {}
    for name, what, arg, iters in [("ffn_gate_up_n4", 1, 4, args.iters), ("ffn_gate_up_n1", 1, 1, args.iters),
                                   ("head_n4", 3, 4, args.iters), ("head_n1", 3, 1, args.iters),
                                   ("draft", 2, 1, args.iters), ("verify_b4", 0, 4, args.iters),
                                   # these run on stale activations (timing only): after the others
                                   ("ffn_down_n4", 5, 4, args.iters), ("out_proj_n4", 6, 4, args.iters),
                                   ("in_proj_n4", 7, 4, args.iters),
                                   # FFN up on the wide tcgen05 GEMM (multi-sequence verify / 32 rows)
                                   ("tcw_ffn_up_n32", 10, 32, args.iters), ("tcw_ffn_up_n16", 10, 16, args.iters)]:
        if args.only and name not in args.only.split(","):
            continue
        ms, b = model.bench(what, arg, iters)
        out[name] = {"ms": ms, "bytes": b, "GB/s": b / ms / 1e6}
    model.close()
    if not args.only or "prefill32" in args.only.split(","):
        # one 32-token prefill chunk (the C4 chunk: IQ4_XS on the wide tcgen05 GEMM, the
        # recurrence over all 32 tokens, attention as 4 groups of 8), device-timed: a
        # 65-token prompt (two such chunks and a last token with the head) less a 33-token one
        model = qb.Model(path, 1024)
        model.enable_wide()
        best = {}
        for n in (33, 65) * (max(args.iters, 1) + 1):
            model.reset()
            model.prefill(prompt_tokens(0)[:n], 1)
            best[n] = min(best.get(n, 1e30), model.last_loop_ms())
        model.close()
        ms = best[65] - best[33]
        out["prefill32"] = {"ms": ms, "tok/s": 32 / ms * 1e3, "ms_33": best[33], "ms_65": best[65]}
    emit(out)


def main():
    global _RESULT_FD
    sys.stdout.flush()
    _RESULT_FD = os.dup(1)   # the JSON line goes here; stray prints of any library to stderr
    os.dup2(2, 1)
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=20.0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-c4", action="store_true", help="skip the long-context configuration C4")
    ap.add_argument("--no-c5", action="store_true", help="skip the multi-sequence configuration C5")
    ap.add_argument("--c5-steps", type=int, default=40, help="timed multi-sequence cycles (C5)")
    ap.add_argument("--mode", default="bench", choices=["bench", "components"])
    ap.add_argument("--shape", default="wide4", choices=["wide4", "full"])
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--only", default="")
    ap.add_argument("--parallel", default="tp", choices=["tp", "replicas"],
                    help="N > 1: one sequence over all GPUs (tp, the default) or one sequence per GPU "
                         "(replicas)")
    args = ap.parse_args()
    if args.mode == "components":
        run_components(args)
        return
    args.warmup = max(args.warmup, 3)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if world > 1:
        import torch
        import torch.distributed as dist
        from datetime import timedelta
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=timedelta(seconds=600))
    run_ours(args, rank, world, local_rank)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
