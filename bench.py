"""Benchmarks of the VAULT v3 inference path on B200 (config 1 is the default headline).

--config 1  VAULT v3 1.54B Q8_0, batch 1: one step = one request (reset the fixed state, chunked prefill of a
            128-token random prompt, 64 greedy decode steps).  Headline: decode tok/s.
--config 2  Hybrid Q4_0, batch 1: one step = one request of a 2,560-token prompt + 256 greedy decode steps (the W=1024
            window rolls over twice).
--config 3  Batched decode, Q8_0 with the segment scorer (layers 8/16/24, seg_budget 1024): 64 sequences, each a
            512-token ChatML system prefix (auto-pinned) and a 4,096-token random body with break id 198 every U[16,48]
            tokens, sharded 64/N per GPU (strong scaling).  The prompts are prefilled once (prefill tok/s); one step
            = one greedy decode step of every sequence of the rank.
--config 4  Long-context stream, BF16 weights (norms / biases / scorer F32): batch 1, a 256-token terminated system
            prefix + random body with break ids, 100,000 tokens prefilled once (prefill tok/s, arena size checked
            constant), then one step = one decode step.
--config 5  Kernel sweep: the tensor-core GEMM (and the decode GEMV at M <= 8) over Q8_0 / Q4_0 N x K shapes at
            M in {1, 8, 32, 128, 512}; decode attention over 3,584 keys (512 sinks + 1,024 bank + 2,048 window) at
            batch {1, 16, 64}.  Prints one JSON line per kernel case plus a summary line.

Timing: W untimed warm-up steps, then K timed steps bracketed by barrier + synchronize; device time from CUDA events
on the engine's stream; max over ranks; whole-job rates.  Weights (1.0-3.1 GB) exceed the 126 MB L2, so every step
streams them from HBM.  `e2e` repeats the decode through the C ABI with HOST buffers (v3g_step_host).
`cpu_baseline` / `--impl reference` time the reference's own C runtime (runtime/vault3_host, built by oracle/Makefile
from the reference sources) on the same model file with all host cores.
"""

from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import threading
import time

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

REF_HOST = os.path.join(HERE, "oracle", "_ref", "vault3_host")
SCORER = dict(seg_layers=(8, 16, 24), seg_budget=1024, seg_hidden=256, seg_min=16, seg_max=48)
# BASELINE configs (--config).  traffic: DRAM bytes (read + write) of one launch of the roofline kernel from the ncu
# capture summarised in `profile` (None: not captured for that config).
CONFIGS = {
    1: dict(kind="request", fmt="q8_0", prompt=128, decode=64, batch=1, model={},
            metric="decode tok/s (B=1, Q8_0, 128-token prompt, 64 greedy steps)",
            workload="BASELINE config 1: VAULT v3 1.54B Q8_0, B=1, 128-token prompt + 64 greedy decode steps",
            traffic=1650602240, profile="profiles/k_decode_q8_0_config1.md"),
    2: dict(kind="request", fmt="q4_0", prompt=2560, decode=256, batch=1, model={},
            metric="decode tok/s (B=1, Hybrid Q4_0, 2,560-token prompt, 256 greedy steps)",
            workload="BASELINE config 2: VAULT v3 1.54B Hybrid Q4_0, B=1, 2,560-token prompt + 256 greedy decode steps "
                     "(the W=1024 window rolls over twice)",
            traffic=None, profile=None),
    3: dict(kind="batched", fmt="q8_0", prompt=4608, decode=128, batch=64, model=SCORER,
            metric="decode tok/s (B=64 sequences sharded over the GPUs, Q8_0, per-sequence segment memory)",
            workload="BASELINE config 3: VAULT v3 1.54B Q8_0 + segment scorer, 64 sequences x (512-token pinned "
                     "prefix + 4,096-token body with break ids), greedy decode",
            traffic=None, profile=None),
    4: dict(kind="stream", fmt="bf16", prompt=100000, decode=128, batch=1, model=SCORER,
            metric="decode tok/s (B=1, BF16, after a 100,000-token prefill with a 256-token sink and segment memory)",
            workload="BASELINE config 4: VAULT v3 1.54B BF16 (F32 norms/biases/scorer), 100,000-token prompt "
                     "(256-token pinned prefix), W=1024, seg_budget 1024, then greedy decode",
            traffic=None, profile=None),
    5: dict(kind="sweep", fmt="q8_0", prompt=0, decode=0, batch=1, model={},
            metric="kernel sweep: GEMM GB/s and TFLOP/s, decode attention GB/s",
            workload="BASELINE config 5: Q8_0 / Q4_0 GEMM at N x K in {1536x1536, 256x1536, 8960x1536 (gate and up "
                     "together), 1536x8960, 151936x1536} x M in {1,8,32,128,512}; attention over 3,584 keys at B in "
                     "{1,16,64}",
            traffic=None, profile=None),
}
CONFIG = 1
FMT = CONFIGS[1]["fmt"]
PROMPT, DECODE = CONFIGS[1]["prompt"], CONFIGS[1]["decode"]
METRIC = CONFIGS[1]["metric"]
TRAFFIC = CONFIGS[1]["traffic"]


def select_config(n: int) -> None:
    """Point the module-level workload constants at BASELINE config n."""
    global CONFIG, FMT, PROMPT, DECODE, METRIC, TRAFFIC
    c = CONFIGS[n]
    CONFIG, FMT, PROMPT, DECODE, METRIC, TRAFFIC = n, c["fmt"], c["prompt"], c["decode"], c["metric"], c["traffic"]


def override_config(batch=None, prompt=None) -> None:
    """A smaller instance of the selected config (profiling captures): the workload text records the change."""
    global PROMPT, TRAFFIC
    c = CONFIGS[CONFIG]
    changes = []
    if batch is not None and batch != c["batch"]:
        c["batch"] = batch
        changes.append(f"{batch} sequences")
    if prompt is not None and prompt != c["prompt"]:
        c["prompt"] = PROMPT = prompt
        changes.append(f"{prompt}-token prompts")
    if changes:
        c["workload"] += " -- OVERRIDDEN to " + ", ".join(changes) + " (not the BASELINE size)"
        c["traffic"] = TRAFFIC = None


def model_path(fmt: str = "q8_0", model=None) -> str:
    from vault_b200 import synth
    return synth.full_model_file(fmt, seed=0, n_sink=0, **(model or {}))


def ensure_model(fmt: str, rank: int, barrier: bool = True, model=None) -> str:
    """Rank 0 writes the cached synthetic model file (once per box); the other ranks wait at the barrier."""
    import torch.distributed as dist
    path = model_path(fmt, model) if rank == 0 else None
    if barrier and dist.is_initialized():
        dist.barrier()
    return path or model_path(fmt, model)


def rank_max(values, device) -> list:
    """Element-wise maximum of per-rank values over every rank: the slowest rank sets each reported time.  Works on
    any process group (NCCL with CUDA tensors on the GPU box, gloo with CPU tensors in the tests)."""
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(v) for v in values], dtype=torch.float64, device=device)
    if dist.is_initialized():
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def aggregate_rate(world: int, units_per_rank: float, seconds: float) -> float:
    """Whole-job rate: every one of `world` ranks processed `units_per_rank` units in at most `seconds`."""
    return world * units_per_rank / seconds


def shard(n_total: int, rank: int, world: int) -> range:
    """Contiguous block of the n_total sequences served by `rank` (the path shards by sequence, no collective)."""
    per = n_total // world
    return range(rank * per, (rank + 1) * per)


def prompt_ids(seed: int, n: int = None):
    import numpy as np
    return np.random.default_rng(seed).integers(0, 151643, size=PROMPT if n is None else n).astype("int64")


def chat_prompt(seed: int, n_pin: int, total: int):
    """A ChatML system prefix closing at exactly n_pin tokens ([<|im_start|>, system, random..., <|im_end|>, '\\n']),
    then a random body with the break token 198 ('\\n', tier 1) after gaps drawn from U[16, 48]."""
    import numpy as np
    rng = np.random.default_rng(seed)
    ids = [151644, 8948] + rng.integers(0, 151643, size=n_pin - 4).tolist() + [151645, 198]
    while len(ids) < total:
        gap = int(rng.integers(16, 49))
        ids += rng.integers(0, 151643, size=gap).tolist() + [198]
    return np.asarray(ids[:total], dtype=np.int64)


class ClockSampler:
    """SM clocks and clock-event (throttle) reasons sampled during the timed region: every 10 ms through NVML
    (read-only queries), or every 200 ms through nvidia-smi when NVML cannot be loaded."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")
    # NVML clock-event reason bits: hw_slowdown, hw_thermal_slowdown, sw_thermal_slowdown, sw_power_cap
    NVML_BITS = (0x8, 0x40, 0x20, 0x4)

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.rows = []
        self.proc = None
        self.nvml = None
        self.stop = threading.Event()

    def __enter__(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nvml = pynvml
            self.handle = pynvml.nvmlDeviceGetHandleByIndex(self.gpu)
            self.t = threading.Thread(target=self._poll, daemon=True)
            self.t.start()
            return self
        except Exception:  # noqa: BLE001
            self.nvml = None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-i", str(self.gpu), "-lms", "200"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _poll(self):
        n = self.nvml
        while not self.stop.is_set():
            try:
                sm = n.nvmlDeviceGetClockInfo(self.handle, n.NVML_CLOCK_SM)
                mx = n.nvmlDeviceGetMaxClockInfo(self.handle, n.NVML_CLOCK_SM)
                rs = n.nvmlDeviceGetCurrentClocksThrottleReasons(self.handle)
                self.rows.append([str(self.gpu), str(sm), str(mx), "", hex(rs)] +
                                 ["Active" if rs & bit else "Not Active" for bit in self.NVML_BITS])
            except Exception:  # noqa: BLE001
                return
            self.stop.wait(0.01)

    def _read(self):
        for ln in self.proc.stdout:
            self.rows.append([c.strip() for c in ln.split(",")])

    def __exit__(self, *a):
        self.stop.set()
        if self.nvml is not None:
            self.t.join(timeout=2)
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if len(r) > 5 + i and r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


# ---------------------------------------------------------------------------------------------- reference arm
def ref_sample(cfg) -> tuple:
    """(prefill tokens, decode tokens) of one bounded reference run: the full request for configs 1-2; for 3 and 4
    (hours on the CPU) a prefix sample."""
    if cfg["kind"] == "request":
        return cfg["prompt"], cfg["decode"]
    return 2048, 64


def run_reference_host(path: str, threads: int, prefill: int, decode: int, timeout: int = 1800):
    """One run of the reference C runtime (runtime/vault3_host.c --bench: `prefill` synthetic prompt ids streamed
    token by token, then `decode` steps)."""
    r = subprocess.run([REF_HOST, path, "--threads", str(threads), "--bench-prefill", str(prefill),
                        "--bench", str(decode)], capture_output=True, text=True, timeout=timeout)
    if r.returncode != 0:
        raise RuntimeError(f"vault3_host failed: {r.stderr[-400:]}")
    return json.loads(r.stdout.strip().splitlines()[-1])


def reference_arm(args, rank: int, world: int) -> None:
    if rank != 0:
        return
    cfg = CONFIGS[CONFIG]
    if cfg["kind"] == "sweep":
        print(json.dumps({"impl": "reference", "unavailable": "config 5 is a GPU kernel sweep; the reference C runtime "
                                                              "has no kernel-level entry points"}))
        return
    if not os.path.exists(REF_HOST):
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/vault3_host not built (needs the reference "
                                                              "sources; run __graft_entry__.build() where they exist)"}))
        return
    path = ensure_model(FMT, 0, barrier=False, model=cfg["model"])
    threads = os.cpu_count() or 1
    pf, dc = ref_sample(cfg)
    for _ in range(args.warmup):
        run_reference_host(path, threads, pf, dc)
    t0 = time.perf_counter()
    runs = [run_reference_host(path, threads, pf, dc) for _ in range(args.steps)]
    wall = time.perf_counter() - t0
    value = dc * len(runs) / sum(r["decode_s"] for r in runs)
    sample = f"{args.steps} x ({pf}-token token-by-token prefill + {dc} decode steps), vault3_host --bench" + \
             ("" if cfg["kind"] == "request" else " (prefix sample of the workload; one sequence)")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * wall / args.steps, 3),
        "higher_is_better": True, "scaling": "weak" if cfg["kind"] == "request" else "strong", "vs_baseline": None,
        "dtype": f"{FMT} weights, fp32 compute",
        "data": "synthetic (random-init N(0,0.02) weights; vault3_host --bench prompt ids)",
        "config": {"workload": cfg["workload"], "global_batch": cfg["batch"], "seq_len": cfg["prompt"] + cfg["decode"],
                   "parallelism": "cpu threads"},
        "prefill_tok_s": round(sum(r["prefill_tokens"] for r in runs) / sum(r["prefill_s"] for r in runs), 3),
        "cpu_baseline": {"value": round(value, 3), "unit": "tok/s", "cores": runs[0]["threads"], "kind": "reference",
                         "sample": sample},
        "e2e": {"value": round(value, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))


def cpu_baseline(path: str, cfg) -> dict:
    pf, dc = ref_sample(cfg)
    try:
        r = run_reference_host(path, os.cpu_count() or 1, pf, dc)
        return {"value": r["decode_tok_s"], "unit": "tok/s", "cores": r["threads"], "kind": "reference",
                "sample": f"1 x ({pf}-token prefill + {dc} decode) with runtime/vault3_host --bench" +
                          ("" if cfg["kind"] == "request" else " (prefix sample of the workload, one sequence)")}
    except Exception as e:  # noqa: BLE001
        return {"value": None, "unit": "tok/s", "cores": os.cpu_count(), "kind": "reference",
                "sample": f"failed: {e}"[:200]}


# ---------------------------------------------------------------------------------------------- engine helpers
class Engine:
    """The model, one state and the ctypes handles of a rank."""

    def __init__(self, path, local_rank, batch, **state_kw):
        import torch
        from vault_b200 import _lib
        from vault_b200.model import VAULTv3ForCausalLM
        self.torch = torch
        self.L = _lib.lib()
        self.check = _lib.check
        self.m = VAULTv3ForCausalLM(path, device=local_rank, verify_crc=False)
        self.stream = torch.cuda.current_stream()
        self.sp = C.c_void_p(self.stream.cuda_stream)
        self.st = self.m.new_state(batch, **state_kw)
        self.dev = f"cuda:{local_rank}"

    def event(self):
        return self.torch.cuda.Event(enable_timing=True)

    def prefill(self, ids_dev, nxt):
        n = ids_dev.shape[1]
        self.check(self.L.v3g_prefill(self.st._h, C.c_void_p(ids_dev.data_ptr()), n, ids_dev.stride(0), None,
                                      C.c_void_p(nxt.data_ptr()), self.sp), "prefill")

    def generate(self, first, n, out):
        self.check(self.L.v3g_generate(self.st._h, C.c_void_p(first.data_ptr()), n, C.c_void_p(out.data_ptr()),
                                       out.stride(0), self.sp), "generate")

    def kv_bytes(self, pos: int) -> int:
        """fp16 K and V bytes one decode step reads at position pos (all layers, every sequence): the keys
        key_span() makes visible -- sinks and bank from 2W on (bank only with segment memory), the previous and the
        current chunk."""
        cfg = self.m.cfg
        total = 0
        for b in range(self.st.batch):
            si = self.st.info(b)
            W = cfg.window
            seg = si.mem_cnt if (si.seg_budget > 0 and cfg.seg_layers) else 0
            keys = ((si.n_pin + seg) if pos >= 2 * W else 0) + (W if pos >= W else 0) + pos % W + 1
            total += keys
        return total * cfg.n_layers * cfg.n_kv_heads * cfg.head_dim * 2 * 2


def peaks():
    p = os.path.join(HERE, "MEASURED_PEAKS.json")
    pk = json.load(open(p)) if os.path.exists(p) else {}
    return pk.get("hbm_gbs", 6650.0), pk.get("bf16_tflops", 1590.0), ("measured" if "hbm_gbs" in pk else "fallback")


def decode_launches(m, st, pos0: int, n_steps: int) -> int:
    """Kernel launches of n_steps greedy decode steps from position pos0 (graph replays launch the same kernels):
    k_begin + k_decode (persistent) or the per-layer tensor-core step + argmax + finish, with the scorer's two
    kernels when segment memory is on, and the boundary kernels at window rollovers."""
    cfg = m.cfg
    seg = st.seg_active
    if st.batch <= 8:
        per = 4 + (2 if seg else 0)
    else:   # tensor-core step: 4 prep + 4 GEMM + attention per layer, lm prep + GEMM
        per = 2 + 9 * cfg.n_layers + 2 + 2 + (2 if seg else 0)
    total = 0
    for p in range(pos0, pos0 + n_steps):
        total += per
        if p > 0 and p % cfg.window == 0:
            total += 2 + (2 if seg else 0)   # k_pin, k_prefix_rot (+ bank merge / gather)
    return total


def prefill_launches(m, st, n: int) -> int:
    """Kernel launches of a chunked prefill of n tokens per sequence from position 0."""
    cfg = m.cfg
    per_piece_cap = max(1, min(2048, st.batch * cfg.window) // st.batch)
    total, pos = 0, 0
    while pos < n:
        take = min(n - pos, cfg.window - pos % cfg.window, per_piece_cap)
        total += 1 + 9 * cfg.n_layers + 1 + (3 if st.seg_active else 0)
        if pos > 0 and pos % cfg.window == 0:
            total += 2 + (2 if st.seg_active else 0)
        pos += take
    return total + (st.batch + 7) // 8 + 1   # lm head GEMV passes and argmax of the last piece


# ---------------------------------------------------------------------------------------------- config kinds
def run_request(args, rank, world, local_rank):
    """Configs 1-2: each step is one request (reset, prefill, greedy decode)."""
    import numpy as np
    import torch
    import torch.distributed as dist
    cfg = CONFIGS[CONFIG]
    path = ensure_model(FMT, rank, model=cfg["model"])
    E = Engine(path, local_rank, 1)
    ids = torch.from_numpy(prompt_ids(1000 + rank)).to(E.dev, torch.int32)[None].contiguous()
    out = torch.empty(1, DECODE, dtype=torch.int32, device=E.dev)
    nxt = torch.empty(1, dtype=torch.int32, device=E.dev)

    def request(evs=None):
        E.st.reset()
        if evs:
            evs[0].record(E.stream)
        E.prefill(ids, nxt)
        if evs:
            evs[1].record(E.stream)
        E.generate(nxt, DECODE, out)
        if evs:
            evs[2].record(E.stream)

    for _ in range(args.warmup):
        request()
    torch.cuda.synchronize()
    evs = [[E.event() for _ in range(3)] for _ in range(args.steps)]
    start, end = E.event(), E.event()
    if dist.is_initialized():
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clk:
        start.record(E.stream)
        for i in range(args.steps):
            request(evs[i])
        end.record(E.stream)
        torch.cuda.synchronize()
    if dist.is_initialized():
        dist.barrier()
    total_ms = start.elapsed_time(end)
    pf_ms = sum(e[0].elapsed_time(e[1]) for e in evs)
    dec_ms = sum(e[1].elapsed_time(e[2]) for e in evs)
    total_ms, pf_ms, dec_ms = rank_max([total_ms, pf_ms, dec_ms], ids.device)
    E.st.check()

    # e2e: the same request through the C ABI with host buffers (one v3g_step_host call per token)
    host_ids = np.ascontiguousarray(prompt_ids(1000 + rank).astype(np.uint32))
    tok = np.zeros(1, np.uint32)
    nxt_h = np.zeros(1, np.uint32)

    def e2e_request():
        E.st.reset()
        torch.cuda.synchronize()
        for t in range(PROMPT):
            tok[0] = host_ids[t]
            E.check(E.L.v3g_step_host(E.st._h, tok.ctypes.data_as(C.c_void_p), None,
                                      nxt_h.ctypes.data_as(C.c_void_p), E.sp), "step_host")
        t1 = time.perf_counter()
        for _ in range(DECODE):
            tok[0] = nxt_h[0]
            E.check(E.L.v3g_step_host(E.st._h, tok.ctypes.data_as(C.c_void_p), None,
                                      nxt_h.ctypes.data_as(C.c_void_p), E.sp), "step_host")
        return time.perf_counter() - t1

    e2e_request()
    e2e = [e2e_request() for _ in range(max(1, min(args.steps, 5)))]
    e2e_dec = rank_max([sum(e2e)], ids.device)[0]
    e2e_value = aggregate_rate(world, DECODE * len(e2e), e2e_dec)

    # the persistent decode kernel (all layers + lm head of one token) timed alone at the request's mid-decode
    # position
    E.st.reset()
    E.prefill(ids, nxt)
    E.generate(nxt, DECODE // 2, out)
    pos = PROMPT + DECODE // 2
    kv = E.kv_bytes(pos)
    persistent = E.L.v3g_decode_pass(E.st._h, 1, E.sp) == 0
    kernel_s = None
    if persistent:
        for _ in range(3):
            E.check(E.L.v3g_decode_pass(E.st._h, 1, E.sp), "decode_pass")
        g0, g1 = E.event(), E.event()
        reps = 20
        g0.record(E.stream)
        for _ in range(reps):
            E.check(E.L.v3g_decode_pass(E.st._h, 1, E.sp), "decode_pass")
        g1.record(E.stream)
        torch.cuda.synchronize()
        kernel_s = g0.elapsed_time(g1) / 1e3 / reps
    E.st.reset()
    if rank != 0:
        return
    hbm, _, peak_kind = peaks()
    n_tok = DECODE * args.steps
    value = aggregate_rate(world, n_tok, dec_ms / 1e3)
    step_s = dec_ms / 1e3 / n_tok
    step_bytes = E.m.info.step_weight_bytes + kv
    achieved = step_bytes / kernel_s / 1e9 if kernel_s else None
    wgb = E.m.info.step_weight_bytes / 1e9
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(total_ms / args.steps, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": f"{FMT} weights; fp16 tensor-core operands (two fp16 parts per activation at batch 1), fp32 "
                 "accumulate; fp16 KV cache",
        "data": "synthetic (random-init N(0,0.02) weights, seeded uniform prompt ids)",
        "config": {"workload": CONFIGS[CONFIG]["workload"], "global_batch": world, "seq_len": PROMPT + DECODE,
                   "parallelism": f"sequence replicas x{world}",
                   "l2": f"weights ({wgb:.2f} GB) larger than L2 (126 MB); no flush needed"},
        "prefill_tok_s": round(aggregate_rate(world, PROMPT * args.steps, pf_ms / 1e3), 2),
        "ms_per_token": round(1e3 * step_s, 4),
        "gpu_launches": args.steps * (prefill_launches(E.m, E.st, PROMPT) + decode_launches(E.m, E.st, PROMPT, DECODE)),
        "roofline": {"kernel": "k_decode (persistent: 28 layers + lm head of one token, timed alone)", "bound": "hbm",
                     "achieved": round(achieved, 1) if achieved else None, "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 4) if achieved else None,
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs, burst copy)", "traffic": TRAFFIC,
                     "traffic_source": ("ncu dram__bytes_read.sum + dram__bytes_write.sum of one k_decode launch "
                                        f"({CONFIGS[CONFIG]['profile']})") if TRAFFIC else "not captured for this config",
                     "algorithmic_bytes_per_launch": int(step_bytes),
                     "avg_launch_us": round(kernel_s * 1e6, 2) if kernel_s else None},
        "step_roofline": {"bytes_per_step": int(step_bytes), "achieved": round(step_bytes / step_s / 1e9, 1),
                          "peak": hbm, "unit": "GB/s", "frac": round(step_bytes / step_s / 1e9 / hbm, 4)},
        "e2e": {"value": round(e2e_value, 2), "unit": "tok/s", "h2d_bytes_per_step": 4 * (PROMPT + DECODE),
                "d2h_bytes_per_step": 4 * (PROMPT + DECODE)},
        "clocks": clk.summary(),
    }
    if world == 1 and os.path.exists(REF_HOST) and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(path, CONFIGS[CONFIG])
    print(json.dumps(line))


def run_batched(args, rank, world, local_rank):
    """Config 3 (batched) and 4 (stream): one prefill of the rank's sequences, then one step = one decode step."""
    import numpy as np
    import torch
    import torch.distributed as dist
    cfg = CONFIGS[CONFIG]
    path = ensure_model(FMT, rank, model=cfg["model"])
    if cfg["kind"] == "batched":
        seqs = shard(cfg["batch"], rank, world)
        B = len(seqs)
        prompts = np.stack([chat_prompt(5000 + s, 512, PROMPT) for s in seqs])
        E = Engine(path, local_rank, B, per_sequence_memory=B > 1)
    else:
        B = 1
        prompts = chat_prompt(7000 + rank, 256, PROMPT)[None]
        E = Engine(path, local_rank, 1)
    ids = torch.from_numpy(prompts).to(E.dev, torch.int32).contiguous()
    nxt = torch.empty(B, dtype=torch.int32, device=E.dev)
    n_dec = args.warmup + args.steps
    out = torch.empty(B, n_dec, dtype=torch.int32, device=E.dev)
    arena0 = E.st.nbytes()
    torch.cuda.synchronize()
    p0, p1 = E.event(), E.event()
    p0.record(E.stream)
    E.prefill(ids, nxt)
    p1.record(E.stream)
    torch.cuda.synchronize()
    pf_ms = rank_max([p0.elapsed_time(p1)], ids.device)[0]
    E.st.check()
    si = E.st.info(0)
    # warm-up decode steps, then the timed ones (greedy, chained on the device)
    E.generate(nxt, args.warmup, out)
    first = out[:, args.warmup - 1].contiguous() if args.warmup else nxt
    torch.cuda.synchronize()
    pos_t = PROMPT + args.warmup
    kv_mid = E.kv_bytes(pos_t + args.steps // 2)
    start, end = E.event(), E.event()
    if dist.is_initialized():
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clk:
        start.record(E.stream)
        E.generate(first, args.steps, out[:, args.warmup:])
        end.record(E.stream)
        torch.cuda.synchronize()
    if dist.is_initialized():
        dist.barrier()
    dec_ms = rank_max([start.elapsed_time(end)], ids.device)[0]
    E.st.check()
    arena_const = E.st.nbytes() == arena0
    # e2e: decode steps through the C ABI with host buffers (B tokens in, B next tokens out per call)
    tok = np.ascontiguousarray(out[:, -1].cpu().numpy().astype(np.uint32))
    nxt_h = np.zeros(B, np.uint32)
    n_e2e = max(4, min(args.steps, 32))
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(n_e2e):
        E.check(E.L.v3g_step_host(E.st._h, tok.ctypes.data_as(C.c_void_p), None, nxt_h.ctypes.data_as(C.c_void_p),
                                  E.sp), "step_host")
        tok[:] = nxt_h
    e2e_s = rank_max([time.perf_counter() - t0], ids.device)[0]
    # the decode attention of every layer timed alone at the current position (the batched step's KV stream)
    att_s = None
    for layer in range(E.m.cfg.n_layers):
        E.check(E.L.v3g_attention(E.st._h, layer, E.sp), "attention")
    a0, a1 = E.event(), E.event()
    a0.record(E.stream)
    for _ in range(3):
        for layer in range(E.m.cfg.n_layers):
            E.check(E.L.v3g_attention(E.st._h, layer, E.sp), "attention")
    a1.record(E.stream)
    torch.cuda.synchronize()
    att_s = a0.elapsed_time(a1) / 1e3 / 3
    kv_now = E.kv_bytes(PROMPT + n_dec + n_e2e)
    if rank != 0:
        return
    hbm, _, peak_kind = peaks()
    value = aggregate_rate(world, B * args.steps, dec_ms / 1e3)
    step_s = dec_ms / 1e3 / args.steps
    wbytes = E.m.info.step_weight_bytes + (E.m.info.scorer_bytes if E.st.seg_active else 0)
    step_bytes = wbytes + kv_mid
    att_gbs = kv_now / att_s / 1e9
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(dec_ms / args.steps, 4), "higher_is_better": True,
        "scaling": "strong" if cfg["kind"] == "batched" else "weak", "vs_baseline": None,
        "dtype": f"{FMT} weights; fp16 tensor-core operands, fp32 accumulate; fp16 KV cache",
        "data": "synthetic (random-init N(0,0.02) weights, seeded ChatML prefixes + random bodies with break ids)",
        "config": {"workload": cfg["workload"], "global_batch": cfg["batch"] if cfg["kind"] == "batched" else world,
                   "sequences_per_gpu": B, "seq_len": PROMPT + n_dec,
                   "parallelism": f"sequences sharded {cfg['batch']}/{world}" if cfg["kind"] == "batched"
                   else f"sequence replicas x{world}",
                   "l2": "weights and KV cache larger than L2 (126 MB); no flush needed"},
        "prefill_tok_s": round(aggregate_rate(world, B * PROMPT, pf_ms / 1e3), 2),
        "prefill_s": round(pf_ms / 1e3, 3),
        "state": {"n_pin": si.n_pin, "mem_cnt": si.mem_cnt, "arena_bytes": arena0, "arena_constant": arena_const},
        "ms_per_token": round(1e3 * step_s, 4),
        "gpu_launches": decode_launches(E.m, E.st, pos_t, args.steps),
        "roofline": {"kernel": "decode step (every kernel of one batched step: weights once + every sequence's KV)",
                     "bound": "hbm", "achieved": round(step_bytes / step_s / 1e9, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(step_bytes / step_s / 1e9 / hbm, 4),
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs, burst copy)", "traffic": TRAFFIC,
                     "algorithmic_bytes_per_launch": int(step_bytes)},
        "attention_roofline": {"kernel": "k_attention (split-KV, up to 16 key tiles per item): 28 layers, every "
                                         "sequence",
                               "achieved": round(att_gbs, 1), "peak": hbm, "unit": "GB/s",
                               "frac": round(att_gbs / hbm, 4), "kv_bytes": int(kv_now),
                               "us_per_step": round(att_s * 1e6, 1)},
        "e2e": {"value": round(aggregate_rate(world, B * n_e2e, e2e_s), 2), "unit": "tok/s",
                "h2d_bytes_per_step": 4 * B, "d2h_bytes_per_step": 4 * B},
        "clocks": clk.summary(),
    }
    if world == 1 and os.path.exists(REF_HOST) and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(path, cfg)
    print(json.dumps(line))


def run_sweep(args, rank, world, local_rank):
    """Config 5: kernel sweep on one GPU."""
    import numpy as np
    import torch
    from vault_b200 import _lib
    from vault_b200.model import VAULTv3ForCausalLM
    if rank != 0:
        return
    hbm, tfl, peak_kind = peaks()
    L = _lib.lib()
    stream = torch.cuda.Stream()   # a side stream: graph capture is not allowed on the legacy default stream
    torch.cuda.set_stream(stream)
    sp = C.c_void_p(stream.cuda_stream)
    cases = []

    def time_it(fn, reps):
        """Device time per call: `reps` calls captured in one CUDA graph and replayed (no host launch overhead)."""
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for _ in range(reps):
                fn()
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        g.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        del g
        return e0.elapsed_time(e1) / 1e3 / reps

    li = 5
    shapes = [("q_proj 1536x1536", (li + 1) << 8 | 2, 1536, 1536), ("k_proj 256x1536", (li + 1) << 8 | 4, 256, 1536),
              ("gate+up 2x8960x1536", (li + 1) << 8 | 10, 17920, 1536), ("down 1536x8960", (li + 1) << 8 | 12, 1536, 8960),
              ("lm_head 151936x1536", 1, 151936, 1536)]
    for fmt in ("q8_0", "q4_0"):
        m = VAULTv3ForCausalLM(model_path(fmt), device=local_rank, verify_crc=False)
        for name, tid, N, K in shapes:
            wdt = "q8_0" if (fmt == "q8_0" or tid in (1, (li + 1) << 8 | 4)) else "q4_0"
            wbytes = N * K * (34 if wdt == "q8_0" else 18) // 32
            for M in (1, 8, 32, 128, 512):
                x = torch.randn(M, K, device=f"cuda:{local_rank}")
                y = torch.empty(M, N, device=x.device)
                nb = int(L.v3g_gemm_work_size(m._h, tid, M))
                work = torch.empty(nb, dtype=torch.uint8, device=x.device)
                kernels = [("tcgen05 GEMM", lambda: _lib.check(L.v3g_gemm(m._h, tid, C.c_void_p(x.data_ptr()), M,
                                                                         C.c_void_p(y.data_ptr()),
                                                                         C.c_void_p(work.data_ptr()), nb, sp), "gemm"))]
                if M <= 8:
                    kernels.append(("mma.sync GEMV", lambda: _lib.check(L.v3g_gemv(m._h, tid, C.c_void_p(x.data_ptr()), M,
                                                                                   C.c_void_p(y.data_ptr()), sp), "gemv")))
                for kname, fn in kernels:
                    s = time_it(fn, 20)
                    byt = wbytes + M * K * 2 + M * N * 4
                    fl = 2.0 * M * N * K
                    cases.append({"case": f"{wdt} {name}", "M": M, "kernel": kname, "us": round(s * 1e6, 2),
                                  "GB/s": round(byt / s / 1e9, 1), "hbm_frac": round(byt / s / 1e9 / hbm, 4),
                                  "TFLOP/s": round(fl / s / 1e12, 2), "tensor_frac": round(fl / s / 1e12 / tfl, 4)})
                    print(json.dumps(cases[-1]), flush=True)
        del m
        torch.cuda.empty_cache()
    # decode attention over 3,584 keys: 512 pinned sinks + 1,024 bank rows + 1,024 previous + 1,024 current keys
    m = VAULTv3ForCausalLM(model_path("q8_0", SCORER), device=local_rank, verify_crc=False)
    for B in (1, 16, 64):
        st = m.new_state(B, per_sequence_memory=B > 1)
        ids = torch.from_numpy(np.stack([chat_prompt(9000 + b, 512, 5 * 1024 - 1) for b in range(B)])).to(
            f"cuda:{local_rank}", torch.int32).contiguous()
        nxt = torch.empty(B, dtype=torch.int32, device=ids.device)
        _lib.check(L.v3g_prefill(st._h, C.c_void_p(ids.data_ptr()), ids.shape[1], ids.shape[1], None,
                                 C.c_void_p(nxt.data_ptr()), sp), "prefill")
        si = st.info(0)
        keys = si.n_pin + si.mem_cnt + 2 * 1024
        s = time_it(lambda: [_lib.check(L.v3g_attention(st._h, layer, sp), "attention") for layer in range(28)], 5) / 28
        byt = B * keys * 2 * 128 * 2 * 2
        cases.append({"case": f"decode attention, {keys} keys ({si.n_pin} sinks + {si.mem_cnt} bank + 2048 window)",
                      "B": B, "kernel": "k_attention (split-KV)", "us_per_layer": round(s * 1e6, 2),
                      "GB/s": round(byt / s / 1e9, 1), "hbm_frac": round(byt / s / 1e9 / hbm, 4)})
        print(json.dumps(cases[-1]), flush=True)
        del st
    print(json.dumps({"metric": METRIC, "config": {"workload": CONFIGS[5]["workload"]}, "n_cases": len(cases),
                      "peaks": {"hbm_gbs": hbm, "bf16_tflops": tfl, "source": peak_kind}}))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--config", type=int, default=1, choices=sorted(CONFIGS))
    ap.add_argument("--batch", type=int, default=None,
                    help="override the config's sequence count (a smaller case of the same path, e.g. for ncu "
                         "captures; the JSON line then names the override)")
    ap.add_argument("--prompt", type=int, default=None, help="override the config's prompt length (same use)")
    args = ap.parse_args()
    select_config(args.config)
    override_config(args.batch, args.prompt)
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local_rank))
    try:
        if args.impl == "reference":
            reference_arm(args, rank, world)
        else:
            import torch
            torch.cuda.set_device(local_rank)
            kind = CONFIGS[CONFIG]["kind"]
            if kind == "request":
                run_request(args, rank, world, local_rank)
            elif kind in ("batched", "stream"):
                run_batched(args, rank, world, local_rank)
            else:
                run_sweep(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
