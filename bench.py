"""Benchmark of the VAULT v3 decode path on B200 (BASELINE config 1 by default).

One bench "step" is one config-1 request: reset the fixed state, stream the 128-token random prompt, then decode
64 tokens greedily (batch 1, Q8_0 weights of the 1.54B architecture, random-init N(0, 0.02), W = 1024, no sinks).
`--config 2` runs BASELINE config 2 instead: Hybrid Q4_0 weights, a 2,560-token prompt and 256 decode steps.
The headline value is decode tokens/s (summed over ranks for --gpus N: every rank serves its own requests; the
path shards by sequence, so there is no collective on the data path -> "scaling": "weak").

Timing: W untimed warm-up steps, then K timed steps bracketed by barrier + synchronize; device time from CUDA
events on the engine's stream; max over ranks.  The weights (1.64 GB) exceed the 126 MB L2, so every decode step
streams them from HBM.  `e2e` repeats the request through the C ABI with HOST buffers (v3g_step_host: token in,
next token out, per call).  `cpu_baseline` / `--impl reference` time the reference's own C runtime
(runtime/vault3_host built by oracle/Makefile) on the same model file with all host cores.
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
# BASELINE configs this bench runs (--config; 1 is the headline).  traffic: DRAM bytes (read + write) of one k_decode
# launch from the ncu capture summarised in `profile` (None: not captured for that config).
CONFIGS = {
    1: dict(fmt="q8_0", prompt=128, decode=64,
            metric="decode tok/s (B=1, Q8_0, 128-token prompt, 64 greedy steps)",
            workload="BASELINE config 1: VAULT v3 1.54B Q8_0, B=1, 128-token prompt + 64 greedy decode steps",
            traffic=1650602240, profile="profiles/k_decode_q8_0_config1.md"),
    2: dict(fmt="q4_0", prompt=2560, decode=256,
            metric="decode tok/s (B=1, Hybrid Q4_0, 2,560-token prompt, 256 greedy steps)",
            workload="BASELINE config 2: VAULT v3 1.54B Hybrid Q4_0, B=1, 2,560-token prompt + 256 greedy decode steps "
                     "(the W=1024 window rolls over twice)",
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


def model_path(fmt: str = "q8_0") -> str:
    from vault_b200 import synth
    return synth.full_model_file(fmt, seed=0, n_sink=0)


def ensure_model(fmt: str, rank: int, barrier: bool = True) -> str:
    """Rank 0 writes the cached synthetic model file (once per box); the other ranks wait at the barrier."""
    import torch.distributed as dist
    path = model_path(fmt) if rank == 0 else None
    if barrier and dist.is_initialized():
        dist.barrier()
    return path or model_path(fmt)


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


def prompt_ids(seed: int):
    import numpy as np
    return np.random.default_rng(seed).integers(0, 151643, size=PROMPT).astype("int64")


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.rows = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-i", str(self.gpu), "-lms", "200"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for ln in self.proc.stdout:
            self.rows.append([c.strip() for c in ln.split(",")])

    def __exit__(self, *a):
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


def run_reference_host(path: str, threads: int, timeout: int = 600):
    """One config-1 request on the reference C runtime (runtime/vault3_host.c --bench mode)."""
    r = subprocess.run([REF_HOST, path, "--threads", str(threads), "--bench-prefill", str(PROMPT),
                        "--bench", str(DECODE)], capture_output=True, text=True, timeout=timeout)
    if r.returncode != 0:
        raise RuntimeError(f"vault3_host failed: {r.stderr[-400:]}")
    return json.loads(r.stdout.strip().splitlines()[-1])


def reference_arm(args, rank: int, world: int) -> None:
    if rank != 0:
        return
    path = ensure_model(FMT, 0, barrier=False)
    threads = os.cpu_count() or 1
    if not os.path.exists(REF_HOST):
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/vault3_host not built (needs the reference "
                                                              "sources; run __graft_entry__.build() where they exist)"}))
        return
    for _ in range(args.warmup):
        run_reference_host(path, threads)
    t0 = time.perf_counter()
    runs = [run_reference_host(path, threads) for _ in range(args.steps)]
    wall = time.perf_counter() - t0
    dec = sum(r["decode_s"] for r in runs)
    value = DECODE * len(runs) / dec
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * wall / args.steps, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": f"{FMT} weights, fp32 compute",
        "data": "synthetic (random-init N(0,0.02) weights, seeded uniform prompt ids; vault3_host --bench ids)",
        "config": {"workload": CONFIGS[CONFIG]["workload"], "global_batch": 1, "seq_len": PROMPT + DECODE,
                   "parallelism": "cpu threads"},
        "prefill_tok_s": round(sum(r["prefill_tokens"] for r in runs) / sum(r["prefill_s"] for r in runs), 3),
        "cpu_baseline": {"value": round(value, 3), "unit": "tok/s", "cores": runs[0]["threads"], "kind": "reference",
                         "sample": f"{args.steps} x ({PROMPT}-token token-by-token prefill + {DECODE} decode), "
                                   "vault3_host --bench"},
        "e2e": {"value": round(value, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))


def engine_arm(args, rank: int, world: int, local_rank: int) -> None:
    import numpy as np
    import torch
    import torch.distributed as dist
    from vault_b200 import _lib
    from vault_b200.model import VAULTv3ForCausalLM

    torch.cuda.set_device(local_rank)
    path = ensure_model(FMT, rank)
    m = VAULTv3ForCausalLM(path, device=local_rank, verify_crc=False)
    L = _lib.lib()
    stream = torch.cuda.current_stream()
    sp = C.c_void_p(stream.cuda_stream)
    st = m.new_state(1)
    ids = torch.from_numpy(prompt_ids(1000 + rank)).to(f"cuda:{local_rank}", torch.int32)[None].contiguous()
    out = torch.empty(1, DECODE, dtype=torch.int32, device=ids.device)
    nxt = torch.empty(1, dtype=torch.int32, device=ids.device)

    def request(evs=None):
        st.reset()
        if evs:
            evs[0].record(stream)
        _lib.check(L.v3g_prefill(st._h, C.c_void_p(ids.data_ptr()), PROMPT, PROMPT, None,
                                 C.c_void_p(nxt.data_ptr()), sp), "prefill")
        if evs:
            evs[1].record(stream)
        _lib.check(L.v3g_generate(st._h, C.c_void_p(nxt.data_ptr()), DECODE, C.c_void_p(out.data_ptr()), DECODE, sp),
                   "generate")
        if evs:
            evs[2].record(stream)

    for _ in range(args.warmup):
        request()
    torch.cuda.synchronize()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist.is_initialized():
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clk:
        start.record(stream)
        for i in range(args.steps):
            request(evs[i])
        end.record(stream)
        torch.cuda.synchronize()
    if dist.is_initialized():
        dist.barrier()
    total_ms = start.elapsed_time(end)
    pf_ms = sum(e[0].elapsed_time(e[1]) for e in evs)
    dec_ms = sum(e[1].elapsed_time(e[2]) for e in evs)
    total_ms, pf_ms, dec_ms = rank_max([total_ms, pf_ms, dec_ms], ids.device)
    st.check()

    # e2e: the same request through the C ABI with host buffers (one v3g_step_host call per token)
    host_ids = np.ascontiguousarray(prompt_ids(1000 + rank).astype(np.uint32))
    tok = np.zeros(1, np.uint32)
    nxt_h = np.zeros(1, np.uint32)

    def e2e_request():
        st.reset()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for t in range(PROMPT):
            tok[0] = host_ids[t]
            _lib.check(L.v3g_step_host(st._h, tok.ctypes.data_as(C.c_void_p), None,
                                       nxt_h.ctypes.data_as(C.c_void_p), sp), "step_host")
        t1 = time.perf_counter()
        for _ in range(DECODE):
            tok[0] = nxt_h[0]
            _lib.check(L.v3g_step_host(st._h, tok.ctypes.data_as(C.c_void_p), None,
                                       nxt_h.ctypes.data_as(C.c_void_p), sp), "step_host")
        return t1 - t0, time.perf_counter() - t1

    e2e_request()
    e2e = [e2e_request() for _ in range(max(1, min(args.steps, 5)))]
    e2e_dec = rank_max([sum(d for _, d in e2e)], ids.device)[0]
    e2e_value = aggregate_rate(world, DECODE * len(e2e), e2e_dec)

    # dominant kernel: the persistent decode kernel (all 28 layers + lm head of one token), timed alone on the
    # engine stream at the mean decode position of the request (prompt + 32)
    st.reset()
    _lib.check(L.v3g_prefill(st._h, C.c_void_p(ids.data_ptr()), PROMPT, PROMPT, None, C.c_void_p(nxt.data_ptr()), sp),
               "prefill")
    _lib.check(L.v3g_generate(st._h, C.c_void_p(nxt.data_ptr()), DECODE // 2, C.c_void_p(out.data_ptr()), DECODE, sp),
               "generate")
    # visible keys at this position (the KV rows one decode step reads): sinks and bank from 2W on, then the
    # previous and the current window chunk
    si = st.info()
    W, pos = m.cfg.window, PROMPT + DECODE // 2
    keys = ((si.n_pin + si.mem_cnt) if pos >= 2 * W else 0) + (W if pos >= W else 0) + pos % W + 1
    persistent = L.v3g_decode_pass(st._h, 1, sp) == 0
    kernel_s = None
    if persistent:
        for _ in range(3):
            _lib.check(L.v3g_decode_pass(st._h, 1, sp), "decode_pass")
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 20
        g0.record(stream)
        for _ in range(reps):
            _lib.check(L.v3g_decode_pass(st._h, 1, sp), "decode_pass")
        g1.record(stream)
        torch.cuda.synchronize()
        kernel_s = g0.elapsed_time(g1) / 1e3 / reps
    st.reset()

    if rank != 0:
        return
    peaks_path = os.path.join(HERE, "MEASURED_PEAKS.json")
    peaks = json.load(open(peaks_path)) if os.path.exists(peaks_path) else {}
    hbm = peaks.get("hbm_gbs", 6650.0)
    peak_kind = "measured" if "hbm_gbs" in peaks else "fallback"
    n_tok = DECODE * args.steps
    value = aggregate_rate(world, n_tok, dec_ms / 1e3)
    step_s = dec_ms / 1e3 / n_tok
    # KV bytes read per decode step (fp16 K and V of every visible key, 2 KV heads x 128, all layers) at the
    # request's mid-decode position
    kv_bytes = 28 * 2 * 2 * 128 * 2 * keys
    step_bytes = m.info.step_weight_bytes + kv_bytes
    kernel_bytes = step_bytes   # one launch of the persistent kernel reads every weight once plus the KV rows
    achieved = kernel_bytes / kernel_s / 1e9 if kernel_s else None
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(total_ms / args.steps, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": f"{FMT} weights; fp16 tensor-core operands, fp32 accumulate; fp16 KV cache",
        "data": "synthetic (random-init N(0,0.02) weights, seeded uniform prompt ids)",
        "config": {"workload": CONFIGS[CONFIG]["workload"], "global_batch": world, "seq_len": PROMPT + DECODE, "parallelism": f"sequence replicas x{world}",
                   "l2": "weights (1.64 GB) larger than L2 (126 MB); no flush needed"},
        "prefill_tok_s": round(aggregate_rate(world, PROMPT * args.steps, pf_ms / 1e3), 2),
        "ms_per_token": round(1e3 * step_s, 4),
        "gpu_launches": None,
        "roofline": {"kernel": "k_decode (persistent: 28 layers + lm head of one token, timed alone)", "bound": "hbm",
                     "achieved": round(achieved, 1) if achieved else None, "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 4) if achieved else None,
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs, burst copy)", "traffic": TRAFFIC,
                     "traffic_source": ("ncu dram__bytes_read.sum + dram__bytes_write.sum of one k_decode launch "
                                        f"({CONFIGS[CONFIG]['profile']})") if TRAFFIC else "not captured for this config",
                     "algorithmic_bytes_per_launch": int(kernel_bytes),
                     "avg_launch_us": round(kernel_s * 1e6, 2) if kernel_s else None},
        "step_roofline": {"bytes_per_step": int(step_bytes), "achieved": round(step_bytes / step_s / 1e9, 1),
                          "peak": hbm, "unit": "GB/s", "frac": round(step_bytes / step_s / 1e9 / hbm, 4)},
        "e2e": {"value": round(e2e_value, 2), "unit": "tok/s", "h2d_bytes_per_step": 4 * (PROMPT + DECODE),
                "d2h_bytes_per_step": 4 * (PROMPT + DECODE)},
        "clocks": clk.summary(),
    }
    # launches inside the timed region, per request: every token runs k_begin + k_decode (persistent) + k_finish,
    # plus k_argmax_partial when its next token is needed (the last prompt token and every decode step)
    if persistent:
        per_request = (PROMPT + DECODE) * 3 + (DECODE + 1)
    else:   # per-phase kernels: k_begin, 5 per layer, lm gemv (with lm head) and k_finish
        per_request = (PROMPT + DECODE) * (2 + 5 * 28) + (DECODE + 1) * 2
    line["gpu_launches"] = args.steps * per_request
    if world == 1 and os.path.exists(REF_HOST) and not args.no_cpu_baseline:
        try:
            r = run_reference_host(path, os.cpu_count() or 1)
            line["cpu_baseline"] = {"value": r["decode_tok_s"], "unit": "tok/s", "cores": r["threads"],
                                    "kind": "reference",
                                    "sample": f"1 x ({PROMPT}-token prefill + {DECODE} decode) with runtime/vault3_host "
                                              "--bench"}
        except Exception as e:  # noqa: BLE001
            line["cpu_baseline"] = {"value": None, "unit": "tok/s", "cores": os.cpu_count(), "kind": "reference",
                                    "sample": f"failed: {e}"[:200]}
    print(json.dumps(line))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--config", type=int, default=1, choices=sorted(CONFIGS))
    args = ap.parse_args()
    select_config(args.config)
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
            engine_arm(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
