#!/usr/bin/env python
"""Benchmark of the fused dequantize + GEMV decode path on B200.

Default workload (the metric's configuration): one
LLaMA-7B-shaped batch-1 decode token through the hot path = the 224 Q4_0
projections of 32 layers (q, k, v, o 4096x4096; gate, up 11008x4096; down
4096x11008) plus the 32000x4096 Q8_0 lm_head, all weights resident in HBM
(3.78 GB per token, far larger than the 126 MB L2, so no flush is needed).
Each projection's input is the previous projection's output (x -> q,k,v;
v -> o; o -> gate, up; up -> down; down -> next layer; -> lm_head), so the
launches form a real dependency chain.  Attention, RMSNorm, RoPE and SwiGLU
are the callers' torch ops and are not part of this path.

A step is one token.  ``value`` = tokens/s with inputs resident (the 225
launches of a token captured once in a CUDA graph with programmatic
dependent launch, replayed per token), timed with CUDA events, max over
ranks.  ``e2e`` = the same tokens/s through the reference-facing op API
(gds_io_ext.fused_dequant_gemv, called exactly as llama.py calls it) with
the token's input copied host->device and the logits device->host every step.
The same line also carries (unless --quick):
  * ``e2e_decode``: config 1 as BASELINE states it -- 128 greedy tokens after
    a 512-position prefill through GdsLLM's own CachedScheduler and
    transformer_block, unchanged (attention, norms, RoPE, KV cache and the
    full-table lm_head included), on this build's gds_io_ext (N = 1);
    ``e2e_decode_scheduler_ops``: the same with gdsllm_b200.scheduler_ops'
    embedding gather and fused lm_head installed;
  * ``config0``: the 11008x4096 Q4_0 GEMV's GB/s and roofline;
  * ``config3_tp``: the LLaMA-70B chain tensor-parallel over the N ranks;
  * ``config4_ep``: the MoE decode expert-parallel over the N ranks, batch 1
    and 8.

--impl reference: the reference's path on this box: its CPU path (its dequant
formula + torch.matmul on all host cores; the oracle port) as ``value``, and
GdsLLM's own CUDA kernels, compiled unchanged for sm_100a, on the same token
as ``ref_cuda``, and through the same unchanged scheduler as ``e2e_decode``.

--gpus N (under torchrun): N independent replicas of the default workload
(weak scaling); config 3 and 4 in the same line run across the N ranks.
--config 0: one 11008x4096 Q4_0 GEMV, rotating over copies larger than L2.
--config 2: Q8_0 / affine-Q4 sweep (4 shapes x batch 1, 4, 8, 16).
--config 3: LLaMA-70B-shaped decode chain, tensor-parallel over --gpus N (NCCL all-reduce).
--config 4: Qwen-MoE-shaped MoE decode, expert-parallel over --gpus N (--batch 1 or 8).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from gdsllm_b200 import synth  # noqa: E402

LAYERS, HIDDEN, FFN, VOCAB = 32, 4096, 11008, 32000
PROJ = [("q", HIDDEN, HIDDEN), ("k", HIDDEN, HIDDEN), ("v", HIDDEN, HIDDEN), ("o", HIDDEN, HIDDEN),
        ("gate", FFN, HIDDEN), ("up", FFN, HIDDEN), ("down", HIDDEN, FFN)]
SRC = {"q": "x", "k": "x", "v": "x", "o": "v", "gate": "o", "up": "o", "down": "up"}


def q4_bytes(n, k):
    return n * (k // 32) * 18


def q8_bytes(n, k):
    return n * (k // 32) * 34


def gemv_alg_bytes(n, k, wbytes):
    return wbytes + 2 * k + 2 * n  # weights + x + y (fp16)


LAYER_WBYTES = sum(q4_bytes(n, k) for _, n, k in PROJ)
TOKEN_WBYTES = LAYERS * LAYER_WBYTES + q8_bytes(VOCAB, HIDDEN)
TOKEN_ALG_BYTES = (LAYERS * sum(gemv_alg_bytes(n, k, q4_bytes(n, k)) for _, n, k in PROJ)
                   + gemv_alg_bytes(VOCAB, HIDDEN, q8_bytes(VOCAB, HIDDEN)))


def load_peaks():
    try:
        p = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ---------------------------------------------------------------------------
# distributed plumbing

class Dist:
    def __init__(self, sample_clocks: bool = True):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        # rank 0 samples its GPU's clocks; started before any GPU work
        self.clocks = ClockSampler(self.local) if (sample_clocks and self.rank == 0) else None
        torch.cuda.set_device(self.local)
        self.device = torch.device("cuda", self.local)
        if self.world > 1:
            import datetime
            import torch.distributed as dist
            # Rank 0's stdout carries exactly one JSON line: keep NCCL's
            # version banner (printed at NCCL_DEBUG=VERSION) off it.
            if os.environ.get("NCCL_DEBUG", "VERSION").upper() == "VERSION":
                os.environ["NCCL_DEBUG"] = "WARN"
            dist.init_process_group("nccl", device_id=self.device,
                                    timeout=datetime.timedelta(seconds=120))

    def barrier(self):
        if self.world > 1:
            import torch.distributed as dist
            dist.barrier()

    def max(self, v: float) -> float:
        if self.world == 1:
            return v
        import torch.distributed as dist
        t = torch.tensor([v], dtype=torch.float64, device=self.device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.clocks is not None:
            self.clocks.close()
        if self.world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


# ---------------------------------------------------------------------------
# clocks during the timed region

class ClockSampler:
    """nvidia-smi samples every 100 ms for the whole run (started before any
    GPU work, so that its start-up -- NVML initialisation of the box -- never
    overlaps a timed region); window() returns the statistics of the samples
    whose timestamps fall inside one timed region."""
    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.proc = None
        self.lines = []
        cvd = os.environ.get("CUDA_VISIBLE_DEVICES")
        target = str(device_index)
        if cvd:
            ids = [c.strip() for c in cvd.split(",") if c.strip()]
            if device_index < len(ids):
                target = ids[device_index]
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", target],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, FileNotFoundError):
            self.proc = None
            return
        import threading
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line)

    def start(self):
        self.t0 = time.time()

    def stop(self):
        if self.proc is None:
            return None
        t1 = time.time()
        time.sleep(0.25)  # let the sample covering the window's end arrive
        import datetime
        sm, smax, reasons, power = [], 0.0, set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in list(self.lines):
            f = [c.strip() for c in line.split(",")]
            if len(f) < 10:
                continue
            try:
                ts = datetime.datetime.strptime(f[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                if not (self.t0 - 0.05 <= ts <= t1 + 0.05):
                    continue
                sm.append(float(f[2]))
                smax = max(smax, float(f[3]))
                power.append(float(f[4]))
            except ValueError:
                continue
            for name, val in zip(names, f[6:10]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm), "power_w_max": max(power) if power else None}

    def close(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.proc = None


# ---------------------------------------------------------------------------
# the token's weights and activations

class Token:
    """Resident weights of a LLaMA-7B-shaped model (Q4_0 body, Q8_0 lm_head),
    one uint8 buffer per layer with 4 KB-aligned tensor offsets like the
    reference's layer files, and preallocated activations."""

    def __init__(self, device, seed=0):
        self.device = device
        self.layers = []
        for li in range(LAYERS):
            offs, cur = {}, 0
            for name, n, k in PROJ:
                offs[name] = (cur, n, k)
                cur += (q4_bytes(n, k) + 4095) // 4096 * 4096
            buf = torch.empty(cur, dtype=torch.uint8, device=device)
            for pi, (name, n, k) in enumerate(PROJ):
                o = offs[name][0]
                w = synth.q4_0_weight(n, k, seed=seed * 1000 + li * 8 + pi, device=device)
                buf[o:o + w.numel()] = w.reshape(-1)
                del w
            self.layers.append((buf, offs))
        self.lm_head = synth.q8_0_weight(VOCAB, HIDDEN, seed=seed * 1000 + 999, device=device)
        self.x0 = synth.activations(1, HIDDEN, seed=seed + 7, device=device).reshape(-1)
        self.act = {"x": torch.empty(HIDDEN, dtype=torch.float16, device=device)}
        for name, n, _ in PROJ:
            self.act[name] = torch.empty(n, dtype=torch.float16, device=device)
        self.layer_out = [torch.empty(HIDDEN, dtype=torch.float16, device=device) for _ in range(LAYERS)]
        self.logits = torch.empty(VOCAB, dtype=torch.float16, device=device)

    def launches(self):
        """(weight ptr, n, k, x ptr, y ptr, fmt) for the 225 GEMVs of a token."""
        seq = []
        x_ptr = self.act["x"].data_ptr()
        for li, (buf, offs) in enumerate(self.layers):
            cur = {"x": x_ptr}
            for name, n, k in PROJ:
                y = self.layer_out[li] if name == "down" else self.act[name]
                seq.append((buf.data_ptr() + offs[name][0], n, k, cur[SRC[name]], y.data_ptr(), "q4_0"))
                cur[name] = y.data_ptr()
            x_ptr = self.layer_out[li].data_ptr()
        seq.append((self.lm_head.data_ptr(), VOCAB, HIDDEN, x_ptr, self.logits.data_ptr(), "q8_0"))
        return seq

    def grouped(self):
        """The same 225 GEMVs with the projections that read one input
        sharing a launch: per layer (q, k, v) from x, o, (gate, up) from o,
        down -- 129 launches.  Entries are lists of (w, n, k, x, y, fmt)."""
        seq = self.launches()
        out, i = [], 0
        while i < len(seq):
            j = i + 1
            while (j < len(seq) and j - i < 4 and seq[j][3] == seq[i][3] and seq[j][2] == seq[i][2]
                   and seq[j][5] == seq[i][5]):
                j += 1
            out.append(seq[i:j])
            i = j
        return out


def run_ours(seq, stream, lib):
    for w, n, k, x, y, fmt in seq:
        fn = lib.gdsq_fused_q4_0_gemv if fmt == "q4_0" else lib.gdsq_fused_q8_0_gemv
        st = fn(w, x, y, n, k, 1, stream)
        if st:
            raise RuntimeError(lib.gdsq_last_error().decode())


def run_grouped(groups, stream, lib):
    import ctypes
    for grp in groups:
        if len(grp) == 1:
            run_ours(grp, stream, lib)
            continue
        c = len(grp)
        wa = (ctypes.c_void_p * c)(*[e[0] for e in grp])
        na = (ctypes.c_int * c)(*[e[1] for e in grp])
        ya = (ctypes.c_void_p * c)(*[e[4] for e in grp])
        st = lib.gdsq_fused_gemv_group(0 if grp[0][5] == "q4_0" else 1, c, wa, na, ya, grp[0][3], grp[0][2], 1,
                                       stream)
        if st:
            raise RuntimeError(lib.gdsq_last_error().decode())


def capture(fn):
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn(s.cuda_stream)  # warm-up outside capture (sets kernel attributes)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    with torch.cuda.graph(g):
        fn(torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return g


STEP_STATS = {}


def time_graph(g, steps, warmup, dist, clocks=None, per_step=False):
    """Replays `g` `steps` times between CUDA events on the current stream;
    returns (max over ranks of the total ms, clock samples).  With
    `per_step`, an event between replays also gives this rank's per-step
    p10 / p50 / p90 (ms) in STEP_STATS."""
    for _ in range(warmup):
        g.replay()
    torch.cuda.synchronize()
    dist.barrier()
    if clocks:
        clocks.start()
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1 if per_step else 2)]
    torch.cuda.synchronize()
    evs[0].record()
    for i in range(steps):
        g.replay()
        if per_step:
            evs[i + 1].record()
    evs[-1].record()
    torch.cuda.synchronize()
    ms = evs[0].elapsed_time(evs[-1])
    info = clocks.stop() if clocks else None
    if per_step:
        per = sorted(evs[i].elapsed_time(evs[i + 1]) for i in range(steps))
        pick = lambda q: round(per[min(steps - 1, int(q * steps))], 4)
        STEP_STATS.update({"p10": pick(0.1), "p50": pick(0.5), "p90": pick(0.9), "unit": "ms", "rank": dist.rank})
    dist.barrier()
    return dist.max(ms), info


def dominant_kernel_time(groups, lib, steps, warmup, dist):
    """Average launch duration of the dominant kernel (the Q4_0 GEMV) as the
    token runs it: the token's 128 Q4_0 launches alone (grouped q/k/v and
    gate/up), captured as one graph with programmatic dependent launch and
    replayed; CUDA events on the replay stream.  Returns (ms per launch,
    launches per replay, algorithmic bytes per launch)."""
    q4 = [grp for grp in groups if grp[0][5] == "q4_0"]

    def fn(stream):
        run_grouped(q4, stream, lib)

    g = capture(fn)
    ms, _ = time_graph(g, steps, warmup, dist)
    alg = sum(gemv_alg_bytes(n, k, q4_bytes(n, k)) for grp in q4 for _, n, k, _, _, _ in grp) / len(q4)
    return ms / (steps * len(q4)), len(q4), alg


def e2e_api(tok, ext, steps, warmup, dist):
    """Tokens/s through gds_io_ext with host buffers: H2D of the token's input
    and D2H of the logits inside the timed region, every step."""
    handles = [(ext.handle_from_tensor(buf), offs) for buf, offs in tok.layers]
    lm = ext.handle_from_tensor(tok.lm_head)
    x_host = tok.x0.cpu().pin_memory()
    logits_host = torch.empty(VOCAB, dtype=torch.float16).pin_memory()
    x_dev = torch.empty(HIDDEN, dtype=torch.float16, device=tok.device)

    def step():
        x_dev.copy_(x_host, non_blocking=True)
        x = x_dev.view(1, 1, -1)
        for h, offs in handles:
            acts = {"x": x}
            for name, n, k in PROJ:
                src = acts[SRC[name]]
                # llama.py:_fused_dequant_gemv: x.view(-1) -> [1, out] -> unsqueeze(0)
                acts[name] = ext.fused_dequant_gemv(h, src.view(-1), [n, k], "q4_0", offs[name][0]).unsqueeze(0)
            x = acts["down"]
        out = ext.fused_dequant_gemv(lm, x.view(-1), [VOCAB, HIDDEN], "q8_0", 0)
        logits_host.copy_(out.view(-1), non_blocking=True)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        step()
    end.record()
    torch.cuda.synchronize()
    return dist.max(start.elapsed_time(end))


# ---------------------------------------------------------------------------
# Config 1 as BASELINE states it: GdsLLM's own scheduler, unchanged

REF_PACKAGE = ROOT / "baseline" / "_ref"
DECODE_PREFILL, DECODE_WARMUP, DECODE_TOKENS = 512, 3, 128
_MODEL_DIR = None


def config1_model_dir(device) -> str:
    """A LLaMA-7B-shaped model directory (config 1: 32 layers, Q4_0 body,
    Q8_0 lm_head, fp16 embedding table, seeded weights) in the converter's
    layout, written once per process under the system temporary directory
    and removed at exit."""
    global _MODEL_DIR
    if _MODEL_DIR is None:
        import atexit
        import shutil
        import tempfile
        path = tempfile.mkdtemp(prefix="gdsllm_b200_config1_")
        atexit.register(shutil.rmtree, path, True)
        synth.write_llama_model_dir(path, layers=LAYERS, hidden=HIDDEN, heads=32, kv_heads=32, ffn=FFN, vocab=VOCAB,
                                    max_seq_len=1024, body="q4_0", lm_head="q8_0", embed="f16", seed=0, device=device)
        _MODEL_DIR = path
    return _MODEL_DIR


def e2e_decode(dist, module: str, scheduler_ops: bool = False, graph: bool = False):
    """Greedy decode through GdsLLM's own CachedScheduler (the reference
    package in baseline/_ref, unchanged): prompt of 509 tokens, 3 untimed
    decode steps (KV prefilled to 512 positions), then 128 timed tokens, each
    step a host token id in and the argmax token out (H2D + D2H per step), as
    the reference's engine drives it.  ``module`` picks the gds_io_ext the
    scheduler imports: "ours" (this build) or "reference" (GdsLLM's kernels
    compiled unchanged, oracle/ref_module.py -- the reference arm only).
    ``scheduler_ops`` also installs gdsllm_b200.scheduler_ops (embedding row
    gather, fused lm_head) into the scheduler module.  ``graph`` decodes the
    timed tokens with gdsllm_b200.decode_step.GraphDecodeStep built from the
    same scheduler and KV cache after the same prefill: one CUDA graph replay
    per token, the token id copied to pinned host memory inside the graph
    and read by the host every step."""
    if not (REF_PACKAGE / "gdsllm" / "runtime" / "scheduler.py").exists():
        return {"unavailable": "the reference package is not installed in baseline/_ref"}
    if str(REF_PACKAGE) not in sys.path:
        sys.path.insert(0, str(REF_PACKAGE))
    import gdsllm_b200
    from gdsllm.runtime import kv_cache, scheduler as sched_mod
    if module == "ours":
        gdsllm_b200.install_as_reference_module()
    else:
        from oracle import ref_module
        ref_module.install()
    saved = (sched_mod._embed_tokens, sched_mod._lm_head_proj)
    if scheduler_ops:
        from gdsllm_b200 import scheduler_ops as ops
        ops.install(sched_mod)
    path = config1_model_dir(dist.device)
    g = torch.Generator().manual_seed(1)
    prompt = torch.randint(0, VOCAB, (1, DECODE_PREFILL - DECODE_WARMUP), generator=g)
    tokens = []
    try:
        with torch.inference_mode(), sched_mod.CachedScheduler(path, device=str(dist.device)) as s:
            c = s.config
            kv = kv_cache.KVCache(c["num_layers"], c["num_kv_heads"], c["head_dim"], c["max_seq_len"],
                                  device=dist.device)
            logits = s.forward(prompt, kv_cache=kv, start_pos=0)
            tok = int(logits[0, -1].argmax())
            pos = prompt.shape[1]
            if graph:
                from gdsllm_b200.decode_step import GraphDecodeStep
                step = GraphDecodeStep.from_scheduler(s, kv)
                step.reset(tok, pos)
                step.capture()
                launches = step.launches_per_step()
                advance = step.step  # one replay; the host reads the token from pinned memory
            else:
                launches = None

                def advance():
                    nonlocal tok, pos
                    logits = s.forward(torch.tensor([[tok]]), kv_cache=kv, start_pos=pos)
                    tok = int(logits[0, -1].argmax())  # D2H of the step's result
                    pos += 1
                    return tok
            for _ in range(DECODE_WARMUP):
                advance()
            torch.cuda.synchronize()
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0 = time.perf_counter()
            start.record()
            for _ in range(DECODE_TOKENS):
                tokens.append(advance())
            end.record()
            torch.cuda.synchronize()
            wall = time.perf_counter() - t0
            ms = start.elapsed_time(end)
            if graph:
                del step, advance
    finally:
        sched_mod._embed_tokens, sched_mod._lm_head_proj = saved
    return {"value": round(DECODE_TOKENS / (ms / 1e3), 2), "unit": "tok/s", "ms_per_token": round(ms / DECODE_TOKENS, 4),
            "wall_s": round(wall, 3), "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 8,
            "tokens_head": tokens[:8],
            **({"gpu_launches_per_token": launches} if graph else {}),
            "what": ("GdsLLM's CachedScheduler + llama.transformer_block unchanged (baseline/_ref), config 1: 32 layers "
                     "Q4_0, Q8_0 lm_head, fp16 embedding, KV prefilled to 512, 128 greedy tokens; gds_io_ext = "
                     + ("this build" if module == "ours" else "GdsLLM's own kernels (oracle/ref_module.py)")
                     + ("; embedding and lm_head through gdsllm_b200.scheduler_ops" if scheduler_ops else "")
                     + ("; prefill by the scheduler, then every token one replay of "
                        "gdsllm_b200.decode_step.GraphDecodeStep (CUDA graph) on the same KV cache" if graph else ""))}


def _summary(res: dict, keys) -> dict:
    return {k: res[k] for k in keys if k in res}


def sub_benches(args, dist) -> dict:
    """The other configurations' headline numbers for the default line (every
    rank takes part, so at N > 1 the tensor- and expert-parallel exchanges
    run): config 0's GB/s, config 3 (tensor parallel over the N ranks) and
    config 4 (expert parallel over the N ranks, batch 1 and 8)."""
    import argparse as _ap
    out = {}

    def sub(**kw):
        a = _ap.Namespace(**vars(args))
        for k, v in kw.items():
            setattr(a, k, v)
        return a

    r = bench_config0(sub(steps=max(20, min(args.steps, 100)), warmup=3), dist)
    out["config0"] = _summary(r, ["metric", "value", "unit", "us_per_launch", "roofline", "clocks", "config"])
    torch.cuda.empty_cache()
    r = bench_config3(sub(steps=10, warmup=3), dist)
    out["config3_tp"] = _summary(r, ["metric", "value", "unit", "ms_per_step", "scaling", "roofline",
                                     "aggregate_weight_gbs", "clocks", "config"])
    torch.cuda.empty_cache()
    out["config4_ep"] = {}
    for b in (1, 8):
        r = bench_config4(sub(steps=10 if b == 1 else 5, warmup=3, batch=b, resident_layers=4), dist)
        out["config4_ep"][f"batch{b}"] = _summary(r, ["value", "unit", "ms_per_step", "roofline", "clocks", "config"])
        torch.cuda.empty_cache()
    return out


# ---------------------------------------------------------------------------
# CPU path of the reference (dequant formula + torch.matmul), bounded sample

def cpu_reference_path(budget_s: float = 0.0, max_items: int | None = None, frac: float = 1.0):
    """Times the reference's CPU path -- dequantize with the formula, then
    torch.matmul in fp32 -- on LLaMA-7B projections generated on the host,
    one projection per item, cycling over the 7 layer shapes, until
    ``max_items`` items (or ``budget_s`` seconds).  ``frac`` < 1 uses only the
    first rows of each projection.  Returns (tok/s, cores, sample, seconds),
    tok/s scaled by weight bytes to one token."""
    import oracle
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    items = []
    for pi, (name, n, k) in enumerate(PROJ):
        rows = max(1, int(math.ceil(n * frac)))
        items.append((synth.q4_0_weight(rows, k, seed=pi).numpy(), rows, k))
    x = synth.activations(1, FFN, seed=3).numpy()
    done_bytes, t_total, count = 0, 0.0, 0
    while True:
        for w, n, k in items:
            t0 = time.perf_counter()
            wd = oracle.dequant_q4_0(w).reshape(n, k)
            oracle.gemv_cpu(wd, x[:, :k])
            t_total += time.perf_counter() - t0
            done_bytes += q4_bytes(n, k)
            count += 1
            if (max_items and count >= max_items) or (not max_items and t_total >= budget_s
                                                      and count >= len(items)):
                tok_s = done_bytes / t_total / TOKEN_WBYTES
                sample = (f"{count} LLaMA-7B Q4_0 projections"
                          f"{'' if frac >= 1 else f' (first {frac:.3f} of rows)'} = "
                          f"{done_bytes / 1e6:.0f} MB of weights, dequantized by the formula "
                          f"(C, OpenMP) and multiplied with torch.matmul (fp32), scaled by bytes "
                          f"to one token ({TOKEN_WBYTES / 1e9:.3f} GB)")
                return tok_s, threads, sample, t_total


# ---------------------------------------------------------------------------

def bench_ours(args, dist):
    from gdsllm_b200 import capi, lib as gdsq_lib
    peak, peak_kind = load_peaks()
    lib = gdsq_lib()
    tok = Token(dist.device, seed=dist.rank)
    seq = tok.launches()
    groups = tok.grouped()

    capi.set_pdl(True)

    def fn(stream):
        tok.act["x"].copy_(tok.x0)
        run_grouped(groups, stream, lib)

    def fn_single(stream):
        tok.act["x"].copy_(tok.x0)
        run_ours(seq, stream, lib)

    g = capture(fn)
    clocks = dist.clocks
    ms, clock_info = time_graph(g, args.steps, args.warmup, dist, clocks, per_step=True)
    step_stats = dict(STEP_STATS)
    tok_s = args.steps * dist.world / (ms / 1e3)
    del g
    g1 = capture(fn_single)
    ms1, _ = time_graph(g1, args.steps, args.warmup, dist)
    del g1

    q4_ms, q4_launches, q4_alg = dominant_kernel_time(groups, lib, max(10, args.steps // 4), args.warmup, dist)
    achieved = q4_alg / (q4_ms / 1e3) / 1e9
    # DRAM traffic per launch: the ncu capture's traffic / algorithmic-bytes
    # ratio (one 11008x4096 launch; every launch streams each weight byte
    # once, so traffic scales with the bytes) applied to the mean launch
    traffic = None
    tf = ROOT / "profiles" / "gemv_q4_0_traffic.json"
    if tf.exists():
        try:
            t = json.loads(tf.read_text())
            traffic = round(t["dram_bytes_per_launch"] / t["algorithmic_bytes_per_launch"] * q4_alg)
        except Exception:
            traffic = None

    import gdsllm_b200
    e2e_ms = e2e_api(tok, gdsllm_b200.ext(), args.steps, max(3, args.warmup), dist)
    e2e = {"value": round(args.steps * dist.world / (e2e_ms / 1e3), 2), "unit": "tok/s",
           "h2d_bytes_per_step": HIDDEN * 2, "d2h_bytes_per_step": VOCAB * 2,
           "api": "gds_io_ext.fused_dequant_gemv x225 per token, as llama.py calls it"}

    cpu = None
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu:
        tps, cores, sample, secs = cpu_reference_path(args.cpu_budget)
        cpu = {"value": round(tps, 4), "unit": "tok/s", "cores": cores, "kind": "port",
               "sample": sample + f"; {secs:.1f} s of CPU time"}

    result = {
        "metric": "LLaMA-7B Q4_0 batch-1 decode tok/s through the fused dequant-GEMV path "
                  "(224 Q4_0 projections + Q8_0 lm_head per token)",
        "value": round(tok_s, 2), "unit": "tok/s", "n_gpus": dist.world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4), "step_ms": step_stats,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (seeded random Q4_0/Q8_0 weights per BASELINE config 0/1 distributions)",
        "config": {"workload": "config 1: LLaMA-7B-shaped decode token, hot path only, batch 1",
                   "layers": LAYERS, "hidden": HIDDEN, "ffn": FFN, "vocab": VOCAB,
                   "lm_head": "q8_0", "weight_bytes_per_token": TOKEN_WBYTES,
                   "l2": "inputs larger than L2 (3.78 GB of weights per step)",
                   "launch": "CUDA graph of 129 launches (q/k/v and gate/up share one launch each), "
                             "programmatic dependent launch",
                   "parallelism": f"replicas x{dist.world}"},
        "gbs": round(TOKEN_ALG_BYTES * tok_s / dist.world / 1e9, 1),
        "per_projection_launches": {"value": round(args.steps * dist.world / (ms1 / 1e3), 2), "unit": "tok/s",
                                    "launches_per_token": len(seq)},
        "roofline": {"bound": "hbm", "kernel": "gemv_fast_kernel<Q4_0, batch 1>",
                     "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                     "traffic": traffic, "us_per_launch": round(q4_ms * 1e3, 3),
                     "alg_bytes_per_launch": round(q4_alg),
                     "how": f"the token's {q4_launches} Q4_0 launches (grouped q/k/v 12288x4096, o 4096x4096, "
                            "grouped gate/up 22016x4096, down 4096x11008) as a CUDA graph, CUDA events, "
                            "mean algorithmic bytes / mean launch time"},
        "cpu_baseline": cpu,
        "e2e": e2e,
        "gpu_launches": len(groups) * args.steps,
        "clocks": clock_info,
    }
    del tok  # the token chain's weights are not needed any more: the scheduler legs start from a freed cache,
    torch.cuda.empty_cache()  # as the reference arm's do
    if not args.quick:
        if dist.world == 1:  # the scheduler loads onto one GPU
            result["e2e_decode"] = e2e_decode(dist, "ours")
            result["e2e_decode_scheduler_ops"] = e2e_decode(dist, "ours", scheduler_ops=True)
            result["e2e_decode_graph"] = e2e_decode(dist, "ours", graph=True)
        result.update(sub_benches(args, dist))
    return result


def bench_reference(args, dist):
    """The reference's path: CPU dequant formula + torch.matmul (value), and
    GdsLLM's own CUDA kernels on the same token (ref_cuda)."""
    result = {"impl": "reference", "metric": None}
    if dist.rank != 0:
        return None
    # Each step is one projection of the token (bounded sample); rows are
    # trimmed so that the K timed steps take about two minutes at most.
    _, _, _, warm_s = cpu_reference_path(max_items=max(7, args.warmup))
    per_step = warm_s / max(7, args.warmup)
    frac = min(1.0, 120.0 / (args.steps * per_step))
    tps, cores, sample, secs = cpu_reference_path(max_items=args.steps, frac=frac)
    result.update({
        "metric": "LLaMA-7B Q4_0 batch-1 decode tok/s through the fused dequant-GEMV path "
                  "(224 Q4_0 projections + Q8_0 lm_head per token)",
        "value": round(tps, 4), "unit": "tok/s", "n_gpus": dist.world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(secs / args.steps * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": "config 1: LLaMA-7B-shaped decode token, hot path only, batch 1",
                   "step": "one projection of the token (rotating over the 7 layer shapes)"},
        "cpu_baseline": {"value": round(tps, 4), "unit": "tok/s", "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(tps, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    })
    # GdsLLM's CUDA kernels (compiled unchanged) on the same token, on this B200.
    try:
        from oracle import reference_kernels as refk
        if refk.available():
            result["ref_cuda"] = bench_reference_cuda(args, dist, refk)
            if dist.world == 1 and not args.quick:
                # config 1 as BASELINE states it, on GdsLLM's own kernels (from a freed cache, as ours)
                torch.cuda.empty_cache()
                result["e2e_decode"] = e2e_decode(dist, "reference")
    except Exception as e:  # the CPU line above stands on its own
        result["ref_cuda"] = {"error": str(e)[:200]}
    return result


def bench_reference_cuda(args, dist, refk):
    tok = Token(dist.device, seed=0)
    seq = tok.launches()
    l = refk.lib()
    lm_fp16 = torch.empty(VOCAB, HIDDEN, dtype=torch.float16, device=dist.device)

    def fn(stream):
        tok.act["x"].copy_(tok.x0)
        for w, n, k, x, y, fmt in seq:
            if fmt == "q4_0":
                l.ref_fused_q4_0_gemv(w, x, y, n, k, stream)
            else:
                # the reference scheduler's lm_head: full dequant + F.linear
                # (gdsllm/runtime/scheduler.py:54-55,69); torch runs on the
                # same (current) stream as the ctypes launches.
                l.ref_dequant_q8_0(w, lm_fp16.data_ptr(), VOCAB * HIDDEN // 32, stream)
                torch.matmul(tok.layer_out[-1].view(1, -1), lm_fp16.t(), out=tok.logits.view(1, -1))

    g = capture(fn)
    ms, _ = time_graph(g, args.steps, args.warmup, dist)
    tps = args.steps / (ms / 1e3)
    return {"value": round(tps, 2), "unit": "tok/s", "ms_per_step": round(ms / args.steps, 4),
            "gbs": round(TOKEN_ALG_BYTES * tps / 1e9, 1),
            "what": "GdsLLM's fused_gemv.cu / gguf_dequant.cu compiled unchanged for sm_100a, same "
                    "token chain in a CUDA graph; lm_head as the reference scheduler does it "
                    "(dequant_q8_0 to fp16 + cuBLAS)"}


# ---------------------------------------------------------------------------

def bench_config0(args, dist):
    """One 11008x4096 Q4_0 GEMV, rotating over copies that together exceed L2."""
    from gdsllm_b200 import capi, lib as gdsq_lib
    peak, peak_kind = load_peaks()
    lib = gdsq_lib()
    n, k = 11008, 4096
    copies = 8
    ws = [synth.q4_0_weight(n, k, seed=i, device=dist.device) for i in range(copies)]
    x = synth.activations(1, k, seed=9, device=dist.device)
    y = torch.empty(1, n, dtype=torch.float16, device=dist.device)
    capi.set_pdl(args.pdl)

    def fn(stream):
        for w in ws:
            st = lib.gdsq_fused_q4_0_gemv(w.data_ptr(), x.data_ptr(), y.data_ptr(), n, k, 1, stream)
            if st:
                raise RuntimeError(lib.gdsq_last_error().decode())

    g = capture(fn)
    ms, clk = time_graph(g, args.steps, args.warmup, dist, dist.clocks)
    launches = args.steps * copies
    us = ms * 1e3 / launches
    b = gemv_alg_bytes(n, k, q4_bytes(n, k))
    gbs = b / (us / 1e6) / 1e9
    return {"metric": "Q4_0 fused dequant-GEMV 11008x4096 batch 1, HBM GB/s", "value": round(gbs, 1),
            "unit": "GB/s", "n_gpus": dist.world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": "config 0", "copies": copies, "pdl": bool(args.pdl),
                       "l2": f"rotating over {copies} weight copies ({copies * q4_bytes(n, k) / 1e6:.0f} MB > L2)"},
            "us_per_launch": round(us, 3),
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(gbs / peak, 4), "peak_kind": peak_kind},
            "gpu_launches": launches, "clocks": clk}


def bench_config2(args, dist):
    """Q8_0 and affine-Q4 GEMV sweep: 4 shapes x batch 1/4/8/16 (BASELINE
    config 2).  Each point is a CUDA graph of launches rotating over weight
    copies that together exceed L2; value = aggregate GB/s over the sweep."""
    from gdsllm_b200 import capi, lib as gdsq_lib
    peak, peak_kind = load_peaks()
    lib = gdsq_lib()
    capi.set_pdl(bool(args.pdl))
    shapes = [(4096, 4096), (11008, 4096), (4096, 11008), (32000, 4096)]
    points = []
    tot_bytes = 0.0
    tot_ms = 0.0
    launches = 0
    for fmt in ("q8_0", "affine_q4"):
        for n, k in shapes:
            if fmt == "q8_0":
                wbytes = q8_bytes(n, k)
            else:
                wbytes = n * k // 2 + 2 * 2 * n * (k // 128)
            copies = max(2, int(300e6 // wbytes) + 1)
            if fmt == "q8_0":
                ws = [(synth.q8_0_weight(n, k, seed=i, device=dist.device),) for i in range(copies)]
            else:
                ws = [synth.affine_q4_weight(n, k, seed=i, device=dist.device) for i in range(copies)]
            for b in (1, 4, 8, 16):
                x = synth.activations(b, k, seed=5, device=dist.device)
                y = torch.empty(b, n, dtype=torch.float16, device=dist.device)

                def fn(stream, ws=ws, x=x, y=y, n=n, k=k, b=b, fmt=fmt):
                    for w in ws:
                        if fmt == "q8_0":
                            st = lib.gdsq_fused_q8_0_gemv(w[0].data_ptr(), x.data_ptr(), y.data_ptr(), n, k, b,
                                                          stream)
                        else:
                            st = lib.gdsq_fused_affine_q4_gemv(w[0].data_ptr(), w[1].data_ptr(), w[2].data_ptr(),
                                                               x.data_ptr(), y.data_ptr(), n, k, 128, b, stream)
                        if st:
                            raise RuntimeError(lib.gdsq_last_error().decode())

                g = capture(fn)
                reps = max(3, args.steps // copies)
                ms, _ = time_graph(g, reps, args.warmup, dist)
                us = ms * 1e3 / (reps * copies)
                alg = wbytes + 2 * b * (k + n)
                gbs = alg / (us / 1e6) / 1e9
                points.append({"fmt": fmt, "n": n, "k": k, "batch": b, "us": round(us, 3),
                               "gbs": round(gbs, 1), "frac": round(gbs / peak, 4)})
                tot_bytes += alg * reps * copies
                tot_ms += ms
                launches += reps * copies
                del g
            del ws
            torch.cuda.empty_cache()
    agg = tot_bytes / (tot_ms / 1e3) / 1e9
    return {"metric": "Q8_0 / affine-Q4 fused dequant-GEMV sweep, aggregate HBM GB/s", "value": round(agg, 1),
            "unit": "GB/s", "n_gpus": dist.world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(tot_ms / max(1, launches), 5), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": "config 2: 4 shapes x batch 1/4/8/16, Q8_0 and affine-Q4 g=128",
                       "l2": "rotating over weight copies > 300 MB per point"},
            "roofline": {"bound": "hbm", "achieved": round(agg, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(agg / peak, 4), "peak_kind": peak_kind},
            "sweep": points, "gpu_launches": launches}


def bench_config3(args, dist):
    """LLaMA-70B-shaped Q4_0 decode GEMV chain, tensor-parallel over the ranks
    per layer q, k, v, gate, up column-split, o and down
    row-split with one NCCL all-reduce each; Q8_0 lm_head column-split with an
    all-gather of the logits.  Every rank holds only its shards (38.5 GB / N).
    One step = one token through all 80 layers; captured as one CUDA graph."""
    from gdsllm_b200 import capi, lib as gdsq_lib
    import torch.distributed as tdist
    peak, peak_kind = load_peaks()
    lib = gdsq_lib()
    capi.set_pdl(bool(args.pdl))
    H, Q, KV, FF, V, NL = 8192, 8192, 1024, 28672, 32000, 80
    ws, rank, dev = dist.world, dist.rank, dist.device
    cols = {"q": (Q // ws, H), "k": (KV // ws, H), "v": (KV // ws, H), "gate": (FF // ws, H), "up": (FF // ws, H)}
    rows = {"o": (H, Q // ws), "down": (H, FF // ws)}
    layers = []
    for layer in range(NL):
        wl = {}
        for j, (name, (n, k)) in enumerate(list(cols.items()) + list(rows.items())):
            wl[name] = synth.q4_0_weight(n, k, seed=(layer * 16 + j) * 64 + rank, device=dev)
        layers.append(wl)
    lm = synth.q8_0_weight(V // ws, H, seed=999 * 64 + rank, device=dev)
    x0 = synth.activations(1, H, seed=5, device=dev)
    buf = {name: torch.empty(1, n, dtype=torch.float16, device=dev) for name, (n, _) in cols.items()}
    o_out = torch.empty(1, H, dtype=torch.float16, device=dev)
    d_out = torch.empty(1, H, dtype=torch.float16, device=dev)
    logits_local = torch.empty(1, V // ws, dtype=torch.float16, device=dev)
    logits = torch.empty(ws, V // ws, dtype=torch.float16, device=dev)
    wbytes_rank = sum(t.numel() for wl in layers for t in wl.values()) + lm.numel()

    def gemv(fmt, w, x, y, n, k, stream):
        fn = lib.gdsq_fused_q4_0_gemv if fmt == "q4_0" else lib.gdsq_fused_q8_0_gemv
        st = fn(w.data_ptr(), x.data_ptr(), y.data_ptr(), n, k, 1, stream)
        if st:
            raise RuntimeError(lib.gdsq_last_error().decode())

    def token(stream):
        x = x0
        for wl in layers:
            for name, (n, k) in cols.items():
                if name in ("q", "k", "v"):
                    gemv("q4_0", wl[name], x, buf[name], n, k, stream)
            if fused is not None:   # attention output stands in as q's shard
                fused_row(wl["o"], buf["q"], o_out, H, Q // ws, stream)
            else:
                gemv("q4_0", wl["o"], buf["q"], o_out, H, Q // ws, stream)
                if ws > 1:
                    allreduce(o_out)
            gemv("q4_0", wl["gate"], o_out, buf["gate"], FF // ws, H, stream)
            gemv("q4_0", wl["up"], o_out, buf["up"], FF // ws, H, stream)
            if fused is not None:
                fused_row(wl["down"], buf["up"], d_out, H, FF // ws, stream)
            else:
                gemv("q4_0", wl["down"], buf["up"], d_out, H, FF // ws, stream)
                if ws > 1:
                    allreduce(d_out)
            x = d_out
        gemv("q8_0", lm, x, logits_local, V // ws, H, stream)
        if ws > 1:
            tdist.all_gather_into_tensor(logits, logits_local)

    if ws > 1:  # NCCL communicators exist before capture
        tdist.all_reduce(o_out)
        tdist.all_gather_into_tensor(logits, logits_local)
        torch.cuda.synchronize()
    peer = None
    fused = None
    if ws > 1 and args.tp_allreduce == "p2p":
        from gdsllm_b200.p2p import PeerAllReduce
        peer = PeerAllReduce(H, device=dev)
    if ws > 1 and args.tp_allreduce == "fused":
        from gdsllm_b200.p2p import PeerRowGemv
        fused = PeerRowGemv(H, device=dev)

    def fused_row(w, x, y, n, k, stream):
        st = lib.gdsq_fused_gemv_allreduce(0, w.data_ptr(), x.data_ptr(), y.data_ptr(), n, k, fused.peer.bufs,
                                           fused.peer.flags, fused.rows, fused.rank, fused.world, stream)
        if st:
            raise RuntimeError(lib.gdsq_last_error().decode())

    def allreduce(t):
        if peer is not None:
            peer(t)
        else:
            tdist.all_reduce(t)
    g = capture(token)
    ms, clk = time_graph(g, args.steps, args.warmup, dist, dist.clocks)
    del g
    if peer is not None:
        peer.close()
    if fused is not None:
        fused.close()
    tok_s = args.steps / (ms / 1e3)
    per_token_bytes = wbytes_rank * ws
    launches = args.steps * (NL * 7 + 1)
    return {"metric": "LLaMA-70B-shaped Q4_0 batch-1 decode tok/s, tensor-parallel GEMV chain (560 Q4_0 "
                      "projections + Q8_0 lm_head per token, all-reduce after o and down)",
            "value": round(tok_s, 2), "unit": "tok/s", "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic (seeded random Q4_0/Q8_0 shards, config 3 shapes)",
            "config": {"workload": "config 3: 80 layers, hidden 8192, q 8192 / kv 1024 rows, FFN 28672, vocab 32000 "
                                   "(Q8_0 lm_head), batch 1; attention and norms are not on the path",
                       "parallelism": f"tp{ws}", "weights_per_gpu_gb": round(wbytes_rank / 1e9, 2),
                       "allreduce": ("inside the row-split GEMV's epilogue over NVLink peer memory "
                                     "(gdsq_fused_gemv_allreduce)" if fused is not None else
                                     "one-shot over NVLink peer memory (gdsq_allreduce_sum_f16)"
                                     if peer is not None else "NCCL") if ws > 1 else None,
                       "l2": "every token streams 38.5 GB / N per GPU (> L2)"},
            "roofline": {"bound": "hbm", "achieved": round(wbytes_rank / (ms / args.steps / 1e3) / 1e9, 1),
                         "peak": peak, "unit": "GB/s",
                         "frac": round(wbytes_rank / (ms / args.steps / 1e3) / 1e9 / peak, 4),
                         "peak_kind": peak_kind, "scope": "per-GPU weight bytes / token time (whole step)"},
            "aggregate_weight_gbs": round(per_token_bytes * tok_s / 1e9, 1),
            "gpu_launches": launches, "clocks": clk}


def bench_config4(args, dist):
    """Qwen-MoE-shaped affine-Q4 MoE decode, expert-parallel over the ranks
    60 MoE layers (8 distinct resident layers cycled),
    512 experts + 1 shared (hidden 4096, intermediate 1024), fp16 router with
    top-10; experts split 512 / N per GPU, one all-reduce of the fp32
    partial sums per layer (over NVLink peer memory, or NCCL).  One step = one decode step of `--batch` tokens."""
    from gdsllm_b200 import capi, ep, moe
    peak, peak_kind = load_peaks()
    capi.set_pdl(bool(args.pdl))
    E, H, I, G, TOPK, NL = args.experts, 4096, 1024, 128, 10, 60
    NPHYS = args.resident_layers
    ws, rank, dev = dist.world, dist.rank, dist.device
    B = args.batch
    first, count = ep.expert_range(rank, ws, E)
    gen = torch.Generator().manual_seed(1)
    layers = []
    for l in range(NPHYS):
        def st(rows, cols, seed, e):
            return synth.affine_q4_weight(rows, cols, group=G, seed=seed, device=dev, lead=(e,))
        base = (l * 8) * 64
        router = (torch.randn(E, H, generator=gen) / H ** 0.5).half().to(dev)
        sgate = (torch.randn(1, H, generator=gen) / H ** 0.5).half().to(dev)
        layers.append(moe.MoeLayer(
            router=router, gate=st(I, H, base + 1 + rank * 8, count), up=st(I, H, base + 2 + rank * 8, count),
            down=st(H, I, base + 3 + rank * 8, count), group=G, expert_first=first, expert_total=E,
            shared=(st(I, H, base + 4, 1), st(I, H, base + 5, 1), st(H, I, base + 6, 1)), shared_gate=sgate))
    exch = None
    if ws > 1 and args.ep_allreduce == "peer":
        from gdsllm_b200.p2p import PeerWordAllReduce
        exch = PeerWordAllReduce(B * H, device=dev)
    mods = [ep.ExpertParallelMoE(layer, top_k=TOPK, allreduce=exch) for layer in layers] if ws > 1 else None
    x0 = synth.activations(B, H, seed=3, device=dev)

    def step(stream):
        x = x0
        for l in range(NL):  # x + moe(x), the residual add inside the layer's last launch
            layer = layers[l % NPHYS]
            x = (mods[l % NPHYS](x, add_residual=True) if ws > 1
                 else moe.moe_mlp_decode(x, layer, TOPK, add_residual=True))
        return x

    # bytes touched per step (whole job): routing of an eager pass
    touched = 0
    x = x0
    with torch.no_grad():
        for l in range(NL):
            layer = layers[l % NPHYS]
            ids = moe.route_fused(x, layer, TOPK)[0]
            distinct = int(torch.unique(ids).numel())
            touched += E * H * 2 + (distinct + 1) * 3 * (I * H // 2 + 2 * 2 * I * H // G)
            x = (mods[l % NPHYS](x, add_residual=True) if ws > 1
                 else moe.moe_mlp_decode(x, layer, TOPK, add_residual=True))
    torch.cuda.synchronize()
    g = capture(step)
    ms, clk = time_graph(g, args.steps, args.warmup, dist, dist.clocks)
    del g
    if exch is not None:
        exch.close()
    step_s = ms / args.steps / 1e3
    return {"metric": "Qwen-MoE-shaped affine-Q4 MoE decode tok/s, expert-parallel (60 layers x (router top-10 + "
                      "fused expert gather + shared expert), all-reduce of the partials per layer)",
            "value": round(B / step_s, 2), "unit": "tok/s", "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic (seeded random affine-Q4 experts, config 4 shapes)",
            "config": {"workload": f"config 4: {E} experts + shared, hidden 4096, expert intermediate 1024, top-10, "
                                   f"batch {B}, 60 layers cycling {NPHYS} resident layers",
                       "parallelism": f"ep{ws}", "experts_per_gpu": count,
                       "allreduce": ("one-shot (value, epoch) words over NVLink peer memory (gdsq_allreduce_sum_words)"
                                     if exch is not None else "NCCL") if ws > 1 else None,
                       "touched_weight_gb_per_step": round(touched / 1e9, 3),
                       "l2": f"{NPHYS} resident layers of {E * 3 * 2.23 / 1e3:.1f} GB each (> L2)"},
            "roofline": {"bound": "hbm", "achieved": round(touched / ws / step_s / 1e9, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(touched / ws / step_s / 1e9 / peak, 4), "peak_kind": peak_kind,
                         "scope": "touched weight bytes per GPU / step time (whole step)"},
            # this build's kernels per layer: router + route, gate/up, down (+ the word exchange over ranks)
            "gpu_launches": args.steps * NL * (3 + (1 if exch is not None else 0)), "clocks": clk}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", type=int, default=1, choices=[0, 1, 2, 3, 4])
    ap.add_argument("--batch", type=int, default=1, help="config 4: tokens per decode step (1 or 8)")
    ap.add_argument("--tp-allreduce", choices=["fused", "p2p", "nccl"], default="fused",
                    help="config 3: the o/down all-reduce: inside the row-split GEMV over peer memory (default), "
                         "a separate one-shot peer-memory kernel, or NCCL")
    ap.add_argument("--ep-allreduce", choices=["peer", "nccl"], default="peer",
                    help="config 4: the per-layer sum of the partials over peer memory (default) or NCCL")
    ap.add_argument("--resident-layers", type=int, default=8,
                    help="config 4: distinct MoE layers held on the GPU and cycled over the 60 (3.4 GB each; "
                         "8 by default, fewer only for profiler captures)")
    ap.add_argument("--experts", type=int, default=512,
                    help="config 4: experts per layer (512; fewer only for profiler captures -- the per-token "
                         "work, 10 routed + 1 shared expert per layer, is the same)")
    ap.add_argument("--pdl", type=int, default=1)
    ap.add_argument("--cpu-budget", type=float, default=12.0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--decode", choices=["scheduler", "scheduler_ops", "graph"], default=None,
                    help="only the end-to-end config 1 decode (e2e_decode*): through the reference scheduler, "
                         "with scheduler_ops, or with the graph-captured decode step")
    ap.add_argument("--quick", action="store_true",
                    help="default line only: skip the scheduler decode and the config 0 / 3 / 4 sub-benchmarks")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    dist = Dist(sample_clocks=args.impl != "reference")
    try:
        if args.decode is not None:
            res = e2e_decode(dist, "ours" if args.impl == "ours" else "reference",
                             scheduler_ops=args.decode == "scheduler_ops", graph=args.decode == "graph")
        elif args.impl == "reference":
            res = bench_reference(args, dist)
        elif args.config == 0:
            res = bench_config0(args, dist)
        elif args.config == 2:
            res = bench_config2(args, dist)
        elif args.config == 3:
            res = bench_config3(args, dist)
        elif args.config == 4:
            res = bench_config4(args, dist)
        else:
            res = bench_ours(args, dist)
        if dist.rank == 0 and res is not None:
            print(json.dumps(res), flush=True)
    finally:
        dist.close()


if __name__ == "__main__":
    main()
