#!/usr/bin/env python3
"""Decode benchmark for the B200 text-decode path (one JSON line on rank 0).

Workload (config 0 of the reference's decode benchmark): the 24-layer, 1024-hidden
HunyuanOCR text decoder, vocab 120818 tied, fp32 weights and KV cache, random-init
~N(0, 0.02) weights (seeded counter generator), a 1024-position prompt (768
N(0,1) image-embedding rows on a 24x32 mRoPE grid + 256 uniform text ids), then
256 greedy tokens with repetition penalty 1.08.

One step = the AR decode of those 256 tokens from the prefilled state (255
decoder steps run by the persistent decode kernel, 64 tokens per launch: embed
-> 24 layers -> LM head -> penalised argmax -> commit, token kept on the
device). `value` = decode tokens/s with the prompt state resident in HBM;
`e2e` = tokens/s of the reference-facing call (hy_run_vlm_decode_with_prompt:
host prompt -> prefill -> 256 tokens -> host). `dflash` = config 3 (KV 2048,
block 16, synthetic drafts at p = 0.3 / 0.7 / 0.9), device-timed, plus the cost of
a block with the draft network (`draft_net`, random-init draft weights).

Multi-GPU (torchrun, one process per GPU): replicas only - each rank decodes its
own request; value = tokens of all ranks / max rank time ("scaling": "weak").

--impl reference: times the CPU oracle (the reference's CPU fp32 decode path
restated in numpy, oracle/hy_oracle.py) on the host cores for the same metric.
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

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
PROMPT_GRID = (24, 32)
PROMPT_TEXT = 256
GEN_TOKENS = 256
HIDDEN = 1024
V = 120818
LAYERS = 24
FFN = 3584
PENALTY = 1.08
# Algorithmic bytes (fp32): weights read once per token, 8 unique KV heads.
DECODER_WEIGHT_BYTES = LAYERS * (4096 * 1024 + 1024 * 2048 + 2 * FFN * 1024 + 1024 * FFN) * 4
LM_HEAD_BYTES = V * HIDDEN * 4
KV_ROW_BYTES = LAYERS * 8 * 128 * 4 * 2
MEGA_CHUNK = 64                      # tokens per persistent-kernel launch (hy_capi.cu kMegaChunk)
# DRAM bytes (read + write) per algorithmic byte of the persistent kernel, from one ncu
# capture of dram__bytes_read.sum + dram__bytes_write.sum on a small case of the same
# kernel (4 layers, vocab 16384, 8 tokens at KV 1024: 3.0287 GB for 3.0211 GB algorithmic;
# a profiler number, it cannot be taken live). The traffic of a full launch is this ratio
# times its algorithmic bytes: every weight and KV byte is read once per token, so the
# traffic grows with the tokens and layers a launch processes.
MEGA_TRAFFIC_RATIO = 1.0025
# Draft depth of the DFlash draft network leg. The reference loads the draft from its
# DFlash package (export/dflash_export.py takes any depth); 5 layers is an assumption.
DRAFT_LAYERS = 5


def measured_peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def ar_bytes_per_token(seq: int, gen: int) -> float:
    """Mean algorithmic bytes per decode token over steps with KV length seq..seq+gen-2."""
    mean_past = seq + (gen - 2) / 2.0
    return DECODER_WEIGHT_BYTES + LM_HEAD_BYTES + (mean_past + 1) * KV_ROW_BYTES + HIDDEN * 4


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def _gpu_id(self) -> str:
        """nvidia-smi numbers GPUs in PCI order and ignores CUDA_VISIBLE_DEVICES: name the
        CUDA device by its UUID so the samples come from the GPU this process runs on."""
        try:
            import torch
            return "GPU-" + str(torch.cuda.get_device_properties(self.index).uuid)
        except Exception:
            return str(self.index)

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", self._gpu_id(), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def dist_max(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def dist_barrier(world: int):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def prompt_arrays(seed: int):
    """Same prompt layout as oracle.synthetic_prompt (counter generator), built without the oracle."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("hy_b200_prompt", os.path.join(REPO, "hunyuanocr-ncnn_b200",
                                                                                   "synthetic.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.synthetic_prompt(seed, PROMPT_GRID[0], PROMPT_GRID[1], PROMPT_TEXT, V)


def pinned_copy(a: np.ndarray) -> np.ndarray:
    """A copy of `a` in page-locked host memory (the e2e inputs the contract asks for)."""
    import torch
    t = torch.empty(a.shape, dtype=getattr(torch, str(a.dtype)), pin_memory=True)
    out = t.numpy()   # its base is a tensor on the same pinned storage, which stays alive with it
    out[...] = a
    return out


def device_ms(rt, fn):
    """Run fn() and return the CUDA-event time (ms) of the work it enqueues on the context's stream."""
    import torch
    ext = torch.cuda.ExternalStream(rt.stream)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(ext)
    out = fn()
    e1.record(ext)
    e1.synchronize()
    return e0.elapsed_time(e1), out


def bf16_leg(pkg, local, seq: int, n_tok: int = GEN_TOKENS):
    """The bf16 variant at config 0 (bf16 weights and KV cache, fp32 activations and
    accumulation): device-timed AR decode of n_tok - 1 tokens from KV length seq, and its
    roofline (bf16 weights + bf16 KV rows per token)."""
    rt = pkg.TextRuntime.synthetic(seed=0, device=local, max_prefill=64, max_tokens=n_tok + 64,
                                   max_context=seq + n_tok + 64, weight_dtype=pkg.DTYPE_BF16,
                                   kv_dtype=pkg.DTYPE_BF16)
    best = None
    for _ in range(3):
        rt.set_length(seq)
        rt.set_history(list(range(1, 257)))
        ms, _ = device_ms(rt, lambda: rt.bench_ar_steps(n_tok - 1))
        best = ms if best is None else min(best, ms)
    rt.close()
    mean_past = seq + (n_tok - 2) / 2.0
    bpt = (DECODER_WEIGHT_BYTES + LM_HEAD_BYTES) / 2 + (mean_past + 1) * KV_ROW_BYTES / 2 + HIDDEN * 4
    peak, _ = measured_peaks()
    tps = (n_tok - 1) / (best / 1e3)
    return {"tokens_per_s": round(tps, 1), "bytes_per_token": round(bpt),
            "roofline_frac": round(tps * bpt / 1e9 / peak, 4), "roofline_tokens_per_s": round(peak * 1e9 / bpt, 1)}


def dflash_leg(pkg, local):
    """DFlash (config 3): KV length 2048, block 16, synthetic drafts equal to the greedy token
    with probability p, repeated for 256 committed tokens; tokens/s per p, device-timed."""
    seq, n_tok = 2048, 257
    rt = pkg.TextRuntime.synthetic(seed=0, device=local, max_prefill=64, max_tokens=n_tok + 64,
                                   max_context=seq + n_tok + 64)
    hist = list(range(1, 257))
    rt.set_length(seq)
    rt.set_history(hist)
    greedy, _ = rt.generate(1234, 1234, n_tok + 16, PENALTY)
    out = {}
    for p in (0.3, 0.7, 0.9):
        best = None
        for _ in range(2):
            rt.set_length(seq)
            rt.set_history(hist)
            ms, r = device_ms(rt, lambda: rt.dflash_generate_synthetic(1234, n_tok, PENALTY, greedy, p, seed=7))
            assert r.generated_tokens == greedy[:len(r.generated_tokens)], "DFlash is not lossless"
            best = ms if best is None else min(best, ms)
        out[f"p{p}"] = {"tokens_per_s": round((len(r.generated_tokens) - 1) / (best / 1e3), 1),
                        "blocks": r.block_count,
                        "mean_accept": round(float(np.mean(r.acceptance_lengths)), 3),
                        "ms_per_block": round(best / max(1, r.block_count), 3)}
    rt.set_length(seq)
    rt.set_history(hist)
    ms, _ = device_ms(rt, lambda: rt.bench_ar_steps(n_tok - 1))
    out["ar_tokens_per_s_kv2048"] = round((n_tok - 1) / (ms / 1e3), 1)

    # The draft network (hy_dflash_generate): a random-init draft of DRAFT_LAYERS layers over a
    # 2048-row draft context. Its drafts are essentially never accepted, so this measures the
    # cost of a block with the draft (draft + verify + context rows + commit), not an acceptance law.
    rt.reset()
    rt.load_draft_synthetic(DRAFT_LAYERS, seed=3, std=0.02)
    aux = np.random.default_rng(0).standard_normal((4, seq, HIDDEN), dtype=np.float32)
    rt.draft_context_append(aux)
    n_draft = 64
    rt.set_length(seq)
    rt.set_history(hist)
    rt.draft_propose(1234)
    d_ms, _ = device_ms(rt, lambda: [rt.draft_propose(1234) for _ in range(10)])
    best = None
    for _ in range(2):
        rt.set_length(seq)
        rt.set_history(hist)
        ms, r = device_ms(rt, lambda: rt.dflash_generate(1234, n_draft, PENALTY))
        assert r.generated_tokens == greedy[:len(r.generated_tokens)], "DFlash with the draft is not lossless"
        best = ms if best is None else min(best, ms)
    out["draft_net"] = {"layers": DRAFT_LAYERS, "draft_ms": round(d_ms / 10, 3),
                        "ms_per_block": round(best / max(1, r.block_count), 3),
                        "tokens_per_s": round(len(r.generated_tokens) / (best / 1e3), 1),
                        "blocks": r.block_count, "mean_accept": round(float(np.mean(r.acceptance_lengths)), 3)}
    rt.close()
    return out


def dist_sum(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def requests_leg(pkg, world, rank, local, n_req: int = 64, n_tok: int = 512):
    """Config 4 on the whole box: n_req records (prompt 1024 = 768 image rows + 256 text ids,
    seeded by record index) x n_tok tokens, split round-robin over the ranks (record i on rank
    i mod world, one GPU each, no collective on the data path). Three modes, each timed on
    every rank from a barrier, whole-box figures = all ranks' tokens (requests) / the slowest
    rank's time: `batched` = the rank's records decoded together by hy_batch_decode (16 slots);
    `one_at_a_time` = each record through hy_run_vlm_decode_with_prompt (the reference's
    sequential run_jsonl_batch, src/batch_jsonl.cpp:384-480); `dflash_p0.7` = each record's
    prefill and first token through the same call, then the on-device DFlash loop with drafts
    equal to the record's one-at-a-time greedy token with probability 0.7."""
    import torch
    seq = PROMPT_GRID[0] * PROMPT_GRID[1] + PROMPT_TEXT
    rt = pkg.TextRuntime.synthetic(seed=0, device=local, max_prefill=seq, max_tokens=n_tok + 64,
                                   max_context=seq + n_tok + 64)
    mine = list(range(rank, n_req, world))
    reqs = {}
    for i in mine:
        ids, pos, feats, img = prompt_arrays(seed=i)
        reqs[i] = (ids, pos, img, feats)
    if mine:   # warm-up: slot buffers, step graphs, first touch
        rt.batch_decode([reqs[mine[0]]], 8)
        ids, pos, img, feats = reqs[mine[0]]
        first = rt.run_vlm_decode_with_prompt(ids, pos, img, feats, max_tokens=8).generated_tokens
        rt.dflash_generate_synthetic(first[0], 8, PENALTY, first, 0.7, seed=0)

    def timed(fn):
        dist_barrier(world)
        torch.cuda.synchronize(local)
        t0 = time.perf_counter()
        out = fn()
        torch.cuda.synchronize(local)
        dt = time.perf_counter() - t0
        return out, dist_max(dt, world)

    out = {"records": n_req, "tokens_per_record": n_tok, "prompt": seq, "gpus": world,
           "partition": "round-robin (record i on rank i mod N)", "timing": "wall clock from a barrier, max over ranks"}
    # Batched.
    (toks, status), dt = timed(lambda: rt.batch_decode([reqs[i] for i in mine], n_tok) if mine else ([], []))
    assert all(st == 0 for st in status), status
    greedy = dict(zip(mine, toks))
    n_all = dist_sum(float(sum(len(t) for t in toks)), world)
    out["batched"] = {"tokens_per_s": round(n_all / dt, 1), "requests_per_s": round(n_req / dt, 3),
                      "seconds": round(dt, 3)}

    # One at a time (AR, bs = 1).
    def one_by_one():
        return {i: rt.run_vlm_decode_with_prompt(*reqs[i], max_tokens=n_tok).generated_tokens for i in mine}
    single, dt = timed(one_by_one)
    # The two modes reduce in different fp32 orders (16-row tensor-core projections
    # against the persistent GEMV), so a near-tie argmax can go either way; report
    # how many records agree rather than require all of them to (the parity tests
    # hold each mode to the oracle).
    same = dist_sum(float(sum(single[i] == greedy[i] for i in mine)), world)
    out["one_at_a_time"] = {"tokens_per_s": round(n_all / dt, 1), "requests_per_s": round(n_req / dt, 3),
                            "seconds": round(dt, 3), "records_equal_to_batched": int(same)}

    # DFlash, p = 0.7, one record at a time.
    def dflash_by_one():
        res = {}
        for i in mine:
            first = rt.run_vlm_decode_with_prompt(*reqs[i], max_tokens=1).generated_tokens[0]
            res[i] = rt.dflash_generate_synthetic(first, n_tok, PENALTY, single[i], 0.7, seed=i)
        return res
    dres, dt = timed(dflash_by_one)
    same_d = dist_sum(float(sum(dres[i].generated_tokens == single[i] for i in mine)), world)
    acc = [a for i in mine for a in dres[i].acceptance_lengths]
    out["dflash_p0.7"] = {"tokens_per_s": round(n_all / dt, 1), "requests_per_s": round(n_req / dt, 3),
                          "seconds": round(dt, 3), "mean_accept_rank0": round(float(np.mean(acc)), 3) if acc else None,
                          "records_equal_to_one_at_a_time": int(same_d)}
    rt.close()
    return out


def workload_config(seq: int, gen: int, world: int) -> dict:
    return {"workload": "config0: 24-layer decoder, prompt 1024 (768 image rows on 24x32 mRoPE + 256 text), "
                        "256 greedy tokens, penalty 1.08, fp32 weights+KV",
            "prompt": seq, "generated": gen, "parallelism": f"replicas x{world}",
            "l2": "weights 2.16 GB per token > 126 MB L2 (no flush needed)"}


def run_b200(args, world, rank, local):
    sys.path.insert(0, REPO)
    import __graft_entry__ as ge
    pkg = ge.load_package()
    pkg.load_library()
    ids, pos, feats, image_token = prompt_arrays(seed=rank)
    seq = ids.shape[0]
    rt = pkg.TextRuntime.synthetic(seed=0, device=local, max_prefill=seq, max_tokens=GEN_TOKENS + 64,
                                   max_context=seq + GEN_TOKENS + 64)
    # Prefill + first token through the reference-facing call (also the e2e warm-up).
    res = rt.run_vlm_decode_with_prompt(ids, pos, image_token, feats, max_tokens=GEN_TOKENS)
    first, first_raw = res.generated_tokens[0], res.raw_top1_tokens[0]
    n_tok = len(res.generated_tokens)

    def one_step():
        # Rewind to the prefilled state: length = prompt, history = prompt ids.
        rt.set_length(seq)
        rt.set_history(ids)
        toks, _ = rt.generate(first, first_raw, GEN_TOKENS, PENALTY)
        return toks

    for _ in range(args.warmup):
        toks = one_step()
        assert toks == res.generated_tokens, "decode is not deterministic"
    import torch
    ext = torch.cuda.ExternalStream(rt.stream, device=local)
    dist_barrier(world)
    torch.cuda.synchronize(local)
    with ClockSampler(local) as clocks:
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(ext)
        for _ in range(args.steps):
            one_step()
        e1.record(ext)
        e1.synchronize()
        torch.cuda.synchronize(local)
        dist_barrier(world)
    ms = e0.elapsed_time(e1)
    ms_max = dist_max(ms, world)
    decode_tokens = (n_tok - 1) * args.steps * world
    value = decode_tokens / (ms_max / 1e3)

    # The dominant kernel: the persistent decode kernel (one launch per <= 64 tokens),
    # launched back to back on the context stream with no host work between launches.
    rt.set_length(seq)
    rt.set_history(ids)
    dev_ms, _ = device_ms(rt, lambda: rt.bench_ar_steps(GEN_TOKENS - 1))
    launches = (GEN_TOKENS - 1 + MEGA_CHUNK - 1) // MEGA_CHUNK
    bpt = ar_bytes_per_token(seq, n_tok)
    peak, peak_kind = measured_peaks()
    mega_gbs = bpt * (GEN_TOKENS - 1) / (dev_ms / 1e3) / 1e9

    # e2e: reference-facing call with host buffers in pinned memory (prompt upload, prefill,
    # 256 tokens, tokens back), with the library's per-stage timing of every call.
    p_ids, p_pos, p_feats = (pinned_copy(a) for a in (ids, pos, feats))
    e2e_times, stages = [], []
    rt.run_vlm_decode_with_prompt(p_ids, p_pos, image_token, p_feats, max_tokens=GEN_TOKENS)   # untimed warm-up
    with ClockSampler(local) as e2e_clocks:
        for _ in range(max(1, args.steps)):
            t0 = time.perf_counter()
            r2 = rt.run_vlm_decode_with_prompt(p_ids, p_pos, image_token, p_feats, max_tokens=GEN_TOKENS)
            e2e_times.append(time.perf_counter() - t0)
            stages.append(r2.timing)
            assert r2.generated_tokens == res.generated_tokens
    # Whole-job throughput over the timed calls (tokens of all calls / their total time), max over ranks.
    e2e_t = dist_max(sum(e2e_times), world)
    e2e_value = len(r2.generated_tokens) * len(e2e_times) * world / e2e_t

    # Configs 1 and 2 alone: LM head + argmax (M=1), gate/up GEMV, attention at KV 1024.
    lm_ms = rt.bench_kernel(0, 20)
    gu_ms = rt.bench_kernel(1, 20)
    attn_ms = rt.bench_kernel(2, 50)
    rt.close()
    dflash = dflash_leg(pkg, local) if (world == 1 and not args.no_dflash) else None
    bf16 = bf16_leg(pkg, local, seq) if world == 1 else None
    requests = requests_leg(pkg, world, rank, local) if not args.no_requests else None
    if rank != 0:
        return None
    cs = clocks.summary()
    return {
        "metric": "decode tokens/s (AR, bs=1, fp32)",
        "value": round(value, 2),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_max / args.steps, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded random-init weights ~N(0,0.02); prompt 768 N(0,1) image rows + 256 text ids)",
        "config": workload_config(seq, n_tok, world),
        "device_loop_tokens_per_s": round((GEN_TOKENS - 1) / (dev_ms / 1e3), 2),
        "roofline": {"bound": "hbm", "kernel": "mega_decode_kernel<f32,f32> (persistent: whole tokens per launch)",
                     "achieved": round(mega_gbs, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(mega_gbs / peak, 4), "traffic": round(MEGA_TRAFFIC_RATIO * bpt * MEGA_CHUNK),
                     "peak_source": peak_kind, "bytes_per_token": round(bpt),
                     "tokens_per_launch": MEGA_CHUNK, "launch_us": round(dev_ms * 1e3 / launches, 1),
                     "roofline_tokens_per_s": round(peak * 1e9 / bpt, 1)},
        "kernel_us": {"lm_head_m1": round(lm_ms * 1e3, 2), "gate_up_gemv_m1": round(gu_ms * 1e3, 2),
                      "attention_kv1024_q1": round(attn_ms * 1e3, 2),
                      "lm_head_m1_gbs": round(LM_HEAD_BYTES / (lm_ms / 1e3) / 1e9, 1)},
        "ar_bf16": bf16,
        "dflash": dflash,
        "requests_config4": requests,
        "e2e": {"value": round(e2e_value, 2), "unit": "tokens/s", "scope": "prefill + 256 tokens per call",
                "ms_per_call": [round(t * 1e3, 1) for t in e2e_times], "clocks": e2e_clocks.summary(),
                "stages_ms_median": {k: round(float(np.median([getattr(t, k) for t in stages])), 3)
                                     for k in ("text_embed_ms", "prefill_ms", "lm_head_ms", "decode_ms", "total_ms",
                                               "host_overhead_ms")},
                "h2d_bytes_per_step": int(ids.nbytes + pos.nbytes + feats.nbytes),
                "d2h_bytes_per_step": int(2 * 4 * len(r2.generated_tokens))},
        "gpu_launches": int(launches * args.steps),
        "clocks": cs,
        "cpu_baseline": cpu_baseline(args) if (world == 1 and not args.no_cpu) else None,
    }


def load_batch_module():
    import importlib.util
    if "hy_b200_batch" in sys.modules:
        return sys.modules["hy_b200_batch"]
    spec = importlib.util.spec_from_file_location("hy_b200_batch", os.path.join(REPO, "hunyuanocr-ncnn_b200", "batch.py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules["hy_b200_batch"] = mod
    spec.loader.exec_module(mod)
    return mod


def run_requests(args, world, rank, local):
    """Config 4: `--requests` independent requests (prompt of request i seeded by i: 768
    image rows + 256 text ids), `--req-tokens` generated tokens each, partitioned
    round-robin across the ranks (one GPU each, full weight copy, no collective on the
    data path). AR mode: the reference-facing call per request. DFlash mode: prefill
    through the same call, then the on-device DFlash loop with synthetic drafts equal to
    the request's greedy tokens with probability 0.7 (the greedy tokens come from an
    untimed AR pass). Batch mode: each rank's records decode together through
    hy_batch_decode, 16 at a time (one 16-row step advances every record by a token)."""
    sys.path.insert(0, REPO)
    import __graft_entry__ as ge
    import torch
    pkg = ge.load_package()
    pkg.load_library()
    batch = load_batch_module()
    n_tok = args.req_tokens
    seq = PROMPT_GRID[0] * PROMPT_GRID[1] + PROMPT_TEXT
    rt = pkg.TextRuntime.synthetic(seed=0, device=local, max_prefill=seq, max_tokens=n_tok + 64,
                                   max_context=seq + n_tok + 64)
    prompts = {i: prompt_arrays(seed=i) for i in batch.partition(args.requests, world, rank)}
    greedy = {}
    if args.mode == "dflash":
        for i, (ids, pos, feats, img) in prompts.items():
            greedy[i] = rt.run_vlm_decode_with_prompt(ids, pos, img, feats, max_tokens=n_tok + 16).generated_tokens

    def infer(i):
        ids, pos, feats, img = prompts[i]
        if args.mode == "ar":
            return rt.run_vlm_decode_with_prompt(ids, pos, img, feats, max_tokens=n_tok).generated_tokens
        first = rt.run_vlm_decode_with_prompt(ids, pos, img, feats, max_tokens=1).generated_tokens[0]
        r = rt.dflash_generate_synthetic(first, n_tok, PENALTY, greedy[i], 0.7, seed=i)
        if r.generated_tokens != greedy[i][:len(r.generated_tokens)]:
            raise RuntimeError(f"request {i}: DFlash tokens differ from the AR tokens")
        return r.generated_tokens

    def infer_many(idx):
        toks, status = rt.batch_decode([(prompts[i][0], prompts[i][1], prompts[i][3], prompts[i][2]) for i in idx],
                                       n_tok, slots=args.slots)
        return [(st == 0, t if st == 0 else f"status {st}") for t, st in zip(toks, status)]

    records = list(range(args.requests))
    if prompts and args.mode == "batch":
        infer_many(list(prompts)[:2])   # warm-up (slot buffers, step graph, first-touch)
    elif prompts:
        infer(next(iter(prompts)))   # warm-up (graphs, first-touch)
    ext = torch.cuda.ExternalStream(rt.stream, device=local)
    dist_barrier(world)
    torch.cuda.synchronize(local)
    with ClockSampler(local) as clocks:
        t0 = time.perf_counter()
        if args.mode == "batch":
            local_out, summary = batch.run_partition_batched(records, infer_many, world=world, rank=rank)
        else:
            local_out, summary = batch.run_partition(records, infer, world=world, rank=rank)
        torch.cuda.synchronize(local)
        dt = time.perf_counter() - t0
        dist_barrier(world)
    dt_max = dist_max(dt, world)
    merged, total = batch.gather_in_order(local_out, world, rank)
    rt.close()
    if rank != 0:
        return None
    tokens = sum(len(r.tokens) for r in merged)
    return {
        "metric": f"request throughput (config 4, {args.mode.upper()}, "
                  f"{'up to ' + str(args.slots) + ' records per step' if args.mode == 'batch' else 'bs=1'} per GPU)",
        "value": round(tokens / dt_max, 2),
        "unit": "tokens/s",
        "requests_per_s": round(total.succeeded / dt_max, 3),
        "n_gpus": world,
        "steps": 1,
        "warmup": 1,
        "ms_per_step": round(dt_max * 1e3, 1),
        "higher_is_better": True,
        "scaling": "weak" if args.requests % world == 0 else "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded random-init weights; request i prompt seeded by i)",
        "config": {"workload": f"config4: {args.requests} requests x ({seq} prompt + {n_tok} tokens), "
                               f"round-robin over {world} GPU(s), {args.mode}",
                   "parallelism": f"replicas x{world} (request-parallel, no collective)"},
        "summary": {"total": total.total, "succeeded": total.succeeded, "failed": total.failed},
        "clocks": clocks.summary(),
    }


def cpu_threads() -> int:
    """Host threads this process may use (its CPU affinity)."""
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


_ORACLE = {}


def oracle_model():
    """The oracle and the config-0 weights, built once per process (untimed)."""
    if not _ORACLE:
        import importlib.util
        spec = importlib.util.spec_from_file_location("hy_oracle_build", os.path.join(REPO, "oracle", "build.py"))
        ob = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(ob)
        ob.build()
        sys.path.insert(0, os.path.join(REPO, "oracle"))
        import hy_oracle as O
        cfg = O.ModelConfig()
        _ORACLE.update(O=O, cfg=cfg, w=O.make_weights(cfg, 0))
    return _ORACLE["O"], _ORACLE["cfg"], _ORACLE["w"]


def blas_threads(n: int):
    """Context that runs numpy's BLAS on n threads, whatever OMP_NUM_THREADS the launcher set
    (torchrun sets it to 1), and the thread count BLAS reports inside it."""
    from threadpoolctl import threadpool_info, threadpool_limits
    lim = threadpool_limits(limits=n, user_api="blas")
    used = max([p.get("num_threads", 1) for p in threadpool_info() if p.get("user_api") == "blas"] or [1])
    return lim, used


def cpu_decode_sample(steps: int):
    """Time the oracle's AR decode step at full size on a KV cache of 1024 rows."""
    O, cfg, w = oracle_model()
    seq = PROMPT_GRID[0] * PROMPT_GRID[1] + PROMPT_TEXT
    cache = O.KVCache.empty(cfg.num_layers, seq + steps + 1)
    rng = np.random.default_rng(0)
    for li in range(cfg.num_layers):
        cache.k[li][:, :seq] = rng.standard_normal((8, seq, 128), dtype=np.float32)
        cache.v[li][:, :seq] = rng.standard_normal((8, seq, 128), dtype=np.float32)
    cache.length = seq
    history = list(range(0, 2 * seq, 2))
    tok = 7
    t0 = time.perf_counter()
    for i in range(steps):
        pos = seq + i
        h, _ = O.decoder_forward(w, cfg, w.embed[tok:tok + 1], O.make_decode_mask(pos), O.rope_rows(pos, 1, True),
                                 O.rope_rows(pos, 1, False), cache)
        tok, _ = O.select_next_token(O.lm_head(w, h)[0], history, PENALTY)
        history.append(tok)
    dt = time.perf_counter() - t0
    return steps / dt, dt


def cpu_prompt_sample(n_decode: int):
    """One bounded sample of the AR decode workload on the host: the 1024-row prompt's prefill
    and first token (run_decoder_prefill + select_next_token), then n_decode decode steps.
    Returns (prefill + first-token seconds, decode seconds)."""
    O, cfg, w = oracle_model()
    prompt = O.synthetic_prompt(0, PROMPT_GRID[0], PROMPT_GRID[1], PROMPT_TEXT, cfg.vocab)
    seq = prompt.input_ids.shape[0]
    t0 = time.perf_counter()
    hidden, cache, _ = O.prefill(w, cfg, prompt, seq + n_decode + 16)
    history = [int(t) for t in prompt.input_ids]
    tok, _ = O.select_next_token(O.lm_head(w, hidden[-1:])[0], history, PENALTY)
    history.append(tok)
    t1 = time.perf_counter()
    for i in range(n_decode):
        pos = seq + i
        h, _ = O.decoder_forward(w, cfg, w.embed[tok:tok + 1], O.make_decode_mask(pos), O.rope_rows(pos, 1, True),
                                 O.rope_rows(pos, 1, False), cache)
        tok, _ = O.select_next_token(O.lm_head(w, h)[0], history, PENALTY)
        history.append(tok)
    return t1 - t0, time.perf_counter() - t1


def cpu_baseline(args):
    n = cpu_threads()
    lim, used = blas_threads(n)
    with lim:
        steps = args.cpu_steps
        tps, dt = cpu_decode_sample(steps)
    return {"value": round(tps, 3), "unit": "tokens/s", "cores": used, "kind": "port",
            "sample": f"{steps} AR decode steps of the config0 model at KV length 1024 (oracle/hy_oracle.py, "
                      f"numpy fp32 GEMV + fp64 attention, {used} BLAS threads, {dt:.1f} s)"}


def run_reference(args, world, rank):
    """The reference's CPU path for this workload (ncnn cannot be built here, so the oracle port:
    numpy fp32 with fp64 attention), on all of this process's host threads. Each step is a
    bounded sample of the AR decode workload: the 1024-row prompt's prefill and first token,
    then --ref-decode decode steps. value = decode tokens/s (as the GPU arm's value); e2e = the
    GPU arm's e2e unit (prefill + 256 tokens per call) estimated from the sample as
    256 / (prefill time + 255 x mean decode-step time)."""
    if rank != 0:
        return None
    n = cpu_threads()
    lim, used = blas_threads(n)
    seq = PROMPT_GRID[0] * PROMPT_GRID[1] + PROMPT_TEXT
    with lim:
        oracle_model()
        for _ in range(args.warmup):
            cpu_decode_sample(2)
        pre, dec = [], []
        for _ in range(args.steps):
            tp, td = cpu_prompt_sample(args.ref_decode)
            pre.append(tp)
            dec.append(td)
    value = args.ref_decode * args.steps / sum(dec)
    t_tok = sum(dec) / (args.ref_decode * args.steps)
    e2e = GEN_TOKENS / (float(np.mean(pre)) + (GEN_TOKENS - 1) * t_tok)
    sample = (f"per step: prefill of the 1024-row prompt + first token ({np.mean(pre):.2f} s mean), then "
              f"{args.ref_decode} decode steps at KV 1024+ ({1e3 * t_tok:.0f} ms each); oracle/hy_oracle.py "
              f"(numpy fp32 + fp64 attention; ncnn is not available to build the reference's own CPU path), "
              f"{used} BLAS threads")
    base = {"value": round(value, 3), "unit": "tokens/s", "cores": used, "kind": "port", "sample": sample}
    return {"impl": "reference", "metric": "decode tokens/s (AR, bs=1, fp32)", "value": base["value"],
            "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(1e3 * (sum(pre) + sum(dec)) / args.steps, 2), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded random-init weights ~N(0,0.02); prompt 768 N(0,1) image rows + 256 text ids)",
            "config": workload_config(seq, GEN_TOKENS, world),
            "cpu_baseline": base,
            "e2e": {"value": round(e2e, 3), "unit": "tokens/s", "scope": "prefill + 256 tokens per call (estimated "
                    "from the sample)", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--cpu-steps", type=int, default=144)   # ~10 s of oracle decode on the host
    ap.add_argument("--ref-decode", type=int, default=16, help="decode steps per reference-arm step")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-dflash", action="store_true")
    ap.add_argument("--no-requests", action="store_true")
    ap.add_argument("--workload", choices=["decode", "requests"], default="decode",
                    help="decode: config 0 step (default); requests: config 4 request throughput")
    ap.add_argument("--requests", type=int, default=64)
    ap.add_argument("--req-tokens", type=int, default=512)
    ap.add_argument("--mode", choices=["ar", "dflash", "batch"], default="ar",
                    help="requests workload: ar (one record at a time), dflash (p = 0.7 synthetic drafts), "
                         "batch (records decode together, --slots at a time)")
    ap.add_argument("--slots", type=int, default=16)
    args = ap.parse_args()
    if args.impl == "reference":
        world, rank = int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0"))
        out = run_reference(args, world, rank)
    else:
        world, rank, local = dist_setup(args.gpus)
        out = run_requests(args, world, rank, local) if args.workload == "requests" else run_b200(args, world, rank, local)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
    if out is not None:
        print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
