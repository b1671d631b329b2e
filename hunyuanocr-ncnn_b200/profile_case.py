"""Small, self-contained decode workload for profiling the decode kernels.

Builds a synthetic context (seeded random weights) with a reduced layer count
and vocabulary so that one kernel launch is short and the device footprint is a
few hundred MB (still larger than L2), sets the KV length, and runs a few AR
decode launches. Meant to be run under a profiler, e.g.

    ncu --set full --clock-control none -k regex:mega_decode -s 1 -c 1 \
        python hunyuanocr-ncnn_b200/profile_case.py

Prints one line with the last launch's device time.
"""
import argparse
import os
import sys

_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if _ROOT not in sys.path:
    sys.path.insert(0, _ROOT)


KERNEL_NAMES = {0x2: "rope/append", 0x3: "step attention", 0x4: "chunk merge", 0x5: "decode attention"}
LM16_ID = 0x100000000 | (16 << 24) | (8 << 8) | (1 << 4) | 2   # 16-row LM head (K 1024, norm, argmax)


def kernel_name(kid: int) -> str:
    kind = kid >> 32
    if kind == 1:
        mt, kp, pro, epi = (kid >> 24) & 0xFF, ((kid >> 8) & 0xFFFF) * 128, (kid >> 4) & 0xF, kid & 0xF
        return (f"proj M{mt} K{kp} " + ["plain", "norm", "swiglu"][pro] + " -> " +
                ["store", "resid", "argmax", "swiglu"][epi])
    return KERNEL_NAMES.get(kind, hex(kid)) + (f" {kid & 0xFF}" if kind in (3, 5) else "")


def print_step_trace(rec, label):
    """Where a block's (or step's) time goes: the launches between the middle pair of
    16-row LM-head launches, grouped by kernel. Per launch i: CTA 0's entry E, the return
    of its griddepcontrol.wait W (= the previous grid complete), the end of its prologue
    P and its end X; critical-path time W[i+1] - W[i]."""
    import numpy as np

    rec = rec.astype(np.int64)
    lm = np.nonzero(rec[:, 0] == LM16_ID)[0]
    if len(lm) < 3:
        print(f"step trace: {len(rec)} records, fewer than 3 blocks")
        return
    a, b = lm[len(lm) // 2 - 1] + 1, lm[len(lm) // 2] + 1   # the block ending at LM-head launch lm[mid]
    seg = rec[a:b + 1]
    W = seg[:, 2]
    total = (W[-1] - W[0]) / 1e3
    print(f"step trace ({label}): {b - a} launches, {total:.1f} us from the first launch's wait to the next "
          f"block's first wait")
    print(f"{'kernel':<40} {'n':>4} {'crit_us':>8} {'entry_early':>11} {'prologue':>9} {'main':>7} {'tail':>7}"
          f" {'spread':>7} {'handoff':>7} {'unit_wait':>9} {'unit_mma':>8} {'epilogue':>8}")
    groups = {}
    for i in range(len(seg) - 1):
        kid = int(seg[i, 0])
        g = groups.setdefault(kid, [])
        e, w, p, x = seg[i, 1:5]
        crit = (seg[i + 1, 2] - w) / 1e3
        early = (w - seg[i + 1, 1]) / 1e3   # how long before this kernel's wait returned the next CTA 0 started
        pro = (p - w) / 1e3 if p else 0.0
        main = (x - (p if p else w)) / 1e3 if x else 0.0
        tail = (seg[i + 1, 2] - x) / 1e3 if x else 0.0
        uw, um = seg[i, 5] / 1e3, seg[i, 6] / 1e3
        epi = (x - seg[i, 7]) / 1e3 if (x and seg[i, 7]) else 0.0
        last = seg[i + 1, 8]   # this grid's last CTA exit, read by the next kernel after its wait
        spread = (last - x) / 1e3 if (x and last) else 0.0
        handoff = (seg[i + 1, 2] - last) / 1e3 if last else 0.0
        g.append((crit, early, pro, main, tail, spread, handoff, uw, um, epi))
    # Per-warp finish of the 16-row projections (CTA 0): last-unit time after the wait.
    for kid in sorted(groups):
        rows_k = [i for i in range(len(seg) - 1) if int(seg[i, 0]) == kid and seg[i, 9]]
        if not rows_k:
            continue
        ends = np.array([(seg[i, 9:17] - seg[i, 2]) / 1e3 for i in rows_k]).mean(axis=0)
        waits = np.array([seg[i, 17:25] / 1e3 for i in rows_k]).mean(axis=0)
        print(f"  {kernel_name(kid):<38} warps' last unit after the wait: " + " ".join(f"{x:5.2f}" for x in ends) +
              "  | waits: " + " ".join(f"{x:4.2f}" for x in waits))
    for kid, g in sorted(groups.items(), key=lambda kv: -sum(v[0] for v in kv[1])):
        v = np.array(g)
        m = v.mean(axis=0)
        print(f"{kernel_name(kid):<40} {len(g):4d} {m[0]:8.2f} {m[1]:11.2f} {m[2]:9.2f} {m[3]:7.2f} {m[4]:7.2f}"
              f" {m[5]:7.2f} {m[6]:7.2f} {m[7]:9.2f} {m[8]:8.2f} {m[9]:8.2f}   (sum {v[:, 0].sum():.1f} us)")


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--vocab", type=int, default=16384)
    ap.add_argument("--past", type=int, default=1024, help="KV length before decoding")
    ap.add_argument("--tokens", type=int, default=8, help="tokens per measured call")
    ap.add_argument("--calls", type=int, default=3)
    ap.add_argument("--path", choices=["persistent", "graph"], default="persistent")
    ap.add_argument("--dtype", choices=["f32", "bf16"], default="f32", help="weight and KV dtype")
    ap.add_argument("--draft-layers", type=int, default=5, help="draft mode: DFlash draft depth")
    ap.add_argument("--records", type=int, default=16, help="batch mode: records decoding together")
    ap.add_argument("--lib", default=None, help="library to load (default: the in-tree build)")
    ap.add_argument("--trace-ctas", type=int, default=4,
                    help="trace mode: CTAs the library traces (its HY_TRACE_CTAS; 4 in the default build)")
    ap.add_argument("--kernel", choices=["decode", "lm", "gate_up", "attention", "verify", "prefill", "draft",
                                         "batch", "trace"],
                    default="decode",
                    help="decode: AR launches; lm / gate_up / attention: the M=1 kernels alone "
                         "(hy_bench_kernel); verify: DFlash verify blocks (16-row kernels); "
                         "prefill: prompt prefill of --past rows (tcgen05 GEMMs, prefill attention); "
                         "draft: DFlash blocks with a synthetic draft network over a --past-row context; "
                         "batch: --records prompts of --past rows decoded together (hy_batch_decode); "
                         "trace: per-phase timeline of the middle token of a --tokens launch of the "
                         "persistent kernel (hy_trace_persistent), averaged over the layers for CTA 0")
    ap.add_argument("--step-trace", action="store_true",
                    help="verify / batch / draft: read the step trace of the last call (a library built with "
                         "HY_STEP_TRACE, given by --lib) and print where the middle block's or step's time goes")
    args = ap.parse_args(argv)

    import __graft_entry__ as ge

    pkg = ge.load_package()
    if args.lib:
        pkg.load_library(os.path.abspath(args.lib))
    dt = pkg.DTYPE_F32 if args.dtype == "f32" else pkg.DTYPE_BF16
    if args.kernel == "prefill":
        import time

        import numpy as np

        rows = args.past
        rt = pkg.TextRuntime.synthetic(seed=0, num_layers=args.layers, vocab_size=args.vocab, max_prefill=rows,
                                       max_tokens=16, max_context=rows + 16, weight_dtype=dt, kv_dtype=dt)
        rng = np.random.default_rng(0)
        emb = rng.standard_normal((rows, 1024)).astype(np.float32)
        ang = np.arange(rows)[:, None] * 1e-3 * np.arange(128)[None, :]
        cos, sin = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
        dt_ms = 0.0
        for _ in range(args.calls):
            rt.reset()
            t0 = time.perf_counter()
            rt.prefill(emb, cos, sin)
            dt_ms = (time.perf_counter() - t0) * 1e3
        print(f"prefill {args.dtype} layers={args.layers} vocab={args.vocab} rows={rows}: {dt_ms:.2f} ms per call (wall)")
        rt.close()
        return
    if args.kernel == "batch":
        import numpy as np

        rt = pkg.TextRuntime.synthetic(seed=0, num_layers=args.layers, vocab_size=args.vocab, max_prefill=args.past,
                                       max_tokens=args.tokens + 8, max_context=args.past + args.tokens + 8,
                                       weight_dtype=dt, kv_dtype=dt)
        rng = np.random.default_rng(0)
        img = args.vocab - 3
        reqs = []
        for _ in range(args.records):
            ids = rng.integers(0, args.vocab - 3, args.past).astype(np.int32)
            ids[:16] = img
            pos = np.tile(np.arange(args.past, dtype=np.int32), (4, 1))
            reqs.append((ids, pos, img, rng.standard_normal((16, 1024)).astype(np.float32)))
        for c in range(args.calls):
            if args.step_trace and c == args.calls - 1:
                rt.step_trace(reset=True)
            toks, _ = rt.batch_decode(reqs, args.tokens)
        print(f"batch {args.dtype} layers={args.layers} vocab={args.vocab} prompt={args.past} "
              f"records={args.records}: {len(toks[0])} tokens per record")
        if args.step_trace:
            print_step_trace(rt.step_trace(reset=True), f"batched decode step, {args.records} records")
        rt.close()
        return
    rt = pkg.TextRuntime.synthetic(seed=0, num_layers=args.layers, vocab_size=args.vocab, max_prefill=64,
                                   max_tokens=args.tokens + 40, max_context=args.past + args.tokens + 40,
                                   weight_dtype=dt, kv_dtype=dt)
    rt.ar_path = pkg.AR_PATH_PERSISTENT if args.path == "persistent" else pkg.AR_PATH_GRAPH
    if args.kernel == "trace":
        import numpy as np

        rt.set_length(args.past)
        rt.set_history([1, 2, 3])
        import ctypes

        phases = 5 * args.layers + 1
        raw = np.zeros((args.trace_ctas, phases, 12), np.uint64)
        lib = pkg.load_library()
        rc = lib.hy_trace_persistent(rt._ctx, args.tokens, args.tokens // 2, raw.ctypes.data_as(ctypes.c_void_p))
        if rc != 0:
            raise RuntimeError(f"hy_trace_persistent: status {rc}")
        tr = raw.astype(np.int64)
        c0 = tr[0]
        names = ["q/k/v", "attention", "o_proj", "gate/up", "down_proj"]
        L = args.layers
        print(f"trace layers={L} vocab={args.vocab} past={args.past} tokens={args.tokens} token={args.tokens // 2}: "
              f"token time {(c0[-1, 3] - c0[0, 0]) / 1e3:.1f} us (CTA 0)")
        print("phase        duration_us  inputs_ready_after_us  work_after_us")
        for k, name in enumerate(names):
            rows = c0[k:5 * L:5]
            dur, ready = (rows[:, 3] - rows[:, 0]) / 1e3, (rows[:, 1] - rows[:, 0]) / 1e3
            print(f"{name:<12} {dur.mean():11.2f} {ready.mean():22.2f} {(dur - ready).mean():14.2f}")
        lm = c0[5 * L]
        print(f"{'LM head':<12} {(lm[3] - lm[0]) / 1e3:11.2f} {(lm[1] - lm[0]) / 1e3:22.2f} "
              f"{(lm[3] - lm[1]) / 1e3:14.2f}")
        spread = (tr[:, :5 * L, 1].max(axis=0) - tr[:, :5 * L, 1].min(axis=0)) / 1e3
        print(f"inputs-ready spread over CTAs 0-{args.trace_ctas - 1}: mean {spread.mean():.2f} us, "
              f"max {spread.max():.2f} us")
        ready = (c0[:5 * L, 1] - c0[:5 * L, 0]) / 1e3
        print(f"token boundary: layer 0 q/k/v inputs ready after {ready[0]:.2f} us, layers 1-{L - 1}: "
              f"{ready[5::5].mean():.2f} us (CTA 0)")
        for k, name in enumerate(names):
            ends = tr[:, k:5 * L:5, 3]
            late = ((ends - ends.min(axis=0, keepdims=True)) / 1e3).mean(axis=1)
            order = np.argsort(-late)[:4]
            print(f"{name:<12} phase end after the earliest CTA's: mean {late.mean():.2f} us, max {late.max():.2f} us "
                  f"(latest CTAs {[int(i) for i in order]})")
        rt.close()
        return
    if args.kernel in ("lm", "gate_up", "attention"):
        rt.set_length(args.past)
        which = {"lm": 0, "gate_up": 1, "attention": 2}[args.kernel]
        if args.step_trace:
            rt.step_trace(reset=True)
        ms = rt.bench_kernel(which, args.calls)
        print(f"{args.kernel} {args.dtype} layers={args.layers} vocab={args.vocab} past={args.past}: "
              f"{ms * 1e3:.2f} us per launch")
        if args.step_trace:
            import numpy as np

            rec = rt.step_trace(reset=True).astype(np.int64)[1:]   # the timed launches
            e, w, x, last = rec[:, 1], rec[:, 2], rec[:, 4], rec[:, 8]
            print(f"step trace ({len(rec)} launches of {kernel_name(int(rec[0, 0]))}, us): "
                  f"critical path {np.mean(np.diff(w)) / 1e3:.2f}, CTA 0 entry before the previous wait "
                  f"{np.mean(w[:-1] - e[1:]) / 1e3:.2f}, CTA 0 wait -> end {np.mean(x - w) / 1e3:.2f}, "
                  f"CTA 0 end -> last CTA end {np.mean(last[1:] - x[:-1]) / 1e3:.2f}, "
                  f"last CTA end -> next wait {np.mean(w[1:] - last[1:]) / 1e3:.2f}")
        rt.close()
        return
    if args.kernel == "draft":
        import numpy as np

        rt.load_draft_synthetic(args.draft_layers, seed=3, std=0.02)
        rt.draft_context_append(np.random.default_rng(0).standard_normal((4, args.past, 1024), dtype=np.float32))
        for c in range(args.calls):
            rt.set_length(args.past)
            rt.set_history([1, 2, 3])
            if args.step_trace and c == args.calls - 1:
                rt.step_trace(reset=True)
            r = rt.dflash_generate(7, args.tokens, 1.08)
        print(f"draft {args.dtype} layers={args.layers} draft_layers={args.draft_layers} vocab={args.vocab} "
              f"past={args.past}: {r.block_count} blocks per call")
        if args.step_trace:
            print_step_trace(rt.step_trace(reset=True), "DFlash block with the draft network")
        rt.close()
        return
    if args.kernel == "verify":
        rt.set_length(args.past)
        rt.set_history([1, 2, 3])
        greedy = [5] * (args.tokens + 32)
        for c in range(args.calls):
            rt.set_length(args.past)
            if args.step_trace and c == args.calls - 1:
                rt.step_trace(reset=True)
            r = rt.dflash_generate_synthetic(7, args.tokens, 1.08, greedy, 0.0, seed=3)
        print(f"verify {args.dtype} layers={args.layers} vocab={args.vocab} past={args.past}: "
              f"{r.block_count} blocks per call")
        if args.step_trace:
            print_step_trace(rt.step_trace(reset=True), "DFlash verify block")
        rt.close()
        return
    ms = 0.0
    for _ in range(args.calls):
        rt.set_length(args.past)
        rt.set_history([1, 2, 3])
        ms = rt.bench_ar_steps(args.tokens)
    print(f"{args.path} {args.dtype} layers={args.layers} vocab={args.vocab} past={args.past} "
          f"tokens={args.tokens}: {ms:.3f} ms per call")
    rt.close()


if __name__ == "__main__":
    main()
