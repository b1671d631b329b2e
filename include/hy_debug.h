/*
 * hy_debug.h — benchmark and diagnosis hooks of libhy_decode.so.
 *
 * These entry points are not part of the reference-facing boundary
 * (include/hy_decode.h): they time kernels, trace the persistent decode kernel
 * and report its waits. They have no counterpart in HunyuanOCR-ncnn except the
 * per-stage timers of include/hunyuan_ocr/text_runtime.h:32-39, which the
 * trace stands in for while tuning.
 */
#ifndef HY_DEBUG_H
#define HY_DEBUG_H

#include "hy_decode.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ---- device-resident timing hooks (benchmarks) ------------------------ */
/* Runs `count` AR steps back to back on the context's stream without host
 * copies (persistent launches of up to 64 tokens, or step-graph replays) and
 * returns the device time in ms (CUDA events). The sequence length is restored. */
int hy_bench_ar_steps(hy_ctx* ctx, int count, float* ms);
/* Times `count` launches of one kernel family on the context's stream:
 * which = 0: LM head GEMV + argmax (M=1); 1: gate/up GEMV of layer 0;
 * 2: attention of layer 0 at the current length (M=1). ms = mean per launch. */
int hy_bench_kernel(hy_ctx* ctx, int which, int count, float* ms);

/* ---- bounded waits ----------------------------------------------------- */
/* Bound of every wait inside the persistent decode kernel (mbarrier waits and
 * polls of epoch words; default 2 s, accepted 1 ms .. 60 s). A wait that runs
 * out makes the kernel wind down and the call return HY_ERR_DEVICE_TIMEOUT. */
int hy_ctx_set_wait_limit(hy_ctx* ctx, unsigned long long limit_ns);
/* Failure-detection self-test: one small kernel waits, with the library's own
 * bounded primitives, for something that nothing provides - kind 0 polls an
 * epoch word that never carries the awaited epoch, kind 1 waits on an
 * mbarrier phase that never completes - and gives up after limit_ns
 * (1 us .. 10 s). Returns HY_ERR_DEVICE_TIMEOUT with the error word cleared, so
 * the context stays usable; HY_OK would mean the wait did not run out. */
int hy_debug_wait_probe(hy_ctx* ctx, int kind, unsigned long long limit_ns);

/* ---- persistent-kernel diagnosis -------------------------------------- */
/* Per-phase trace: runs `tokens` AR steps from the current state and, for the
 * traced CTAs during token `trace_token`, stores
 * out[(cta * (5 * num_layers + 1) + phase) * 12 + i] (thread 0 of the CTA):
 *   i = 0..3  %globaltimer (ns) at phase start, when the phase's inputs were
 *             ready, after the prologue and at phase end;
 *   i = 4..6  GEMV phases: warp 0's SM cycles waiting for its stages, cycles
 *             in its dot products and epilogues, and its stage count;
 *   i = 7, 8, 10  GEMV phases that poll (not layer 0's q/k/v): poll rounds,
 *             ns from the first poll to the last word, and the first poll's
 *             %globaltimer;
 *   i = 7..10 attention: the slot-wait / work cycles and stages of the warp
 *             owning the split's first stage, and the time its stage loop ended.
 * The sequence length is restored afterwards. */
int hy_trace_persistent(hy_ctx* ctx, int tokens, int trace_token, unsigned long long* out);
/* With HY_DEBUG_PROGRESS=1 in the environment at context creation, each CTA
 * records in host-mapped memory how many phases it completed; readable even
 * after a device fault. */
int hy_debug_progress(const hy_ctx* ctx, unsigned* out, int n);
/* Wait statistics of the persistent kernel, in a library built with
 * HY_WAIT_STATS defined (HY_ERR_UNSUPPORTED otherwise). out[n_words] receives
 * (up to) the statistics buffer: for CTA b < 160 and wait kind k < 10 (slot
 * free, slot full, producer slot, producer token, residual poll, SwiGLU poll,
 * attention-output poll, q/k/v poll, split-partial poll, token poll), at
 * (b * 10 + k) * 3: the number of waits longer than 20 us, their total ns and
 * the longest such wait; then for launch slot s < 64 (launches numbered from
 * the last reset) at 4800 + 2 s: the bitwise NOT of the first CTA's start and
 * the last CTA's exit (%globaltimer ns). reset != 0 zeroes the buffer and the
 * launch numbering after the copy. */
int hy_debug_wait_stats(hy_ctx* ctx, unsigned long long* out, int n_words, int reset);
/* Step trace of the per-phase kernels (projections, RoPE/append, attention,
 * merges), in a library built with HY_STEP_TRACE defined (HY_ERR_UNSUPPORTED
 * otherwise): after the context's stream is idle, out[25 * i ..] receives, for
 * the first max_records launches since the last reset in the order their
 * CTA 0 started, {kernel id, %globaltimer ns at CTA 0's entry, after its
 * griddepcontrol.wait, after its prologue (projections), at its end; for the
 * 16-row projections the ns thread 0 waited for its weight units, the ns in
 * their MMAs and the %globaltimer after its last unit; the latest exit of any
 * CTA of the kernels before it, read after its wait; for the 16-row
 * projections each consumer warp's %globaltimer after its last unit (8 words)
 * and its ns waiting for units (8 words)} (25 words per record), 0 where a
 * point was not passed; *n_records = the launches recorded (at most 16384).
 * Kernel ids: 0x1_MM_KK_PE projections (MM rows, KK = K / 128, P prologue,
 * E epilogue), 0x2 RoPE/append, 0x3_QR step attention, 0x4 chunk merge,
 * 0x5_MT decode attention. reset != 0 restarts the record count. */
int hy_debug_step_trace(hy_ctx* ctx, unsigned long long* out, int max_records, int* n_records, int reset);

#ifdef __cplusplus
}
#endif

#endif /* HY_DEBUG_H */
