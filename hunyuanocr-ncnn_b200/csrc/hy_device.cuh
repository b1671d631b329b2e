// Device primitives shared by the decode kernels (sm_100a).
//
// Weight and KV rows are streamed from HBM into shared memory with the bulk
// copy engine (cp.async.bulk, the non-tensor form of TMA; never with
// multicast), completing on an mbarrier. Every wait on an mbarrier is bounded
// by a wall-clock limit read from %globaltimer; a wait that gives up sets a
// bit in the context's device error word and the kernel drains its own copies
// before returning, so a fault in the pipeline reports an error instead of
// hanging the GPU.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace hy {

constexpr int kHidden = 1024;
constexpr int kHeadDim = 128;
constexpr int kNumQHeads = 16;
constexpr int kNumKVHeads = 8;
constexpr int kQWidth = kNumQHeads * kHeadDim;    // 2048
constexpr int kKVWidth = kNumKVHeads * kHeadDim;  // 1024
constexpr int kQKVRows = kQWidth + 2 * kKVWidth;  // 4096
constexpr int kMaxStepRows = 16;
constexpr int kBlock = 16;   // DFlash block
constexpr int kMaxEos = 8;
constexpr int kAuxLayers = 4;

// Device error bits (context error word).
constexpr int kErrTimeoutFull = 1;
constexpr int kErrTimeoutEmpty = 2;
constexpr int kErrBounds = 4;

constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s

// ---------------------------------------------------------------------------
// Decode state kept on the device between steps (no host round trip).
// ---------------------------------------------------------------------------
struct DecodeState {
    int kv_len;        // rows in the KV cache
    int cur_token;     // next token to embed (AR) / proposed[0] of the next block (DFlash)
    int n_gen;         // tokens written to the token log
    int max_tokens;    // generation limit (token log)
    int done;          // set by the commit when EOS or max_tokens is reached
    int block_count;   // DFlash blocks run
    int n_eos;
    int eos[kMaxEos];
    float penalty;
    // synthetic drafter
    int n_greedy;
    float draft_p;
    int pad0;
    unsigned long long draft_base;
    // last verify block outputs
    int accept;        // dflash_acceptance_length
    int committed;
    int stop;
    int pad1;
};

// One sequence of a batched decode (hy_batch_decode): step row m decodes the
// sequence in slot m, with its own KV cache, history bitmap and token log.
struct SlotState {
    int kv_len;       // rows in this slot's KV cache
    int active;       // 1 while the slot decodes; 0: empty or finished
    int n_gen;        // tokens in this slot's log
    int max_tokens;
};

// ---------------------------------------------------------------------------
// PTX wrappers.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init()
{
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// try_wait with a suspend-time hint: a thread whose phase has not completed is
// suspended (it stops issuing) until the phase completes or ~1 ms passes, so
// waiting warps leave the issue slots to the warps doing work.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(1000000u)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ unsigned long long global_ns()
{
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Bounded wait for phase `parity` of `bar`. Returns false (and sets `err_bit`
// in *err) when the wall-clock limit (limit_ns) passes first.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int err_bit,
                                          unsigned long long limit_ns = kWaitLimitNs)
{
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = global_ns();
    while (true)
    {
        if (mbar_try_wait(bar, parity)) return true;
        if (global_ns() - t0 > limit_ns)
        {
            if (err) atomicOr(err, err_bit);
            return false;
        }
    }
}

__device__ __forceinline__ uint64_t l2_evict_first_policy()
{
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// Bulk global->shared copy (no multicast). dst, src and bytes must be 16-byte aligned.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t pol)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}

// Bulk global->shared copy with the default L2 policy (for data other CTAs read too).
__device__ __forceinline__ void bulk_g2s_plain(void* dst, const void* src, uint32_t bytes, uint64_t* bar)
{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// Bulk prefetch of global memory into L2 (no destination, no completion).
// src and bytes must be 16-byte aligned.
// 2-D tiled TMA load (no multicast) of the box at element coordinates (x, y)
// of the tensor map `tmap` (kernel-parameter space), completing on `bar`.
__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, int x, int y, uint64_t* bar)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes)
{
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// Programmatic dependent launch: wait for the previous grid in the stream
// (a no-op when the launch carried no programmatic dependency) / let the next
// grid start its prologue.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Lets the next kernel in the stream (launched with programmatic stream
// serialization) start its CTAs once every CTA of this grid has called it or
// exited; that kernel's producers then stream constant weights while this one
// finishes, and its griddepcontrol.wait still waits for this grid's completion.
// Every kernel calls it only after its own pdl_wait, so whatever the grid
// before this one wrote is complete and visible when the next kernel starts:
// code before that kernel's wait may read data written two kernels back.
__device__ __forceinline__ void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Step trace (instrumented builds, -DHY_STEP_TRACE): CTA (0, 0, 0)'s thread 0 of
// every kernel of the per-phase paths opens a record {kernel id, %globaltimer at
// entry, after griddepcontrol.wait, after its prologue, at its end, three
// kernel-specific words, the latest exit of any CTA of the kernels before it,
// 16 more kernel-specific words}
// in g_step_trace, in launch order; hy_debug_step_trace reads them back. Every
// CTA's thread 0 raises g_step_last_exit when it ends (HY_STEP_TRACE_EXIT);
// read right after the wait, it is the previous grid's last exit. Off by
// default: the macros expand to nothing.
constexpr int kStepTraceMax = 16384;   // records
constexpr int kStepTraceWords = 25;    // words per record
#ifdef HY_STEP_TRACE
__device__ unsigned long long g_step_trace[kStepTraceMax * kStepTraceWords];
__device__ unsigned g_step_trace_n;
__device__ unsigned long long g_step_last_exit;
__device__ __forceinline__ unsigned long long step_trace_now()
{
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ unsigned long long* step_trace_open(unsigned long long id)
{
    const unsigned i = atomicAdd(&g_step_trace_n, 1u);
    if (i >= static_cast<unsigned>(kStepTraceMax)) return nullptr;
    unsigned long long* r = g_step_trace + static_cast<unsigned long long>(kStepTraceWords) * i;
    r[0] = id;
    r[1] = step_trace_now();
    for (int j = 2; j < kStepTraceWords; ++j) r[j] = 0;
    return r;
}
__device__ __forceinline__ void step_trace_mark(unsigned long long* r, int slot)
{
    if (!r) return;
    r[slot] = step_trace_now();
    if (slot == 2) r[8] = atomicAdd(&g_step_last_exit, 0ull);
}
#define HY_STEP_TRACE_OPEN(id)                                                                               \
    unsigned long long* hy_str_ =                                                                            \
        (blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && threadIdx.x == 0) ? step_trace_open(id) \
                                                                                    : nullptr
#define HY_STEP_TRACE_MARK(slot) step_trace_mark(hy_str_, (slot))
#define HY_STEP_TRACE_EXIT()                                                       \
    do                                                                             \
    {                                                                              \
        if (threadIdx.x == 0) atomicMax(&g_step_last_exit, step_trace_now());     \
    } while (0)
#else
#define HY_STEP_TRACE_OPEN(id)
#define HY_STEP_TRACE_MARK(slot)
#define HY_STEP_TRACE_EXIT()
#endif

// ---------------------------------------------------------------------------
// Numeric helpers.
// ---------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// Four consecutive elements of T as float4 (T = float: one 16-byte load;
// T = bf16: one 8-byte load).
template <typename T>
__device__ __forceinline__ float4 load4(const T* p);
template <>
__device__ __forceinline__ float4 load4<float>(const float* p) { return *reinterpret_cast<const float4*>(p); }
template <>
__device__ __forceinline__ float4 load4<__nv_bfloat16>(const __nv_bfloat16* p)
{
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    float4 r;
    r.x = __uint_as_float(u.x << 16);
    r.y = __uint_as_float(u.x & 0xFFFF0000u);
    r.z = __uint_as_float(u.y << 16);
    r.w = __uint_as_float(u.y & 0xFFFF0000u);
    return r;
}

__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float dot4(float4 a, float4 b)
{
    return a.x * b.x + a.y * b.y + a.z * b.z + a.w * b.w;
}

// splitmix64 finalizer; the synthetic weight generator and the synthetic
// drafter are both counter streams of it.
__host__ __device__ __forceinline__ unsigned long long splitmix64(unsigned long long z)
{
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__host__ __device__ __forceinline__ unsigned long long synth_base(unsigned long long seed, unsigned long long tid)
{
    return splitmix64(seed * 0x9E3779B97F4A7C15ull + tid * 0xD1B54A32D192ED03ull);
}

// Value i of a counter stream: offset + float(c) * mult with
// c = (sum of the four 16-bit fields of splitmix64(base + i)) - 131070,
// each step correctly rounded (no contraction into an FMA).
__device__ __forceinline__ float synth_value(unsigned long long base, unsigned long long i, float mult, float offset)
{
    const unsigned long long h = splitmix64(base + i);
    const int c = static_cast<int>((h & 0xFFFFull) + ((h >> 16) & 0xFFFFull) + ((h >> 32) & 0xFFFFull) + (h >> 48)) -
                  131070;
    return __fadd_rn(offset, __fmul_rn(static_cast<float>(c), mult));
}

}  // namespace hy
