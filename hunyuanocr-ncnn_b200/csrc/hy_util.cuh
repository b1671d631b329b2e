// Small device utilities: synthetic weight fill, dtype conversion, final
// RMSNorm of hidden rows, prompt embedding with vision-feature injection,
// penalty-history bitmap updates.
#pragma once

#include "hy_device.cuh"

namespace hy {

template <typename WT>
__global__ void synth_fill_kernel(WT* out, size_t count, unsigned long long base, float mult, float offset)
{
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < count;
         i += static_cast<size_t>(gridDim.x) * blockDim.x)
        out[i] = from_f32<WT>(synth_value(base, i, mult, offset));
}

// Row r of a [rows x cols] counter stream goes to row r * row_mult + row_off of out.
template <typename WT>
__global__ void synth_fill_rows_kernel(WT* out, int rows, int cols, int row_mult, int row_off, unsigned long long base,
                                       float mult)
{
    const size_t count = static_cast<size_t>(rows) * cols;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < count;
         i += static_cast<size_t>(gridDim.x) * blockDim.x)
    {
        const size_t r = i / cols, c = i % cols;
        out[(r * row_mult + row_off) * cols + c] = from_f32<WT>(synth_value(base, i, mult, 0.0f));
    }
}

__global__ void f32_to_bf16_rows_kernel(const float* in, __nv_bfloat16* out, int rows, int cols, int row_mult,
                                        int row_off)
{
    const size_t count = static_cast<size_t>(rows) * cols;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < count;
         i += static_cast<size_t>(gridDim.x) * blockDim.x)
    {
        const size_t r = i / cols, c = i % cols;
        out[(r * row_mult + row_off) * cols + c] = __float2bfloat16_rn(in[i]);
    }
}

__global__ void f32_to_bf16_kernel(const float* in, __nv_bfloat16* out, size_t count)
{
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < count;
         i += static_cast<size_t>(gridDim.x) * blockDim.x)
        out[i] = __float2bfloat16_rn(in[i]);
}

template <typename T>
__global__ void to_f32_kernel(const T* in, float* out, size_t count)
{
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < count;
         i += static_cast<size_t>(gridDim.x) * blockDim.x)
        out[i] = to_f32<T>(in[i]);
}

// hidden[m] = final RMSNorm of x[m] (the decoder's `norm`, export/text_decoder_kv.py:112, 183).
// One CTA of 256 threads per row.
__global__ void rmsnorm_rows_kernel(const float* x, const float* w, float eps, float* out, int ld_in)
{
    __shared__ float red[8];
    const int m = blockIdx.x, tid = threadIdx.x;
    const float* xr = x + static_cast<size_t>(m) * ld_in;
    const float4 v = *reinterpret_cast<const float4*>(xr + tid * 4);
    float ss = warp_sum(v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    float t = 0.f;
    for (int i = 0; i < 8; ++i) t += red[i];
    const float ri = 1.0f / sqrtf(t / static_cast<float>(kHidden) + eps);
    const float4 wv = *reinterpret_cast<const float4*>(w + tid * 4);
    float4 o;
    o.x = wv.x * (v.x * ri);
    o.y = wv.y * (v.y * ri);
    o.z = wv.z * (v.z * ri);
    o.w = wv.w * (v.w * ri);
    *reinterpret_cast<float4*>(out + static_cast<size_t>(m) * kHidden + tid * 4) = o;
}

// prepare_prompt_embeddings (src/text_runtime.cpp:506-568): row t is the
// embedding of ids[t], or vision feature feat_idx[t] when feat_idx[t] >= 0.
template <typename WT>
__global__ void embed_prompt_kernel(const int* ids, const int* feat_idx, const float* feats, const WT* table, int vocab,
                                    float* out, int* err)
{
    const int t = blockIdx.x, tid = threadIdx.x;
    float4* dst = reinterpret_cast<float4*>(out + static_cast<size_t>(t) * kHidden) + tid;
    const int f = feat_idx[t];
    if (f >= 0)
    {
        *dst = reinterpret_cast<const float4*>(feats + static_cast<size_t>(f) * kHidden)[tid];
        return;
    }
    int id = ids[t];
    if (id < 0 || id >= vocab)
    {
        if (tid == 0) atomicOr(err, kErrBounds);
        id = 0;
    }
    *dst = load4(table + static_cast<size_t>(id) * kHidden + tid * 4);
}

// build_mrope (src/text_runtime.cpp:42-63) for positions inside the context's
// 1-D RoPE table: entry (t, d) of the 4-axis table is the 1-D table's entry at
// position_ids[d / 32][t] (the same base, inverse frequency and float angle per
// element), so the prompt's tables are gathered on the device rather than
// evaluated on the host. Block t, thread d; positions outside the table were
// rejected on the host (a bounds error here is a defect).
__global__ void mrope_gather_kernel(const int* pos, int seq, const float* cos1, const float* sin1, int rows,
                                    float* cos_out, float* sin_out, int* err)
{
    const int t = blockIdx.x, d = threadIdx.x;
    int p = pos[(d / (kHeadDim / 4)) * seq + t];
    if (p < 0 || p >= rows)
    {
        atomicOr(err, kErrBounds);
        p = 0;
    }
    cos_out[static_cast<size_t>(t) * kHeadDim + d] = cos1[static_cast<size_t>(p) * kHeadDim + d];
    sin_out[static_cast<size_t>(t) * kHeadDim + d] = sin1[static_cast<size_t>(p) * kHeadDim + d];
}

__global__ void hist_add_kernel(unsigned* bits, const int* ids, int n, int vocab)
{
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    {
        const int t = ids[i];
        if (t >= 0 && t < vocab) atomicOr(&bits[t >> 5], 1u << (t & 31));
    }
}

}  // namespace hy
