/*
 * Test infrastructure, not product code: the counter-based synthetic weight
 * generator in plain C, used by the CPU oracle to build full-size (24-layer,
 * 120818-vocab) weight sets in a few seconds. Only tests/, the smoke check and
 * bench.py's CPU-baseline leg load this library.
 *
 * The generator is defined so that numpy (oracle/hy_oracle.py::synth_tensor),
 * this file and the CUDA generator in the product library produce bit-identical
 * fp32 values: everything up to the last step is integer arithmetic, and the
 * last step is one correctly rounded fp32 multiply (and one fp32 add when an
 * offset is requested).
 *
 *   base  = splitmix64(seed * 0x9E3779B97F4A7C15 + tensor_id * 0xD1B54A32D192ED03)
 *   h_i   = splitmix64(base + i)
 *   c_i   = sum of the four 16-bit fields of h_i  - 131070      (Irwin-Hall n=4)
 *   v_i   = offset + (float)c_i * mult,  mult = (float)(std * sqrt(3) / 65536)
 *
 * c_i has mean 0 and standard deviation 65536/sqrt(3), so v_i has mean `offset`
 * and standard deviation `std`. The reference's random-init N(0, 0.02) weights
 * are stood in for by this bounded approximation of the normal law.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>

static inline uint64_t splitmix64(uint64_t z)
{
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

float hy_synth_mult(float std_dev)
{
    return (float)((double)std_dev * sqrt(3.0) / 65536.0);
}

void hy_synth_fill(uint64_t seed, uint64_t tensor_id, float std_dev, float offset,
                   float* out, size_t count)
{
    const uint64_t base = splitmix64(seed * 0x9E3779B97F4A7C15ull + tensor_id * 0xD1B54A32D192ED03ull);
    const float mult = hy_synth_mult(std_dev);
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)count; ++i)
    {
        const uint64_t h = splitmix64(base + (uint64_t)i);
        const int32_t c = (int32_t)((h & 0xFFFFu) + ((h >> 16) & 0xFFFFu) + ((h >> 32) & 0xFFFFu) + (h >> 48)) - 131070;
        const float v = (float)c * mult;
        out[i] = offset + v;
    }
}
