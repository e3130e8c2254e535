// Shared device helpers of the UltraNCA-B200 kernels: update-mask RNG, TF32 rounding, tile geometry, error word.
//
// Semantics restated from the UltraNCA reference (paths relative to that repository):
//   - Philox4x32-10 update mask: ncaops/nca_step.cuh:187-212 (key = seed, counter = (n H + Y) ceil(W/4) + X/4, word X%4,
//     m = floor(U + rate) != 0 with U = (word >> 8) 2^-24), the published algorithm of Salmon et al. (SC'11);
//   - TF32 operand rounding, round to nearest, ties away: ncaops/nca_step.cuh:115-120 (cvt.rna.tf32.f32);
//   - perception filters [identity, sobel_x, sobel_x^T, laplacian], circular padding, feature 4c + f:
//     ncaops/nca_step.cuh:81-87,311-321 and ncaops/testing/test_nca.py:11-12,29.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace unca {

// ---------------------------------------------------------------- error word
// Device-side failures (a bounded wait that ran out) set this word instead of trapping; the host reads it with
// nca_device_error(). Codes: 1 = MMA completion wait timed out. (The library is one translation unit.)
__device__ int g_device_error = 0;

__device__ __forceinline__ void set_device_error(int code) { atomicCAS(&g_device_error, 0, code); }

// ---------------------------------------------------------------- step seeds
// splitmix64 seed of rollout step i from the rollout's seed (ncaops/nca_cuda.cu:157-164): the host derives it for a
// host-driven launch, the kernels for a launch that reads its rollout seed from device memory.
__host__ __device__ __forceinline__ uint64_t splitmix_step(uint64_t seed, uint64_t i)
{
    uint64_t z = seed + (i + 1) * 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// ---------------------------------------------------------------- Philox mask
__device__ __forceinline__ uint4 philox4x32_10(uint64_t seed, uint64_t counter)
{
    uint32_t c0 = (uint32_t)counter, c1 = (uint32_t)(counter >> 32), c2 = 0u, c3 = 0u;
    uint32_t k0 = (uint32_t)seed, k1 = (uint32_t)(seed >> 32);
#pragma unroll
    for (int r = 0; r < 10; ++r) {
        const uint32_t lo0 = 0xD2511F53u * c0, hi0 = __umulhi(0xD2511F53u, c0);
        const uint32_t lo1 = 0xCD9E8D57u * c2, hi1 = __umulhi(0xCD9E8D57u, c2);
        const uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
        c0 = n0; c1 = lo1; c2 = n2; c3 = lo0;
        k0 += 0x9E3779B9u; k1 += 0xBB67AE85u;
    }
    return make_uint4(c0, c1, c2, c3);
}

// m(n, Y, X) in {0, 1}; n is the GLOBAL image index (a shard adds its image offset).
__device__ __forceinline__ float update_mask_at(uint64_t seed, float rate, int64_t n, int H, int W, int Y, int X)
{
    const uint64_t quads = (uint64_t)((W + 3) / 4);
    const uint64_t counter = ((uint64_t)n * (uint64_t)H + (uint64_t)Y) * quads + (uint64_t)(X / 4);
    const uint4 w = philox4x32_10(seed, counter);
    const int e = X & 3;
    const uint32_t word = e == 0 ? w.x : e == 1 ? w.y : e == 2 ? w.z : w.w;
    const float u = __fmul_rn((float)(word >> 8), 1.0f / 16777216.0f);
    return floorf(__fadd_rn(u, rate)) != 0.f ? 1.f : 0.f;
}

// ---------------------------------------------------------------- TF32
// Round to TF32 (10 explicit mantissa bits), to nearest with ties away from zero: the result of cvt.rna.tf32.f32 for
// every finite input, computed with two integer ALU operations instead of the conversion unit (adding half of the
// dropped 13-bit unit to the magnitude carries exactly when the dropped bits are >= half; the sign is untouched).
__device__ __forceinline__ float tf32_rna(float v)
{
    return __uint_as_float((__float_as_uint(v) + 0x1000u) & 0xFFFFE000u);
}

// tf32_rna for a value that only tcgen05.mma kind::tf32 reads: the MMA takes the upper 19 bits of an fp32 operand
// (sign, exponent, 10 mantissa bits) and ignores the other 13, so adding the rounding bias is enough (one integer
// operation). Measured on the B200: the step kernels' outputs are bitwise those of tf32_rna operands.
__device__ __forceinline__ float tf32_bias(float v) { return __uint_as_float(__float_as_uint(v) + 0x1000u); }

// ---------------------------------------------------------------- perception
// The four filters of one channel from its 3x3 neighbourhood v (rows dy = -1..1, columns dx = -1..1), summed in the
// reference's grouping (ncaops/nca_step.cuh:317-320).
__device__ __forceinline__ float4 perceive3x3(const float (&v)[3][3])
{
    float4 p;
    p.x = v[1][1];
    p.y = __fadd_rn(__fadd_rn(__fsub_rn(v[0][2], v[0][0]), __fmul_rn(2.f, __fsub_rn(v[1][2], v[1][0]))), __fsub_rn(v[2][2], v[2][0]));
    p.z = __fadd_rn(__fadd_rn(__fsub_rn(v[2][0], v[0][0]), __fmul_rn(2.f, __fsub_rn(v[2][1], v[0][1]))), __fsub_rn(v[2][2], v[0][2]));
    const float corners = __fadd_rn(__fadd_rn(__fadd_rn(v[0][0], v[0][2]), v[2][0]), v[2][2]);
    const float edges = __fadd_rn(__fadd_rn(__fadd_rn(v[0][1], v[1][0]), v[1][2]), v[2][1]);
    p.w = __fsub_rn(__fadd_rn(corners, __fmul_rn(2.f, edges)), __fmul_rn(12.f, v[1][1]));
    return p;
}

// Filter tap f at (i, j) (row dy = i - 1, column dx = j - 1), cross-correlation.
__host__ __device__ __forceinline__ constexpr float filter_tap(int f, int i, int j)
{
    return f == 0 ? (i == 1 && j == 1 ? 1.f : 0.f)
         : f == 1 ? (float)((j - 1) * (i == 1 ? 2 : 1))
         : f == 2 ? (float)((i - 1) * (j == 1 ? 2 : 1))
                  : (i == 1 && j == 1 ? -12.f : (i == 1 || j == 1) ? 2.f : 1.f);
}

__device__ __forceinline__ int wrap_index(int i, int n)
{
    i %= n;
    return i < 0 ? i + n : i;
}

// wrap_index for i at most one period outside [0, n) without a division (general i falls back to it).
__device__ __forceinline__ int wrap_near(int i, int n)
{
    if (i >= 0 && i < n)
        return i;
    if (i < 0 && i >= -n)
        return i + n;
    if (i >= n && i < 2 * n)
        return i - n;
    return wrap_index(i, n);
}

// ---------------------------------------------------------------- tile geometry
// A tile is R rows x S columns (R S <= 128) of one image: S = min(W, 128) columns, R = 128 / W rows when W <= 128
// (else one row of a 128-column strip). Compact tiles (growing NCAs, W >= 16): 8 rows x 16 columns, so that the tiles
// around a small living region are few (a growing grid is mostly dead, and dead tiles are skipped). Tile pixel i
// (0..127) is (i / S, i % S); tiles of an image are strips-fastest.
struct TileGeom {
    int H, W, S, R, strips, tiles_per_image;
};

__host__ __device__ inline TileGeom make_geom(int H, int W, bool compact = false)
{
    TileGeom g;
    g.H = H; g.W = W;
    g.S = compact && W >= 16 ? 16 : W <= 128 ? W : 128;
    g.R = compact && W >= 16 ? 8 : W <= 128 ? 128 / W : 1;
    g.strips = (W + g.S - 1) / g.S;
    g.tiles_per_image = g.strips * ((H + g.R - 1) / g.R);
    return g;
}

// The contiguous tile range [*a, *b) of persistent CTA c out of G over T tiles.
__host__ __device__ inline void cta_range(int64_t T, int G, int c, int64_t *a, int64_t *b)
{
    *a = T * c / G;  // T * G stays far below 2^63 for any grid that fits in device memory
    *b = T * (c + 1) / G;
}

// Cost-balanced bands of a row-kernel launch over T = N H image rows (images of H rows, NCAs of BH rows): CTA c gets
// rows [band_lo(c), band_lo(c + 1)), band_lo(c) = the last row u with cost(u) G <= c cost(T), where cost(u) = 4 u +
// s4 (image starts in (0, u)) + n4 (NCA starts in (0, u)) in quarter rows: a band that switches to another image
// inside costs its kernel s4 / 4 rows more (halo rows, pipeline drain and refill), one that switches to another NCA
// n4 / 4 rows more again (weights restaged). s4 = n4 = 0: the uniform split of cta_range.
struct Bands {
    int64_t T, H, BH;
    int G, s4, n4;
};
__host__ __device__ inline int64_t band_cost(const Bands &b, int64_t u)  // T < 2^31 rows: 32-bit divisions
{
    const uint32_t v = u > 0 ? (uint32_t)(u - 1) : 0u;
    return 4 * u + (u > 0 ? (int64_t)b.s4 * (v / (uint32_t)b.H) + (int64_t)b.n4 * (v / (uint32_t)b.BH) : 0);
}
__host__ __device__ inline int64_t band_lo(const Bands &b, int c)
{
    int64_t u = b.T * c / b.G;  // the uniform split; the balanced start lies within about (s4 + n4) / 4 rows of it
    if (b.s4 == 0 && b.n4 == 0)
        return u;
    const int64_t target = band_cost(b, b.T) * c;  // the last u with cost(u) G <= target (cost rises >= 4 per row)
    while (u > 0 && band_cost(b, u) * b.G > target)
        --u;
    while (u < b.T && band_cost(b, u + 1) * b.G <= target)
        ++u;
    return u;
}
__host__ __device__ inline void band_range(const Bands &b, int c, int64_t *lo, int64_t *hi)
{
    *lo = band_lo(b, c);
    *hi = band_lo(b, c + 1);
}

}  // namespace unca
