/*
 * CPU oracle for the stochastic update mask (TEST INFRASTRUCTURE ONLY: tests, smoke() and bench.py's CPU baseline may
 * load it; the product path never does).
 *
 * Restates, in plain C, the published Philox4x32-10 counter-based generator (Salmon, Moraes, Dror, Shaw, "Parallel
 * random numbers: as easy as 1, 2, 3", SC'11) as the reference uses it for the NCA update mask:
 *   - philox():        ncaops/nca_step.cuh:190-201 (key = seed as two 32-bit words, counter = (lo, hi, 0, 0),
 *                      multipliers 0xD2511F53 / 0xCD9E8D57, Weyl key bumps 0x9E3779B9 / 0xBB67AE85, 10 rounds);
 *   - mask_bit():      ncaops/nca_step.cuh:203-206, m = floorf(U + rate) != 0 with U = (word >> 8) * 2^-24;
 *   - mask_counter():  ncaops/nca_step.cuh:208-211, counter = (n H + Y) ceil(W / 4) + X / 4, word X % 4;
 *   - step_seed():     ncaops/nca_cuda.cu:157-164 (splitmix64 of the rollout seed and the step index).
 * Parity is pinned by the Random123 known-answer vectors for philox4x32-10 (tests/golden/philox_kat.json) and, on the
 * GPU box, bitwise against the reference's own mask_kernel compiled from its sources (oracle/_ref).
 */
#include <stdint.h>
#include <math.h>

static uint32_t mulhi32(uint32_t a, uint32_t b) { return (uint32_t)(((uint64_t)a * b) >> 32); }

/* out[0..3] = Philox4x32-10(counter = (c0, c1, c2, c3), key = (k0, k1)) */
void oracle_philox4x32_10(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3, uint32_t k0, uint32_t k1, uint32_t out[4])
{
    for (int r = 0; r < 10; ++r) {
        const uint32_t lo0 = 0xD2511F53u * c0, hi0 = mulhi32(0xD2511F53u, c0);
        const uint32_t lo1 = 0xCD9E8D57u * c2, hi1 = mulhi32(0xCD9E8D57u, c2);
        const uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
        c0 = n0; c1 = lo1; c2 = n2; c3 = lo0;
        k0 += 0x9E3779B9u; k1 += 0xBB67AE85u;
    }
    out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

uint64_t oracle_step_seed(uint64_t seed, uint64_t i)
{
    uint64_t z = seed + (i + 1) * 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

/* mask[(n - 0) H W + Y W + X] for images n_offset .. n_offset + n_images - 1 (global image index in the counter) */
void oracle_update_mask(float *mask, int64_t n_images, int64_t H, int64_t W, uint64_t seed, float update_rate,
                        int64_t n_offset)
{
    const uint32_t k0 = (uint32_t)seed, k1 = (uint32_t)(seed >> 32);
    const int64_t quads = (W + 3) / 4;
    for (int64_t n = 0; n < n_images; ++n)
        for (int64_t Y = 0; Y < H; ++Y)
            for (int64_t q = 0; q < quads; ++q) {
                const uint64_t counter = ((uint64_t)(n + n_offset) * (uint64_t)H + (uint64_t)Y) * (uint64_t)quads + (uint64_t)q;
                uint32_t w[4];
                oracle_philox4x32_10((uint32_t)counter, (uint32_t)(counter >> 32), 0u, 0u, k0, k1, w);
                for (int e = 0; e < 4; ++e) {
                    const int64_t X = 4 * q + e;
                    if (X >= W)
                        break;
                    /* float arithmetic exactly as written in the reference: product in fp32, then + rate, then floor */
                    const float u = (float)(w[e] >> 8) * (1.0f / 16777216.0f);
                    const float s = u + update_rate;
                    mask[(n * H + Y) * W + X] = floorf(s) != 0.f ? 1.f : 0.f;
                }
            }
}
