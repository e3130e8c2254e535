// Row-streaming step kernels (TF32, texture NCAs, W <= 128 and W % 4 == 0, or W a multiple of 128 as column strips):
// the hot path of the benchmark configs.
//
// A CTA owns a contiguous band of global rows of the N images (cost-balanced bands, Bands); one image row (or one
// 128-column strip of it) is one 128-lane MMA tile (lane = column). Rows of x (and, in the backward, gy) stream through shared-memory rings by
// bulk-async copies (the TMA engine), one row per channel per copy, completing on mbarriers; consecutive rows of a
// band share their neighbours, so every x row is read from HBM once per band.
//
// Forward (fwd_rows_kernel): per row, perception -> p' in TMEM, H = p' W1'^T (A from TMEM), relu(h) back into TMEM,
// U = relu(h) W2^T (A from TMEM), y = x + u m. NPART warpgroups split the per-pixel work (channels / hidden units).
//
// Backward (bwd_rows_kernel): per row as in bwd_kernel_tc, but the adjoint is fused: dp never leaves TMEM. Each
// row's dp is turned into its contributions to gx of rows y-1, y, y+1 (the filters are separable: a vertical
// weight per row times a horizontal transpose within the row, exchanged through shared memory), accumulated in
// registers, and gx of row y-1 is final once row y is done. A band is processed with one halo row on each side
// (dp only, no weight gradients, no gx of its own) so that its edge rows receive their neighbours' contributions.
// Transpose of the perception (ncaops/nca_step.cuh:1195-1263, reference adjoint_kernel):
//   gx(Y) += sum_i a_f[i] R_f(Y - i + 1),  R_f = horizontal transpose of dp_f within its row,
//   sobel_x: a = (1, 2, 1), b = (-1, 0, 1);  sobel_y: a = (-1, 0, 1), b = (1, 2, 1);  laplacian: s (x) s - 16 delta.
#pragma once
#include "nca_kernels.cuh"

namespace unca {

struct RowSeg {
    int n, r0, r1;  // image, owned rows [r0, r1)
};

// The next segment (rows of one image) of the global row range [g, gend); advances g.
__device__ __forceinline__ bool next_segment(int64_t &g, int64_t gend, int H, RowSeg &s)
{
    if (g >= gend)
        return false;
    s.n = (int)(g / H);
    s.r0 = (int)(g - (int64_t)s.n * H);
    const int64_t e = min(gend, (int64_t)(s.n + 1) * H);
    s.r1 = s.r0 + (int)(e - g);
    g = e;
    return true;
}

// Waits for ring entries [*waited, upto] (slot = entry % RING, parity bits in *par); false on timeout. Called by one
// thread; the barrier that follows publishes the data to the CTA.
template <int RING>
__device__ __forceinline__ bool ring_wait(uint64_t *full, int &waited, int upto, uint32_t &par)
{
    bool ok = true;
    while (waited <= upto) {
        const int slot = waited % RING;
        ok &= umma::mbar_wait(&full[slot], (par >> slot) & 1u);
        par ^= 1u << slot;
        ++waited;
    }
    return ok;
}

// Update mask of one image row (global image index n, row Y, W <= 128) by one warp: lane l draws the Philox block of
// pixels 4l .. 4l + 3 (one call per 4 pixels, as the counter layout intends) and writes mk[x] in {0, 1}.
template <class T>
__device__ __forceinline__ void row_mask_warp(T *mk, uint64_t seed, float rate, int64_t n, int H, int W, int Y, int lane)
{
    const int quads = (W + 3) / 4;
    if (rate >= 1.f) {
        for (int x = lane; x < W; x += 32)
            mk[x] = T(1);
        return;
    }
    if (lane < quads) {
        const uint64_t counter = ((uint64_t)n * (uint64_t)H + (uint64_t)Y) * (uint64_t)quads + (uint64_t)lane;
        const uint4 w = philox4x32_10(seed, counter);
        const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int x = 4 * lane + e;
            if (x < W)
                mk[x] = floorf(__fadd_rn(__fmul_rn((float)(words[e] >> 8), 1.0f / 16777216.0f), rate)) != 0.f ? T(1) : T(0);
        }
    }
}

// The same for the 128 pixels x0 .. x0 + 127 of a wider row (x0 % 4 == 0, x0 + 128 <= W): lane l draws the Philox
// block of pixels x0 + 4l .. x0 + 4l + 3 and writes mk[x - x0].
template <class T>
__device__ __forceinline__ void row_mask_strip_warp(T *mk, uint64_t seed, float rate, int64_t n, int H, int W, int Y,
                                                    int lane, int x0)
{
    if (rate >= 1.f) {
        for (int x = lane; x < 128; x += 32)
            mk[x] = T(1);
        return;
    }
    const uint64_t counter = ((uint64_t)n * (uint64_t)H + (uint64_t)Y) * (uint64_t)(W / 4) + (uint64_t)(x0 / 4 + lane);
    const uint4 w = philox4x32_10(seed, counter);
    const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int e = 0; e < 4; ++e)
        mk[4 * lane + e] = floorf(__fadd_rn(__fmul_rn((float)(words[e] >> 8), 1.0f / 16777216.0f), rate)) != 0.f ? T(1) : T(0);
}

// Named barrier `id` over `count` threads, and the same with an AND over `pred`.
__device__ __forceinline__ void bar_sync(int id, int count)
{
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}
__device__ __forceinline__ void bar_arrive(int id, int count)
{
    asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(count) : "memory");
}
__device__ __forceinline__ bool bar_and(int id, int count, bool pred)
{
    uint32_t r;
    asm volatile("{\n\t.reg .pred q, r;\n\tsetp.ne.u32 q, %1, 0;\n\tbar.red.and.pred r, %2, %3, q;\n\t"
                 "selp.u32 %0, 1, 0, r;\n\t}\n"
                 : "=r"(r)
                 : "r"((uint32_t)pred), "r"(id), "r"(count)
                 : "memory");
    return r != 0;
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar)
{
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}\n" ::"r"(umma::smem_u32(bar))
                 : "memory");
}

// Bounded mbarrier wait that gives up early once any warp of the CTA has given up (abort != 0), and sets abort when
// its own 2 s limit runs out: after a failure every warp keeps its loop and barrier sequence (so no named barrier is
// left short of a participant) while its remaining waits return at once. A phase that has already completed is
// reported as completed before abort is read (one shared load fewer on the common path).
__device__ __forceinline__ bool wait_bar(uint64_t *bar, uint32_t parity, volatile uint32_t *abort,
                                         uint64_t limit_ns = 2000000000ull)
{
    if (umma::mbar_try_wait(bar, parity))
        return true;
    if (*abort)
        return false;
    uint64_t t0;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    while (true) {
        if (umma::mbar_try_wait(bar, parity))
            return true;
        if (*abort)
            return false;
        uint64_t t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        if (t - t0 > limit_ns) {
            *abort = 1;
            return false;
        }
    }
}

// Failure-detection self-test of the bounded waits (one CTA of 64 threads): warp 0 holds a Tensor Memory allocation and
// waits on an mbarrier that nothing arrives on, with a limit of limit_ns; warp 1 waits on the same barrier with the
// kernels' 2 s limit and must return as soon as warp 0 has given up (the abort word). Both then take the kernels'
// teardown: Tensor Memory freed, the device error word set (code 1). out[0] / out[2]: nanoseconds warp 0 / warp 1
// waited; out[1] / out[3]: 1 if the wait of warp 0 / warp 1 reported success (it must not).
__global__ void __launch_bounds__(64, 1) wait_selftest_kernel(uint64_t limit_ns, unsigned long long *out)
{
    __shared__ uint64_t never;
    __shared__ uint32_t tslot;
    __shared__ uint32_t abort_word;
    volatile uint32_t *abort = &abort_word;
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    if (threadIdx.x == 0) {
        umma::mbar_init(&never, 1);
        *abort = 0;
        umma::fence_mbar_init();
    }
    if (warp == 0) {
        umma::tmem_alloc(&tslot, 32);
        umma::tmem_relinquish();
    }
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    uint64_t t0, t1;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    bool ok = true;
    if (lane == 0)
        ok = warp == 0 ? wait_bar(&never, 0, abort, limit_ns) : wait_bar(&never, 0, abort);
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t1));
    if (lane == 0) {
        out[2 * warp] = t1 - t0;
        out[2 * warp + 1] = ok ? 1ull : 0ull;
    }
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    if (warp == 0)
        umma::tmem_dealloc(tslot, 32);
    if (*abort && threadIdx.x == 0)
        set_device_error(1);
}

// Update mask of one image row (global image index n, row Y, W <= 128, W % 4 == 0) by one warp as 128 bits in four
// words: lane l draws the Philox block of pixels 4l .. 4l + 3 and word e collects, by ballot, bit l = mask(4l + e), so
// mask(x) = (word[x % 4] >> (x / 4)) & 1. Same draws and threshold as row_mask_warp.
__device__ __forceinline__ void row_mask_bits_warp(uint32_t *dst, uint64_t seed, float rate, int64_t n, int H, int W, int Y,
                                                   int lane)
{
    const int quads = W / 4;
    bool bits[4] = {false, false, false, false};
    if (lane < quads) {
        if (rate >= 1.f) {
            bits[0] = bits[1] = bits[2] = bits[3] = true;
        } else {
            const uint64_t counter = ((uint64_t)n * (uint64_t)H + (uint64_t)Y) * (uint64_t)quads + (uint64_t)lane;
            const uint4 w = philox4x32_10(seed, counter);
            const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int e = 0; e < 4; ++e)
                bits[e] = floorf(__fadd_rn(__fmul_rn((float)(words[e] >> 8), 1.0f / 16777216.0f), rate)) != 0.f;
        }
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const uint32_t word = __ballot_sync(~0u, bits[e]);
        if (lane == 0)
            dst[e] = word;
    }
}

// Weights of NCA k for the row kernels (TF32), as float4 items whose shared-memory address is linear in the item index:
//   W1s  (HID x KP, K-major chunk-planar: plane f/4 of HID rows x 4): w1 | b1_hi, b1_lo (the bias as two TF32 columns) | 0
//   W1T  (backward only; PIN x HID: plane j/4 of PIN rows x 4): w1 transposed
//   W2x  forward: W2s (CP x HID: plane j/4 of CP rows x 4), channels C..CP-1 zero;
//        backward: W2T (HID x CP: plane k/4 of HID rows x 4), channel c at k = c + gm_off, other k zero.
// Each thread loads a batch of items before it rounds and stores any (the loads of a batch are in flight together).
template <class D, bool BWD>
__device__ __forceinline__ void stage_rows_weights(float *W1s, float *W1T, float *W2x, const float *w1, const float *b1,
                                                   const float *w2, int t0, int nt, int gm_off)
{
    constexpr int Q = D::PIN / 4, N1 = (D::KP / 4) * D::HID;
    constexpr int N2 = BWD ? (D::HID / 4) * D::PIN : 0;
    constexpr int N3 = BWD ? (D::CP / 4) * D::HID : (D::HID / 4) * D::CP;
    constexpr int NT = N1 + N2 + N3, BATCH = 4;
    // rows of w1 (and, forward, of w2) as 16-byte loads where the base pointers allow: one load instruction instead of
    // four for the items whose lanes read 4 consecutive floats (the scattered rows keep the L1 busy per instruction)
    const bool v4 = ((reinterpret_cast<uintptr_t>(w1) | reinterpret_cast<uintptr_t>(w2)) & 15) == 0;
    for (int base = t0; base < NT; base += BATCH * nt) {
        float v[BATCH][4];
#pragma unroll
        for (int b = 0; b < BATCH; ++b) {
            const int it = base + b * nt;
#pragma unroll
            for (int t = 0; t < 4; ++t)
                v[b][t] = 0.f;
            if (it < N1) {
                const int q = it / D::HID, j = it % D::HID;
                if (q < Q) {
                    if (v4) {
                        const float4 f4 = __ldg(reinterpret_cast<const float4 *>(w1 + j * D::PIN + 4 * q));
                        v[b][0] = f4.x;
                        v[b][1] = f4.y;
                        v[b][2] = f4.z;
                        v[b][3] = f4.w;
                    } else {
#pragma unroll
                        for (int t = 0; t < 4; ++t)
                            v[b][t] = __ldg(w1 + j * D::PIN + 4 * q + t);
                    }
                } else if (q == Q) {
                    v[b][0] = __ldg(b1 + j);
                }
            } else if (it < N1 + N2) {
                const int r = (it - N1) / D::PIN, f = (it - N1) % D::PIN;
#pragma unroll
                for (int t = 0; t < 4; ++t)
                    v[b][t] = __ldg(w1 + (4 * r + t) * D::PIN + f);
            } else if (it < NT) {
                const int i3 = it - N1 - N2;
                if (BWD) {
                    const int pl = i3 / D::HID, j = i3 % D::HID;
#pragma unroll
                    for (int t = 0; t < 4; ++t) {
                        const int c = 4 * pl + t - gm_off;
                        if (c >= 0 && c < D::C)
                            v[b][t] = __ldg(w2 + c * D::HID + j);
                    }
                } else {
                    const int pl = i3 / D::CP, c = i3 % D::CP;
                    if (c < D::C) {
                        if (v4) {
                            const float4 f4 = __ldg(reinterpret_cast<const float4 *>(w2 + c * D::HID + 4 * pl));
                            v[b][0] = f4.x;
                            v[b][1] = f4.y;
                            v[b][2] = f4.z;
                            v[b][3] = f4.w;
                        } else {
#pragma unroll
                            for (int t = 0; t < 4; ++t)
                                v[b][t] = __ldg(w2 + c * D::HID + 4 * pl + t);
                        }
                    }
                }
            }
        }
#pragma unroll
        for (int b = 0; b < BATCH; ++b) {
            const int it = base + b * nt;
            if (it >= NT)
                continue;
            float4 o;
            if (it < N1 && it / D::HID == Q) {  // bias columns: b1_hi, b1_lo, 0, 0
                const float hi = tf32_rna(v[b][0]);
                o = make_float4(hi, tf32_rna(v[b][0] - hi), 0.f, 0.f);
            } else {
                o = make_float4(tf32_rna(v[b][0]), tf32_rna(v[b][1]), tf32_rna(v[b][2]), tf32_rna(v[b][3]));
            }
            float *dst = it < N1 ? W1s + (size_t)it * 4 : it < N1 + N2 ? W1T + (size_t)(it - N1) * 4
                                                                        : W2x + (size_t)(it - N1 - N2) * 4;
            *reinterpret_cast<float4 *>(dst) = o;
        }
    }
}

// ================================================================ forward
// Update mask of one image row (global image index n, row Y, W <= 128, W % 4 == 0) by one warp as 128 bits in x order:
// word w holds pixels 32 w .. 32 w + 31 (bit x % 32), so mask(x) = (word[x / 32] >> (x % 32)) & 1. Lane l draws the
// Philox block of pixels 4l .. 4l + 3 (the reference's counter layout, one call per 4 pixels) and the 4-bit groups of
// 8 lanes are merged by shuffles. Same draws and threshold as row_mask_warp.
__device__ __forceinline__ void row_mask_xorder_warp(uint32_t *dst, uint64_t seed, float rate, int64_t n, int H, int W,
                                                     int Y, int lane)
{
    const int quads = W / 4;
    uint32_t nib = 0;
    if (lane < quads) {
        if (rate >= 1.f) {
            nib = 0xFu;
        } else {
            const uint64_t counter = ((uint64_t)n * (uint64_t)H + (uint64_t)Y) * (uint64_t)quads + (uint64_t)lane;
            const uint4 w = philox4x32_10(seed, counter);
            const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int e = 0; e < 4; ++e)
                nib |= (floorf(__fadd_rn(__fmul_rn((float)(words[e] >> 8), 1.0f / 16777216.0f), rate)) != 0.f ? 1u : 0u)
                       << e;
        }
    }
    uint32_t v = nib << (4 * (lane & 7));
    v |= __shfl_xor_sync(~0u, v, 1);
    v |= __shfl_xor_sync(~0u, v, 2);
    v |= __shfl_xor_sync(~0u, v, 4);
    if ((lane & 7) == 0)
        dst[lane >> 3] = v;
}

// The same for the 128 pixels x0 .. x0 + 127 of a wider row (x0 % 128 == 0, x0 + 128 <= W): bit x - x0.
__device__ __forceinline__ void row_mask_xorder_strip_warp(uint32_t *dst, uint64_t seed, float rate, int64_t n, int H,
                                                           int W, int Y, int lane, int x0)
{
    uint32_t nib = 0xFu;
    if (rate < 1.f) {
        const uint64_t counter = ((uint64_t)n * (uint64_t)H + (uint64_t)Y) * (uint64_t)(W / 4) + (uint64_t)(x0 / 4 + lane);
        const uint4 w = philox4x32_10(seed, counter);
        const uint32_t words[4] = {w.x, w.y, w.z, w.w};
        nib = 0;
#pragma unroll
        for (int e = 0; e < 4; ++e)
            nib |= (floorf(__fadd_rn(__fmul_rn((float)(words[e] >> 8), 1.0f / 16777216.0f), rate)) != 0.f ? 1u : 0u) << e;
    }
    uint32_t v = nib << (4 * (lane & 7));
    v |= __shfl_xor_sync(~0u, v, 1);
    v |= __shfl_xor_sync(~0u, v, 2);
    v |= __shfl_xor_sync(~0u, v, 4);
    if ((lane & 7) == 0)
        dst[lane >> 3] = v;
}

// Position of the n-th (0-based) set bit of w (n < popc(w)).
__device__ __forceinline__ int nth_set_bit(uint32_t w, int n)
{
    int pos = 0, c = __popc(w & 0xFFFFu);
    if (n >= c) { n -= c; w >>= 16; pos += 16; }
    c = __popc(w & 0xFFu);
    if (n >= c) { n -= c; w >>= 8; pos += 8; }
    c = __popc(w & 0xFu);
    if (n >= c) { n -= c; w >>= 4; pos += 4; }
    c = __popc(w & 0x3u);
    if (n >= c) { n -= c; w >>= 2; pos += 2; }
    return pos + (n >= (int)(w & 1u) ? 1 : 0);
}

// Column of the n-th updating pixel of a row (x-order mask words m[0..3]).
__device__ __forceinline__ int nth_pixel(const uint32_t *m, int n)
{
    int w = 0;
#pragma unroll
    for (int i = 0; i < 3; ++i) {
        const int c = __popc(m[w]);
        if (n >= c) {
            n -= c;
            ++w;
        }
    }
    return 32 * w + nth_set_bit(m[w], n);
}

// Tile table of a CTA's row band [g0, g1), built by one warp (every lane calls it). Each segment of the band (the rows of
// one image; each of its S column strips in turn) is a sequence of L rows: its owned rows and, when halo = 1, one halo
// row on each side, whose 128-bit update masks MKX holds in sequence order. Writes CUM (per segment, the exclusive
// prefix counts of the updating pixels of its rows), TILE (per tile: queue start; count | first row << 8 | last row <<
// 20, rows segment-relative) and SEGT (per segment, the cumulative tile count).
template <int SPAN>
__device__ __forceinline__ void build_tile_table(const uint32_t *MKX, int *CUM, int2 *TILE, int *SEGT, int64_t g0,
                                                 int64_t g1, int H, int S, int halo, int lane32)
{
    int64_t g = g0;
    RowSeg sg;
    int s = 0, nt = 0, u0 = 0;
    while (next_segment(g, g1, H, sg))
      for (int strip = 0; strip < S; ++strip) {
        const int L = sg.r1 - sg.r0 + 2 * halo;
        int run = 0;
        for (int b = 0; b < L; b += 32) {
            const int j = b + lane32;
            int cnt = 0;
            if (j < L) {
                const uint32_t *m = MKX + (size_t)(u0 + j) * 4;
                cnt = __popc(m[0]) + __popc(m[1]) + __popc(m[2]) + __popc(m[3]);
            }
            int inc = cnt;
#pragma unroll
            for (int d = 1; d < 32; d <<= 1) {
                const int t = __shfl_up_sync(~0u, inc, d);
                if (lane32 >= d)
                    inc += t;
            }
            if (j < L)
                CUM[u0 + j] = run + inc - cnt;
            run += __shfl_sync(~0u, inc, 31);
        }
        __syncwarp();
        const int Q = run;
        // The tiles are the greedy cut of the queue: from q, up to 128 pixels, ending before the pixels of row
        // j(q) + SPAN, where j(p) is the row holding queue position p (the last row whose prefix count is <= p).
        // Usually no tile is cut short by the SPAN rule, and then the tiles are the fixed cut q = 128 t: every lane
        // builds one fixed tile (binary searches in the prefix counts) and checks the rule; only a segment where
        // some tile would be cut short takes the sequential greedy pass, which rewrites its entries.
        auto row_bs = [&](int p) {
            int lo = 0, hi = L - 1;
            while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if (CUM[u0 + mid] <= p)
                    lo = mid;
                else
                    hi = mid - 1;
            }
            return lo;
        };
        const int TF = (Q + 127) / 128;
        bool fixed = true;
        for (int t0 = 0; t0 < TF; t0 += 32) {
            const int t = t0 + lane32;
            bool fits = true;
            if (t < TF) {
                const int q = 128 * t, end = min(q + 128, Q);
                const int j = row_bs(q), jh = row_bs(end - 1);
                const int lim = j + SPAN < L ? CUM[u0 + j + SPAN] : Q;
                fits = lim >= end;
                TILE[nt + t] = make_int2(q, (end - q) | (j << 8) | (jh << 20));
            }
            fixed &= __all_sync(~0u, fits);
        }
        if (fixed) {
            nt += TF;
        } else {
            // greedy tiles, warp-parallel: lanes hold the prefix counts of a 64-row window [wb, wb + 64) (rows past
            // the segment: Q)
            auto cx = [&](int jj) { return jj < L ? CUM[u0 + jj] : Q; };
            int wb = 0, cw0 = cx(lane32), cw1 = cx(32 + lane32);
            auto row_of = [&](int p) {
                const uint32_t b0 = __ballot_sync(~0u, cw0 <= p), b1 = __ballot_sync(~0u, cw1 <= p);
                return wb + (b1 ? 63 - __clz(b1) : 31 - __clz(b0));
            };
            int q = 0;
            while (q < Q) {
                while (__shfl_sync(~0u, cw1, 0) <= q) {  // the tile's first row is past the window's first half
                    wb += 32;
                    cw0 = cw1;
                    cw1 = cx(wb + 32 + lane32);
                }
                const int j = row_of(q);  // in [wb, wb + 32): the tile's rows stay inside the window
                const int lim = __shfl_sync(~0u, j + SPAN - wb < 32 ? cw0 : cw1, (j + SPAN - wb) & 31);
                const int end = min(q + 128, lim), jh = row_of(end - 1);
                __syncwarp();
                if (lane32 == 0)
                    TILE[nt] = make_int2(q, (end - q) | (j << 8) | (jh << 20));
                ++nt;
                q = end;
            }
        }
        if (lane32 == 0)
            SEGT[s] = nt;
        __syncwarp();
        ++s;
        u0 += L;
    }
}

// Forward over the updating pixels only (the reference's forward also runs the MLP on the updating pixels alone,
// ncaops/nca_step.cuh:344-349): the pixels with m = 1 of a segment of rows, in row-major order, are cut into tiles of
// up to 128 (one MMA tile, lane = queue position) that span at most SPAN rows; the other pixels get y = x. Warps
// 0 .. 4 NPART - 1 compute (part p owns channels [CPP p, CPP (p+1)) and hidden units [HPP p, HPP (p+1)) of its lane's
// pixel); W_M1 issues MMA1 (h = [p' 1 1 0..] W1ext^T) and W_M2 issues MMA2 (u = relu(h) W2^T), from two different SM
// sub-partitions; W_PROD keeps an XRING-deep ring of x rows filled with bulk copies (one lane per channel), refilling
// a slot when every compute warp has released it. The prologue draws the update masks of all of the CTA's rows (at
// most MAXROWS rows per CTA; the grid grows beyond that) as 128-bit rows and builds the tile table (per segment:
// prefix counts of the rows, then tiles greedily). Per tile t each compute warp runs (the front end two tiles ahead)
//   EPI(t)  [MMA1(t)]        h -> tf32(relu(h)) in TMEM H[t%2]                                       -> epi_done
//   FE(t+2) [x rows]         lane -> (row, column) of its pixel; p' -> TMEM P[t%2]; centre x kept     -> fe_done[t%2]
//           then the ring entries no later front end reads are retired: the non-updating pixels of their rows are
//           copied (y = x) and the slots released
//   OUT(t)  [MMA2(t)]        y = x + u at the lane's pixel
// MMA1, MMA2 and the front-end signals use one mbarrier per buffer parity, so that no waiter can see a phase of the
// tile two ahead in place of its own. A tile's rows and the front end's lag keep at most SPAN + 2 ring entries live.
// STRIP: rows wider than one tile (W = 128 S, S >= 2) run as S column strips of 128 per segment ("passes": the
// rows of a segment at the strip's columns; masks, prefix counts and tiles per pass), with ring rows of XS = 136
// floats (4 halo columns on each side of the strip). MAXROWS then counts rows times strips.
template <int C, int HID, int NPART, bool STRIP = false>
struct FwdRows {
    using D = Dims<C, HID>;
    static constexpr int CW = 128 * NPART, W_M1 = CW / 32, W_M2 = W_M1 + 1, W_PROD = W_M1 + 2;
    static constexpr int THREADS = CW + 96, CPP = C / NPART, HPP = HID / NPART, XRING = 8, SPAN = 4;
    static constexpr int MAXROWS = STRIP ? 4096 : 1024, XS = STRIP ? 136 : 128;
    // TMEM: H[2] (h, then tf32(relu(h)) in place), U[2], P[2] (p'; 1, 1 at PIN, PIN+1; zeros to KP)
    static constexpr int T_H0 = 0, T_H1 = HID, T_U0 = 2 * HID, T_U1 = 2 * HID + 32, T_P0 = 256, T_P1 = 320;
    static constexpr int TMEM = 512;
    static_assert(C % NPART == 0 && HPP % 8 == 0 && D::KP <= 64 && T_U1 + 16 <= T_P0 && HID % 32 == 0 &&
                  D::CP == 16 && C <= 32 && (XRING & (XRING - 1)) == 0 && XRING >= SPAN + 3, "forward row-kernel layout");
    // shared memory: W1 (K-major, bias folded) | W2 | x ring | masks (4 words per row) | prefix counts (per row) |
    // tiles (int2 per tile: queue start; count | first row << 8 | last row << 20) | tiles per segment (cumulative) |
    // mbarriers
    static constexpr size_t OFF_XR = (size_t)(D::W1S + D::W2S) * 4;
    static constexpr size_t OFF_MK = OFF_XR + (size_t)XRING * C * XS * 4;
    static constexpr size_t OFF_CUM = OFF_MK + (size_t)MAXROWS * 16;
    static constexpr size_t OFF_TILE = OFF_CUM + (size_t)MAXROWS * 4;
    static constexpr size_t OFF_SEGT = OFF_TILE + (size_t)MAXROWS * 8;
    static constexpr size_t OFF_BAR = OFF_SEGT + (size_t)MAXROWS * 4;
    static constexpr int NBAR = 2 * XRING + 7;  // x ring full / empty, MMA1, MMA2, fe_done per buffer, epi_done
    static constexpr size_t smem() { return OFF_BAR + 8 * NBAR + 16; }
    static_assert(OFF_BAR % 8 == 0 && OFF_TILE % 8 == 0, "alignment");
    static_assert(smem() <= 232448, "227 KB of shared memory per CTA");
};

template <int C, int HID, int NPART, bool STRIP = false>
__global__ void __maxnreg__(128) fwd_rows_kernel(StepArgs a)
{
    using F = FwdRows<C, HID, NPART, STRIP>;
    using D = typename F::D;
    // the next step's kernel may launch now (it waits for this one before reading the state it writes)
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    extern __shared__ __align__(128) unsigned char smem_raw[];
    float *W1s = reinterpret_cast<float *>(smem_raw), *W2s = W1s + D::W1S;
    float *XR = reinterpret_cast<float *>(smem_raw + F::OFF_XR);
    uint32_t *MKX = reinterpret_cast<uint32_t *>(smem_raw + F::OFF_MK);
    int *CUM = reinterpret_cast<int *>(smem_raw + F::OFF_CUM), *SEGT = reinterpret_cast<int *>(smem_raw + F::OFF_SEGT);
    int2 *TILE = reinterpret_cast<int2 *>(smem_raw + F::OFF_TILE);
    uint64_t *xfull = reinterpret_cast<uint64_t *>(smem_raw + F::OFF_BAR), *xempty = xfull + F::XRING,
             *g1bar = xempty + F::XRING, *g2bar = g1bar + 2, *fe_done = g2bar + 2, *epi_done = fe_done + 2;
    uint32_t *tslot = reinterpret_cast<uint32_t *>(epi_done + 1);
    volatile uint32_t *abort = tslot + 1;

    const int tid = threadIdx.x, warp = tid / 32, lane32 = tid % 32;
    const bool compute = warp < F::W_M1, m1 = warp == F::W_M1, m2 = warp == F::W_M2, prod = warp == F::W_PROD;
    const int part = compute ? tid / 128 : 0, x = tid % 128;
    const int H = a.H, W = a.W;
    const int S = STRIP ? W / 128 : 1;  // column strips per row
    const int RS = STRIP ? F::XS : W;   // ring row stride
    const size_t plane = (size_t)H * W;
    __shared__ int64_t band[2];  // this CTA's rows [g0, g1), found by thread 0
    __shared__ uint64_t seed_sh; // the step's mask seed (a device read when the seed lives on the device)

    if (tid == 0) {
        const uint64_t sd = step_seed_of(a);  // in flight while the band is found and the mbarriers initialised
        band_range(row_bands(a, gridDim.x), blockIdx.x, &band[0], &band[1]);
        for (int i = 0; i < 2 * F::XRING; ++i)
            umma::mbar_init(&xfull[i], i < F::XRING ? 1 : F::W_M1);  // full: the copy bytes; empty: every compute warp
        for (int b2 = 0; b2 < 2; ++b2) {
            umma::mbar_init(&g1bar[b2], 1);
            umma::mbar_init(&g2bar[b2], 1);
            umma::mbar_init(&fe_done[b2], F::W_M1);
        }
        umma::mbar_init(epi_done, F::W_M1);
        *abort = 0;
        umma::fence_mbar_init();
        seed_sh = sd;
    }
    __syncthreads();
    const int64_t g0 = band[0], g1 = band[1];
    if ((g1 - g0) * S > F::MAXROWS) {  // the host sizes the grid so that this never happens: refuse rather than overflow
        if (tid == 0)
            set_device_error(2);
        return;
    }
    // Set-up, in two phases whose parts run on different warps (this set-up is the part of a step a launch cannot hide
    // under the previous step's tail on the SMs that previous step frees last):
    //   1. warp 0 allocates the Tensor Memory; warps 1.. draw the update masks of the CTA's rows;
    //   2. warp 0 builds the tile table; warps 1.. stage the first NCA's weights.
    const int nrows = (int)(g1 - g0);  // <= MAXROWS / S (the host sizes the grid so)
    const int64_t n0 = g0 / H;         // the band's first image and row
    const int r0 = (int)(g0 - n0 * H), nw = blockDim.x / 32;
    // EARLY_X (one tile per row): the producer takes no part in the set-up; it waits for the previous kernel at once and
    // copies the first segment's first ring entries, which land while the others build the tables and stage the
    // weights (on the SMs the previous step frees last, that wait is already over). The set-up's barriers are then
    // named barrier 1 over the other warps.
    constexpr bool EARLY_X = !STRIP;
    const int nset = EARLY_X ? nw - 1 : nw;  // warps of the set-up
    auto setup_sync = [&]() {
        if (EARLY_X)
            bar_sync(1, 32 * nset);
        else
            __syncthreads();
    };
    int x_pre = 0;  // producer: ring entries of the first segment copied during the set-up
    if (EARLY_X && prod) {
        if (nrows > 0) {
            asm volatile("griddepcontrol.wait;" ::: "memory");
            int64_t gg = g0;
            RowSeg sg0;
            next_segment(gg, g1, H, sg0);
            const float *xn0 = a.x + (size_t)sg0.n * C * plane;
            x_pre = min(F::XRING, sg0.r1 - sg0.r0 + 2);
            for (int e = 0; e < x_pre; ++e) {
                if (lane32 == 0)
                    umma::mbar_arrive_expect_tx(&xfull[e], (uint32_t)(C * W * 4));
                __syncwarp();
                if (lane32 < C)
                    umma::bulk_g2s(XR + ((size_t)e * C + lane32) * W,
                                   xn0 + ((size_t)lane32 * H + wrap_near(sg0.r0 - 1 + e, H)) * W, (uint32_t)(W * 4),
                                   &xfull[e]);
            }
        }
    } else if (warp == 0) {
        umma::tmem_alloc(tslot, F::TMEM);
        umma::tmem_relinquish();
    } else {
        const uint64_t seed = seed_sh;
        for (int rel = warp - 1; rel < nrows; rel += nset - 1) {
            const int yy = r0 + rel, dn = yy / H, Y = yy - dn * H;
            if (!STRIP) {
                row_mask_xorder_warp(MKX + (size_t)rel * 4, seed, a.rate, n0 + dn + a.n_offset, H, W, Y, lane32);
            } else {
                // pass-major: row rel of the segment [lo, hi) (CTA-relative) at strip s is mask row S lo + s (hi - lo) +
                // rel - lo
                const int lo = max(0, dn * H - r0), hi = min(nrows, (dn + 1) * H - r0);
                for (int s = 0; s < S; ++s)
                    row_mask_xorder_strip_warp(MKX + (size_t)(S * lo + s * (hi - lo) + (rel - lo)) * 4, seed, a.rate,
                                               n0 + dn + a.n_offset, H, W, Y, lane32, 128 * s);
            }
        }
    }
    if (!(EARLY_X && prod))
        setup_sync();
    int cur_k = -1;
    if (EARLY_X && prod) {
    } else if (warp == 0) {  // tile table: tiles of <= 128 updating pixels over <= SPAN rows
        build_tile_table<F::SPAN>(MKX, CUM, TILE, SEGT, g0, g1, H, S, 0, lane32);
    } else if (nrows > 0) {  // the first segment's NCA: its weights, by warps 1 .. nset - 1
        const int k = (int)(n0 / a.B);
        stage_rows_weights<D, false>(W1s, nullptr, W2s, a.w1 + (size_t)k * HID * D::PIN, a.b1 + (size_t)k * HID,
                                     a.w2 + (size_t)k * C * HID, tid - 32, 32 * (nset - 1), 0);
        umma::fence_proxy_async();
    }
    if (nrows > 0)
        cur_k = (int)(n0 / a.B);
    uint32_t tmem = 0, lane = 0;  // (the producer uses no Tensor Memory)
    if (!(EARLY_X && prod)) {
        tmem = *tslot;
        lane = umma::tmem_addr(tmem, warp, 0);
    }
    if (compute && part == 0) {  // p' columns past the channel features: bias-hi, bias-lo = 1, zeros (never overwritten)
        const float v[8] = {1.f, 1.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        umma::tmem_st8(lane + F::T_P0 + D::PIN, v);
        umma::tmem_st8(lane + F::T_P1 + D::PIN, v);
        umma::tmem_wait_st();
    }
    if (!(EARLY_X && prod)) {
        umma::fence_before_sync();
        setup_sync();
        umma::fence_after_sync();
    }

    const uint64_t dW1 = umma::smem_desc(umma::smem_u32(W1s), HID * 16, 128);
    const uint64_t dW2 = umma::smem_desc(umma::smem_u32(W2s), D::CP * 16, 128);
    constexpr uint32_t I1 = umma::idesc_tf32(128, HID, false, false), I2 = umma::idesc_tf32(128, 16, false, false);
    constexpr int JM = STRIP ? 0xFFF : 0x3FF;  // row fields of a tile entry
    bool ok = true;
    uint32_t epar = 0, g1par = 0, g2par = 0, eph = 0, fepar = 0;  // *par: one parity bit per buffer / ring slot
    int x_uses[F::XRING] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int e = 0; e < x_pre; ++e)  // producer: the entries copied during the set-up
        x_uses[e] = 1;
    uint64_t *last_bar = nullptr;
    uint32_t last_par = 0;
    auto wait_par = [&](uint64_t *bars, uint32_t &par, int bj) {  // the next phase of bars[bj]
        ok &= wait_bar(&bars[bj], (par >> bj) & 1u, abort);
        par ^= 1u << bj;
    };
    auto wait_g2 = [&](int bj) { wait_par(g2bar, g2par, bj); };  // MMA2 into U[bj] complete
    auto signal = [&](uint64_t *bar) {  // this warp's TMEM / shared-memory reads and writes are complete
        umma::fence_before_sync();
        __syncwarp();
        if (lane32 == 0)
            mbar_arrive(bar);
    };

    int64_t g = g0;
    RowSeg sg;
    int seg = 0, u0 = 0, ebase = 0;  // segment ordinal, its first row (CTA-relative), ring entries of earlier segments
    bool dep_waited = false;
    while (next_segment(g, g1, H, sg))
      for (int s = 0; s < S; ++s) {  // the column strips of the segment, one pass each (one pass unless STRIP)
        const int n = sg.n, k = n / a.B, L = sg.r1 - sg.r0, c0 = 128 * s;
        const int tb = seg == 0 ? 0 : SEGT[seg - 1], T = SEGT[seg] - tb;
        const float *xn = a.x + (size_t)n * C * plane;
        float *yn = a.y + (size_t)n * C * plane;
        if (k != cur_k) {  // every warp finished the previous segment (and its MMAs completed): restage the weights
            umma::fence_before_sync();
            __syncthreads();
            stage_rows_weights<D, false>(W1s, nullptr, W2s, a.w1 + (size_t)k * HID * D::PIN, a.b1 + (size_t)k * HID,
                                         a.w2 + (size_t)k * C * HID, tid, blockDim.x, 0);
            umma::fence_proxy_async();
            __syncthreads();
            umma::fence_after_sync();
            cur_k = k;
        }
        if (!dep_waited) {  // set-up done: wait for the previous step's kernel (launched as its programmatic
            asm volatile("griddepcontrol.wait;" ::: "memory");  // dependent) before reading x, which it wrote
            dep_waited = true;
        }
        if (prod) {
            // ======== producer: x row wrap(r0 - 1 + e) -> slot (ebase + e) % XRING, e = 0 .. L + 1; lane c copies
            // channel c (a starved single lane issuing all of them falls behind the compute warps)
            for (int e = seg == 0 && s == 0 ? x_pre : 0; e < L + 2; ++e) {
                const int slot = (ebase + e) & (F::XRING - 1);
                if (lane32 == 0 && x_uses[slot] > 0)  // every compute warp released the slot's previous row
                    ok &= wait_bar(&xempty[slot], (uint32_t)((x_uses[slot] - 1) & 1), abort);
                ++x_uses[slot];
                ok = __shfl_sync(~0u, ok, 0);
                if (ok) {
                    const int Y = wrap_near(sg.r0 - 1 + e, H);
                    if (lane32 == 0)
                        umma::mbar_arrive_expect_tx(&xfull[slot], (uint32_t)(C * RS * 4));
                    __syncwarp();
                    if (!STRIP) {
                        if (lane32 < C)
                            umma::bulk_g2s(XR + ((size_t)slot * C + lane32) * W, xn + ((size_t)lane32 * H + Y) * W,
                                           (uint32_t)(W * 4), &xfull[slot]);
                    } else if (lane32 < C) {
                        // columns c0 - 4 .. c0 + 131 (circular) -> ring columns 0 .. 135, one piece or two where the
                        // range wraps (16-byte aligned: W and c0 are multiples of 128)
                        float *dst = XR + ((size_t)slot * C + lane32) * RS;
                        const float *src = xn + ((size_t)lane32 * H + Y) * W;
                        if (s == 0) {
                            umma::bulk_g2s(dst, src + W - 4, 16u, &xfull[slot]);
                            umma::bulk_g2s(dst + 4, src, 132u * 4u, &xfull[slot]);
                        } else if (s == S - 1) {
                            umma::bulk_g2s(dst, src + c0 - 4, 132u * 4u, &xfull[slot]);
                            umma::bulk_g2s(dst + 132, src, 16u, &xfull[slot]);
                        } else {
                            umma::bulk_g2s(dst, src + c0 - 4, 136u * 4u, &xfull[slot]);
                        }
                    }
                }
            }
        } else if (m1) {
            // ======== MMA1 warp: h of tile j -> H[j % 2] once FE(j) is done and MMA2(j-2) no longer reads H
            if (lane32 == 0) {
                for (int j = 0; j < T; ++j) {
                    const int bj = j & 1;
                    wait_par(fe_done, fepar, bj);
                    if (j >= 2)  // MMA2(j-2) read H[bj]
                        wait_g2(bj);
                    if (ok) {
                        umma::fence_after_sync();
                        const uint32_t tp = tmem + (bj ? F::T_P1 : F::T_P0), th = tmem + (bj ? F::T_H1 : F::T_H0);
#pragma unroll
                        for (int ks = 0; ks < D::KP / 8; ++ks)
                            umma::mma_ts(th, tp + ks * 8, dW1 + (uint64_t)(ks * 2 * HID), I1, ks > 0);
                        umma::commit(&g1bar[bj]);
                        last_bar = &g1bar[bj];
                        last_par = (g1par >> bj) & 1u;  // this warp counts its own commits per H buffer
                        g1par ^= 1u << bj;
                    }
                }
                for (int j = (T >= 2 ? T - 2 : 0); j < T; ++j)  // MMA2 of the last two tiles: every phase waited once
                    wait_g2(j & 1);
            }
        } else if (m2) {
            // ======== MMA2 warp: u of tile i -> U[i % 2] once EPI(i) is done
            if (lane32 == 0) {
                for (int i = 0; i < T; ++i) {
                    const int b = i & 1;
                    ok &= wait_bar(epi_done, eph, abort);
                    eph ^= 1;
                    if (ok) {
                        umma::fence_after_sync();
                        const uint32_t th = tmem + (b ? F::T_H1 : F::T_H0), tu = tmem + (b ? F::T_U1 : F::T_U0);
#pragma unroll
                        for (int ks = 0; ks < HID / 8; ++ks)
                            umma::mma_ts(tu, th + ks * 8, dW2 + (uint64_t)(ks * 2 * D::CP), I2, ks > 0);
                        umma::commit(&g2bar[b]);
                        last_bar = &g2bar[b];
                        last_par = (g2par >> b) & 1u;  // this warp counts its own commits per U buffer
                        g2par ^= 1u << b;
                    }
                }
            }
        } else if (compute) {
            // ======== compute warps
            float xcur[F::CPP], xn1[F::CPP], xnext[F::CPP];
            int pcur = -1, pn1 = -1, pnext = -1;  // the lane's pixel of a tile (row << 8 | column), -1: no pixel
            int ewaited = 0, released = 0;        // ring entries of this segment waited for / released
            const uint32_t *mseg = MKX + (size_t)u0 * 4;
            auto slot_of = [&](int e) { return (ebase + e) & (F::XRING - 1); };
            auto wait_entries = [&](int upto) {  // ring entries .. upto landed
                while (ewaited <= upto) {
                    const int slot = slot_of(ewaited);
                    ok &= wait_bar(&xfull[slot], (epar >> slot) & 1u, abort);
                    epar ^= 1u << slot;
                    ++ewaited;
                }
            };
            // release ring entries < target (no later front end reads them), copying y = x at the non-updating pixels
            // of the owned row each one holds first
            auto retire = [&](int target) {
                for (; released < target; ++released) {
                    const int e = released, j = e - 1;
                    wait_entries(e);
                    if (j >= 0 && j < L && (STRIP || x < W) && ok) {
                        const float *src = XR + (size_t)slot_of(e) * C * RS + (STRIP ? x + 4 : x);
                        float *dst = yn + (size_t)(sg.r0 + j) * W + c0 + x;
                        if (!((mseg[j * 4 + (x >> 5)] >> (x & 31)) & 1u)) {
#pragma unroll
                            for (int cc = 0; cc < F::CPP; ++cc) {
                                const int c = F::CPP * part + cc;
                                dst[(size_t)c * plane] = src[(size_t)c * RS];
                            }
                        }
                    }
                    signal(&xempty[slot_of(e)]);
                }
            };
            auto front_end = [&](int t, int bj) {  // p' of tile t's pixels -> P[bj]; centre x and pixel kept
                const int2 tl = TILE[tb + t];
                const int nq = tl.y & 0xFF, jlo = (tl.y >> 8) & JM, jhi = (tl.y >> 20) & JM;
                wait_entries(jhi + 2);  // rows Y - 1 .. Y + 1 of the tile's rows
                const bool valid = x < nq;
                const int q = tl.x + (valid ? x : 0);
                int j = jlo;
                while (j < jhi && CUM[u0 + j + 1] <= q)
                    ++j;
                const int px = nth_pixel(mseg + j * 4, q - CUM[u0 + j]);
                // the pixel's left, centre and right columns in a ring row (STRIP: 4 halo columns precede the strip)
                const int pl = STRIP ? px + 3 : px == 0 ? W - 1 : px - 1, pc = STRIP ? px + 4 : px,
                          pr = STRIP ? px + 5 : px + 1 >= W ? 0 : px + 1;
                const float *rm = XR + (size_t)slot_of(j) * C * RS, *r0 = XR + (size_t)slot_of(j + 1) * C * RS,
                            *rp = XR + (size_t)slot_of(j + 2) * C * RS;
                const uint32_t tp = lane + (bj ? F::T_P1 : F::T_P0);
#pragma unroll
                for (int cc = 0; cc < F::CPP; ++cc) {  // warp-uniform channel: tcgen05.st takes one column per warp
                    const int c = F::CPP * part + cc;
                    const float *bm = rm + c * RS, *b0 = r0 + c * RS, *bp = rp + c * RS;
                    const float v[3][3] = {{bm[pl], bm[pc], bm[pr]}, {b0[pl], b0[pc], b0[pr]}, {bp[pl], bp[pc], bp[pr]}};
                    const float4 p = perceive3x3(v);
                    const float pv[4] = {tf32_bias(p.x), tf32_bias(p.y), tf32_bias(p.z), tf32_bias(p.w)};
                    umma::tmem_st4(tp + 4 * c, pv);
                    xnext[cc] = v[1][1];
                }
                pnext = valid ? (((sg.r0 + j) << 8) | px) : -1;
                umma::tmem_wait_st();
                signal(&fe_done[bj]);
                retire(t + 1 < T ? ((TILE[tb + t + 1].y >> 8) & JM) : L + 2);
            };
            if (T > 0) {
                front_end(0, 0);
#pragma unroll
                for (int cc = 0; cc < F::CPP; ++cc)
                    xn1[cc] = xnext[cc];
                pn1 = pnext;
                if (T > 1)
                    front_end(1, 1);
            } else {
                retire(L + 2);  // no updating pixel: y = x everywhere
            }
            for (int i = 0; i < T; ++i) {
                const int b = i & 1;
#pragma unroll
                for (int cc = 0; cc < F::CPP; ++cc) {  // tiles i, i + 1 (front end done): xcur, xn1
                    xcur[cc] = xn1[cc];
                    xn1[cc] = xnext[cc];
                }
                pcur = pn1;
                pn1 = pnext;
                // ---- EPI(i): h -> tf32(relu(h)) in place
                wait_par(g1bar, g1par, b);
                umma::fence_after_sync();
                const uint32_t th = lane + (b ? F::T_H1 : F::T_H0) + part * F::HPP;
#pragma unroll
                for (int q = 0; q < F::HPP / 8; ++q) {
                    float h[8];
                    umma::tmem_ld8(th + q * 8, h);
                    umma::tmem_wait_ld();
#pragma unroll
                    for (int e = 0; e < 8; ++e)
                        h[e] = tf32_bias(fmaxf(h[e], 0.f));
                    umma::tmem_st8(th + q * 8, h);
                }
                umma::tmem_wait_st();
                signal(epi_done);
                // ---- FE(i+2)
                if (i + 2 < T)
                    front_end(i + 2, b);
                // ---- OUT(i): y = x + u at the lane's pixel
                wait_g2(b);
                umma::fence_after_sync();
                const uint32_t tu = lane + (b ? F::T_U1 : F::T_U0) + F::CPP * part;
                float u[F::CPP];
#pragma unroll
                for (int cc = 0; cc < F::CPP; ++cc)
                    u[cc] = umma::tmem_ld1(tu + cc);
                umma::tmem_wait_ld();  // the loaded registers are defined only after this wait
                if (pcur >= 0 && ok) {
                    float *yr = yn + (size_t)(pcur >> 8) * W + c0 + (pcur & 0xFF);
#pragma unroll
                    for (int cc = 0; cc < F::CPP; ++cc)
                        yr[(size_t)(F::CPP * part + cc) * plane] = xcur[cc] + u[cc];
                }
            }
        }
        ebase += L + 2;
        u0 += L;
        ++seg;
    }
    if ((m1 || m2) && lane32 == 0 && last_bar != nullptr)  // this warp's MMAs are complete before the teardown
        umma::mbar_wait(last_bar, last_par);
    if (prod && lane32 == 0)  // and so are this warp's bulk copies
        for (int s2 = 0; s2 < F::XRING; ++s2)
            if (x_uses[s2] > 0)
                umma::mbar_wait(&xfull[s2], (uint32_t)((x_uses[s2] - 1) & 1));
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    if (warp == 0)
        umma::tmem_dealloc(tmem, F::TMEM);
    if ((*abort || !ok) && tid == 0)
        set_device_error(1);
}

// ================================================================ backward with the fused adjoint
// Eight consecutive values v[0..7] of MN index mn0 (mn0 % 8 == 0) at K row k of a swizzled MN-major tile, as two
// 16-byte stores whose order alternates with bit 2 of k: a warp's 32 rows then cover all eight 16-byte bank slots of a
// 128-byte row four times per instruction (the minimum of 4 wavefronts; one fixed order costs 8).
__device__ __forceinline__ void st_sw32x8_balanced(float *tile, int mn0, int k, int krows, const float *v)
{
    float *dst = tile + umma::sw32_offset(mn0, k, krows) / 4;
    const int flip = (k >> 2) & 1;
    const float4 lo = make_float4(v[0], v[1], v[2], v[3]), hi = make_float4(v[4], v[5], v[6], v[7]);
    *reinterpret_cast<float4 *>(dst + 4 * flip) = flip ? hi : lo;
    *reinterpret_cast<float4 *>(dst + 4 * (1 - flip)) = flip ? lo : hi;
}

// Backward, software-pipelined across rows, with the warps synchronised by mbarriers only (no CTA-wide barrier per
// row). Warps 0 .. 4 NPART - 1 compute (NPART parts of 4 warps: part p owns channels [CPP p, CPP (p+1)) and hidden
// units [HPP p, HPP (p+1)) of pixel x = its TMEM lane); warp W_MMA issues G1 (h = p' W1^T, dhp = W2^T gm) and DP
// (dp = dh W1); warp W_PROD issues the bulk copies of x rows (one lane per channel) and draws the update masks two
// rows ahead; warp W_WG issues the weight-gradient group WG. Per row i of the band
// sequence (halo, owned rows, halo), each compute warp runs
//   EA(i)   [G1(i), WG(i-1)]   relu(h) -> RH, dh -> DH (owned rows, swizzled smem) and TMEM H   -> ea_done
//   FE(i+1) [x rows, mask]     p', gm -> TMEM P[(i+1)%2] and PSW[(i+1)%2]                      -> fe_done
//   ADJ(i)  [DP(i)]            dp(i) -> adjoint (edge lanes exchanged per part) -> gx(Y_{i-1}) final
// while the MMA warp issues DP(i) after ea_done(i) (then lets WG(i) start) and G1(i+1) after fe_done(i+1) and DP(i),
// and the producer, after fe_done(j), refills the x slot of row j and draws the mask of row j + 2.
// WG is one chain of M = 128 (features of PSW: p' 0..PIN-1, the constant 1 at PIN, gm at GM0..GM0+C-1), N = 2 HID
// (relu(h) | dh), K = 128 pixels: columns [0, HID) of rows GM0.. hold dW2, columns [HID, 2 HID) of rows 0..PIN hold
// dW1 and db1 (transposed); the other blocks are not used.
// STRIP: rows wider than one tile (W = 128 S, S >= 2) are processed as S column strips of 128, one after the other
// over the rows of a segment. A strip's x rows carry 4 halo columns on each side (ring rows of XS = 136 floats); the
// adjoint treats the columns next to a strip as zero and publishes the strip's first and last columns of dp for every
// owned row to the edge scratch, from which strip_edge_fixup_kernel adds the cross-strip terms.
template <int C, int HID, int NPART, bool STRIP = false>
struct BwdRows {
    using D = Dims<C, HID>;
    static constexpr int CW = 128 * NPART, W_MMA = CW / 32, W_PROD = W_MMA + 1, W_WG = W_MMA + 2;
    static constexpr int THREADS = CW + 96, GROUP = CW + 64;  // GROUP: the warps on named barrier 1 (all but W_WG)
    static constexpr int CPP = C / NPART, HPP = HID / NPART, XRING = 3, GM0 = D::PIN + 2;
    static constexpr int XS = STRIP ? 136 : 128;  // ring row stride (floats)
    // TMEM: h / dh, dhp, WG accumulator, P[2] (p' 0..PIN-1 then dp; 1, 1 at PIN, PIN+1; gm at GM0..; zeros)
    static constexpr int T_H = 0, T_DHP = HID, T_ACC = 2 * HID, NACC = 2 * HID, T_P0 = T_ACC + NACC, T_P1 = T_P0 + 64;
    static constexpr int TMEM = 512;
    static_assert(C % NPART == 0 && C <= 16 && HPP % 8 == 0 && D::KP == 56 && GM0 + C <= 62 && T_P1 + 64 <= TMEM &&
                  HID % 32 == 0 && NACC <= 256 && D::NPW == 64, "backward row-kernel layout");
    // shared memory, 1024-aligned base: weights | PSW[2] | RH | DH (swizzled MN-major) | XR | EDGE | MK[2] | bars
    // (WG reads 4 MN blocks of PSW[b] for M = 128: for b = 1 the last two are RH, in bounds and unused)
    static constexpr size_t OFF_PSW = (size_t)D::BWD_W;
    static constexpr size_t OFF_RH = OFF_PSW + (size_t)2 * D::PSW * 4;
    static constexpr size_t OFF_XR = OFF_RH + (size_t)2 * D::RHDH * 4;
    static constexpr size_t OFF_EDGE = OFF_XR + (size_t)XRING * C * XS * 4;
    // left / right edge lane of each of the 4 warps of a part, and (not STRIP) x = W - 1
    // (one buffer: row i + 1's edges are written only after every warp finished row i's adjoint, since DP(i + 1)
    // follows every warp's EA(i + 1))
    static constexpr int EDGE_SLOTS = STRIP ? 8 : 9;
    static constexpr size_t OFF_MK = OFF_EDGE + (size_t)EDGE_SLOTS * C * 16;
    static constexpr size_t OFF_BAR = OFF_MK + 2 * 128;
    // x ring, mask buffers, g1, dp, wg (tensor-core completions), wg_go, ea_done, fe_done (one arrival per warp)
    static constexpr int NBAR = XRING + 8;
    // then the TMEM slot and abort words (8 bytes) and the step's mask seed (8 bytes)
    static constexpr size_t OFF_SEED = OFF_BAR + 8 * NBAR + 8;
    // The swizzled operands need a 1024-byte aligned base. The strip layout leaves no room for alignment slack: its
    // kernel requires the dynamic shared memory to start 1024-aligned (it does when the kernel has no static shared
    // memory) and reports a device error otherwise.
    static constexpr size_t ALIGN_SLACK = STRIP ? 0 : 1024;
    static constexpr size_t smem() { return ALIGN_SLACK + OFF_SEED + 8; }
    static_assert(OFF_BAR % 8 == 0, "mbarrier alignment");
    static_assert(smem() <= 232448, "227 KB of shared memory per CTA");
};

// X_STABLE: x was written before the previous non-step kernel on the stream, so its first rows may be copied before
// the wait for the previous kernel (a compile-time choice: the two instances keep the same register allocation).
template <int C, int HID, int NPART, bool X_STABLE, bool STRIP = false>
__global__ void __launch_bounds__(128 * NPART + 96, 1) bwd_rows_kernel(StepArgs a)
{
    using F = BwdRows<C, HID, NPART, STRIP>;
    using D = typename F::D;
    // the next step's kernel may launch now (it waits for this one before reading the state it writes)
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    extern __shared__ __align__(128) unsigned char smem_raw[];
    if (STRIP && (umma::smem_u32(smem_raw) & 1023) != 0) {  // no room for alignment slack (the layout would overrun)
        if (threadIdx.x == 0)
            set_device_error(3);
        return;
    }
    unsigned char *base = smem_raw + ((1024 - (umma::smem_u32(smem_raw) & 1023)) & 1023);
    float *W1s = reinterpret_cast<float *>(base), *W1T = W1s + D::W1S, *W2T = W1T + D::W1T;
    float *PSW = reinterpret_cast<float *>(base + F::OFF_PSW), *RH = reinterpret_cast<float *>(base + F::OFF_RH),
          *DH = RH + D::RHDH;
    float *XR = reinterpret_cast<float *>(base + F::OFF_XR);
    float4 *EDGE = reinterpret_cast<float4 *>(base + F::OFF_EDGE);
    uint8_t *MK = base + F::OFF_MK;
    uint64_t *xfull = reinterpret_cast<uint64_t *>(base + F::OFF_BAR), *g1bar = xfull + F::XRING, *dpbar = g1bar + 1,
             *wgbar = dpbar + 1, *wggo = wgbar + 1, *ea_done = wggo + 1, *fe_done = ea_done + 1, *mkfull = fe_done + 1;
    uint32_t *tslot = reinterpret_cast<uint32_t *>(mkfull + 2);
    volatile uint32_t *abort = tslot + 1;

    const int tid = threadIdx.x, warp = tid / 32, lane32 = tid % 32;
    const bool compute = warp < F::W_MMA, mma = warp == F::W_MMA, prod = warp == F::W_PROD;
    const int part = compute ? tid / 128 : 0, x = tid % 128, wq = warp & 3;
    const int H = a.H, W = a.W;
    const int S = STRIP ? W / 128 : 1;  // column strips per row
    const bool vx = compute && (STRIP || x < W);
    const int xc = STRIP ? x : x < W ? x : 0;
    // the lane's left, centre and right columns in a ring row (STRIP: 4 halo columns precede the strip's first)
    const int il = STRIP ? x + 3 : xc == 0 ? W - 1 : xc - 1, ic = STRIP ? x + 4 : xc,
              ir = STRIP ? x + 5 : xc + 1 >= W ? 0 : xc + 1;
    const int RS = STRIP ? F::XS : W;  // ring row stride
    const size_t plane = (size_t)H * W;
    // this CTA's rows [g0, g1), found by every thread (no thread waits for another to find them), and the step's mask
    // seed, read once by thread 0 (STRIP: in the dynamic shared memory, so that the kernel has no static shared memory
    // and its dynamic shared memory starts 1024-aligned)
    __shared__ uint64_t seed_static;
    uint64_t *seed_sh = STRIP ? reinterpret_cast<uint64_t *>(base + F::OFF_SEED) : &seed_static;
    int64_t g0, g1;
    band_range(row_bands(a, gridDim.x), blockIdx.x, &g0, &g1);
    const int k_first = g1 > g0 ? (int)(g0 / ((int64_t)a.B * H)) : -1;  // the NCA of the band's first row
    // X_STABLE (x not written by the previous kernel) and one tile per row: the producer copies the first segment's
    // first x rows, and prefetches the next ones into L2, as soon as the mbarriers exist, while the weights are staged
    constexpr bool EARLY_X = X_STABLE && !STRIP;
    const bool early_x = EARLY_X && k_first >= 0;

    // constant PSW features of both buffers: 1 at PIN and PIN + 1, 0 at GM0 + C .. 63
    constexpr int NCONST = 64 - C - D::PIN;  // features PIN .. 63 other than gm
    for (int e = tid; e < 2 * 128 * NCONST; e += blockDim.x) {
        const int b = e / (128 * NCONST), q = (e / NCONST) % 128, i = e % NCONST;
        const int f = i < F::GM0 - D::PIN ? D::PIN + i : F::GM0 + C + (i - (F::GM0 - D::PIN));
        PSW[b * D::PSW + umma::sw32_offset(f, q, 128) / 4] = f < F::GM0 ? 1.f : 0.f;
    }
    // Set-up: warp 0 initialises the mbarriers (then the producer may copy) and allocates the Tensor Memory; the
    // producer copies / prefetches the first rows (early_x); warps 1 .. W_PROD - 1 stage the first NCA's weights, the
    // set-up's longest part, from the kernel's entry on.
    if (warp == 0) {
        if (lane32 == 0) {
            const uint64_t sd = step_seed_of(a);  // in flight while the mbarriers are initialised
            for (int i = 0; i < F::XRING; ++i)
                umma::mbar_init(&xfull[i], 1);
            umma::mbar_init(&mkfull[0], 1);
            umma::mbar_init(&mkfull[1], 1);
            umma::mbar_init(g1bar, 1);
            umma::mbar_init(dpbar, 1);
            umma::mbar_init(wgbar, 1);
            umma::mbar_init(wggo, 1);
            umma::mbar_init(ea_done, F::W_MMA);
            umma::mbar_init(fe_done, F::W_MMA);
            *abort = 0;
            umma::fence_mbar_init();
            *seed_sh = sd;
        }
        __syncwarp();
        if (early_x)
            bar_arrive(2, 64);
        umma::tmem_alloc(tslot, F::TMEM);
        umma::tmem_relinquish();
    } else if (prod) {
        if (early_x) {
            bar_sync(2, 64);  // warp 0 initialised the mbarriers
            int64_t gg = g0;
            RowSeg sg0;
            next_segment(gg, g1, H, sg0);
            const int L0 = sg0.r1 - sg0.r0 + 2;
            const float *xn0 = a.x + (size_t)sg0.n * C * plane, *gyn0 = a.gy + (size_t)sg0.n * C * plane;
            for (int e = 0; e < F::XRING; ++e) {  // entries 0 .. XRING - 1 (the segment's prologue skips them)
                if (lane32 == 0)
                    umma::mbar_arrive_expect_tx(&xfull[e], (uint32_t)(C * W * 4));
                __syncwarp();
                if (lane32 < C)
                    umma::bulk_g2s(XR + ((size_t)e * C + lane32) * W,
                                   xn0 + ((size_t)lane32 * H + wrap_index(sg0.r0 - 2 + e, H)) * W, (uint32_t)(W * 4),
                                   &xfull[e]);
            }
            for (int e = F::XRING; e < 2 * F::XRING && e <= L0 + 1; ++e) {  // the prologue's L2 prefetches, early
                const int Y = wrap_index(sg0.r0 - 2 + e, H), c = lane32 - 16;
                if (lane32 < C)
                    umma::bulk_prefetch_l2(xn0 + ((size_t)lane32 * H + Y) * W, (uint32_t)(W * 4));
                if (c >= 0 && c < C && e - 1 < L0)
                    umma::bulk_prefetch_l2(gyn0 + ((size_t)c * H + Y) * W, (uint32_t)(W * 4));
            }
        }
    } else if (warp < F::W_PROD && k_first >= 0) {
        const int k = k_first;
        stage_rows_weights<D, true>(W1s, W1T, W2T, a.w1 + (size_t)k * HID * D::PIN, a.b1 + (size_t)k * HID,
                                    a.w2 + (size_t)k * C * HID, tid - 32, 32 * (F::W_PROD - 1), F::GM0 - D::PIN);
        umma::fence_proxy_async();
    }
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    const uint32_t tmem = *tslot, lane = umma::tmem_addr(tmem, warp, 0);
    if (compute && part == 0) {  // constant P columns of both buffers: 1, 1 at PIN, PIN + 1; 0 up to 63
        const float v[8] = {1.f, 1.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f}, z[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        umma::tmem_st8(lane + F::T_P0 + D::PIN, v);
        umma::tmem_st8(lane + F::T_P0 + D::PIN + 8, z);
        umma::tmem_st8(lane + F::T_P1 + D::PIN, v);
        umma::tmem_st8(lane + F::T_P1 + D::PIN + 8, z);
        umma::tmem_wait_st();
    }
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    bool ok = true;

    if (warp == F::W_WG) {
        // ---------------- weight-gradient issuer: one WG group per owned row, in the order of the rows
        if (lane32 == 0) {
            const uint64_t dA0 = umma::smem_desc(umma::smem_u32(PSW), 128 * 128, 512, umma::LAYOUT_SW128_32B);
            const uint64_t dA1 = umma::smem_desc(umma::smem_u32(PSW + D::PSW), 128 * 128, 512, umma::LAYOUT_SW128_32B);
            const uint64_t dB = umma::smem_desc(umma::smem_u32(RH), 128 * 128, 512, umma::LAYOUT_SW128_32B);
            constexpr uint32_t IWG = umma::idesc_tf32(128, F::NACC, true, true);
            uint32_t goph = 0;
            int wk = -1, issued = 0;
            bool started = false;
            int64_t g = g0;
            RowSeg sg;
            while (next_segment(g, g1, H, sg)) {
                const int k = sg.n / a.B, L = sg.r1 - sg.r0 + 2;
                if (k != wk) {
                    wk = k;
                    started = false;
                }
                for (int s = 0; s < S; ++s)
                    for (int i = 1; i <= L - 2; ++i) {
                        ok &= wait_bar(wggo, goph, abort);
                        goph ^= 1;
                        if (!ok)
                            continue;
                        umma::fence_after_sync();
                        const uint64_t dA = (i & 1) ? dA1 : dA0;
#pragma unroll
                        for (int ks = 0; ks < 16; ++ks)
                            umma::mma_ss(tmem + F::T_ACC, dA + (uint64_t)(ks * 64), dB + (uint64_t)(ks * 64), IWG,
                                         started || ks > 0);
                        umma::commit(wgbar);
                        started = true;
                        ++issued;
                    }
            }
            if (issued > 0)  // this warp's MMAs are complete before the teardown
                umma::mbar_wait(wgbar, (uint32_t)((issued - 1) & 1));
        }
    } else {
        // ---------------- compute, MMA and producer warps
        const uint64_t dW1 = umma::smem_desc(umma::smem_u32(W1s), HID * 16, 128);
        const uint64_t dW1T = umma::smem_desc(umma::smem_u32(W1T), D::PIN * 16, 128);
        const uint64_t dW2T = umma::smem_desc(umma::smem_u32(W2T), HID * 16, 128);
        constexpr uint32_t I1 = umma::idesc_tf32(128, HID, false, false), IP = umma::idesc_tf32(128, D::PIN, false, false);
        uint32_t xpar = 0, mkpar = 0, g1ph = 0, dpph = 0, wgph = 0, eaph = 0, feph = 0;
        // k_first's weights were staged above; early_x: the first segment's entries 0 .. XRING - 1 were issued and its
        // prologue's prefetches made above
        int cur_k = k_first, g1_issued = 0, dp_issued = 0, x_issued[F::XRING] = {0, 0, 0};
        bool x_pre = early_x && prod;
        if (x_pre)
            for (int e = 0; e < F::XRING; ++e)
                x_issued[e] = 1;
        bool dep_waited = false;
        auto group_sync = [&]() {
            umma::fence_before_sync();
            bar_sync(1, F::GROUP);
            umma::fence_after_sync();
        };
        auto signal = [&](uint64_t *bar) {  // this warp's TMEM and shared-memory writes are complete
            umma::fence_before_sync();
            __syncwarp();
            if (lane32 == 0)
                mbar_arrive(bar);
        };
        // WG accumulator -> partial slot (blockIdx.x + kk). TMEM lane f is the accumulator row f: dW1[.][f] (f < PIN) and
        // db1 (f = PIN) in columns HID.., dW2[f - GM0][.] (GM0 <= f < GM0 + C) in columns 0..HID-1. Only the warps of lane
        // quadrants 0 and 1 can read lanes 0..63; each reads the column groups its rows need, in chunks of 8 columns,
        // chunk i of a group going to part i % NPART. partial_add: the slot already holds this rollout's later steps and
        // the chunk is added by reductions at L2 (red.global.add: no old value travels to the SM; this CTA is the slot's
        // only writer in the launch, so each element is old + v rounded once, as a load-add-store would give, except
        // that a subnormal sum flushes to zero); otherwise the chunk is stored.
        auto flush = [&](int kk) {
            if (!compute || wq >= 2)
                return;
            const int f = x;
            float *out = a.partial + (size_t)(blockIdx.x + kk) * D::PART;
            const bool add = a.partial_add != 0;
            constexpr int NCH = HID / 8;  // chunks per group
            const int q0 = 32 * wq;       // the warp's rows q0 .. q0 + 31
            const bool need2 = q0 < F::GM0 + C && q0 + 32 > F::GM0, need1 = q0 <= D::PIN;  // warp-uniform
            const bool row2 = f >= F::GM0 && f < F::GM0 + C;
            float *row = row2 ? out + HID * (D::PIN + 1) + (f - F::GM0) * HID : f < D::PIN ? out + f : out + HID * D::PIN;
            const int js = row2 || f == D::PIN ? 1 : D::PIN;  // element stride along the columns j
            const bool mine = row2 || f <= D::PIN;
#pragma unroll 1
            for (int i = part; i < NCH; i += NPART) {
                float v2[8] = {}, v1[8] = {};
                if (need2)
                    umma::tmem_ld8(lane + F::T_ACC + i * 8, v2);
                if (need1)
                    umma::tmem_ld8(lane + F::T_ACC + HID + i * 8, v1);
                umma::tmem_wait_ld();
                if (mine) {
                    float *o = row + (size_t)(i * 8) * js;
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        const float v = row2 ? v2[e] : v1[e];
                        if (add)
                            atomicAdd(o + e * js, v);
                        else
                            o[e * js] = v;
                    }
                }
            }
        };
        auto g1_issue = [&](int bj) {  // G1: h = [p' 1 1 0..] W1ext^T -> H, dhp = [1 1 gm 0 0] W2T' -> DHP
            const uint32_t tp = tmem + (bj ? F::T_P1 : F::T_P0);
#pragma unroll
            for (int ks = 0; ks < D::KP / 8; ++ks)
                umma::mma_ts(tmem + F::T_H, tp + ks * 8, dW1 + (uint64_t)(ks * 2 * HID), I1, ks > 0);
#pragma unroll
            for (int ks = 0; ks < 2; ++ks)
                umma::mma_ts(tmem + F::T_DHP, tp + D::PIN + ks * 8, dW2T + (uint64_t)(ks * 2 * HID), I1, ks > 0);
            umma::commit(g1bar);
            ++g1_issued;
        };
        auto ring_wait_x = [&](int &waited, int upto) {  // compute threads: x entries .. upto landed
            while (waited <= upto) {
                const int slot = waited % F::XRING;
                ok &= wait_bar(&xfull[slot], (xpar >> slot) & 1u, abort);
                xpar ^= 1u << slot;
                ++waited;
            }
        };

        int64_t g = g0;
        RowSeg sg;
        while (next_segment(g, g1, H, sg))
          for (int s = 0; s < S; ++s) {  // the column strips of the segment (one pass unless STRIP)
            const int n = sg.n, k = n / a.B, L = sg.r1 - sg.r0 + 2;  // sequence: halo, owned rows, halo
            const int c0 = 128 * s, gcol = c0 + xc;  // the strip's first column; the lane's column in the image
            const float *xn = a.x + (size_t)n * C * plane, *gyn = a.gy + (size_t)n * C * plane;
            float *gxn = a.gx + (size_t)n * C * plane;
            auto rowY = [&](int i) { return wrap_index(sg.r0 - 1 + i, H); };
            // producer warp: x row wrap(r0 - 2 + e) -> slot e % XRING (one lane per channel). STRIP: columns
            // c0 - 4 .. c0 + 131 (circular) -> ring columns 0 .. 135, as one copy or two where the range wraps (every
            // piece starts and ends on a 16-byte boundary: W and c0 are multiples of 128)
            auto issue_x = [&](int e) {
                const int slot = e % F::XRING, Y = wrap_index(sg.r0 - 2 + e, H);
                ok = __shfl_sync(~0u, ok, 0);  // lane 0 did the waits: the whole warp takes one path
                if (ok) {
                    if (lane32 == 0)
                        umma::mbar_arrive_expect_tx(&xfull[slot], (uint32_t)(C * RS * 4));
                    __syncwarp();
                    if (lane32 < C) {
                        float *dst = XR + ((size_t)slot * C + lane32) * RS;
                        const float *src = xn + ((size_t)lane32 * H + Y) * W;
                        if (!STRIP) {
                            umma::bulk_g2s(dst, src, (uint32_t)(W * 4), &xfull[slot]);
                        } else if (s == 0) {
                            umma::bulk_g2s(dst, src + W - 4, 16u, &xfull[slot]);
                            umma::bulk_g2s(dst + 4, src, 132u * 4u, &xfull[slot]);
                        } else if (s == S - 1) {
                            umma::bulk_g2s(dst, src + c0 - 4, 132u * 4u, &xfull[slot]);
                            umma::bulk_g2s(dst + 132, src, 16u, &xfull[slot]);
                        } else {
                            umma::bulk_g2s(dst, src + c0 - 4, 136u * 4u, &xfull[slot]);
                        }
                    }
                    ++x_issued[slot];
                }
            };
            // producer warp: the x row of entry e and the gy row of sequence row e - 1 (read by the front end of that
            // row) into L2, some rows before their copy / load: the three-slot ring alone does not cover the latency
            // of HBM (one lane per channel row; STRIP: the strip's 128 columns)
            auto prefetch_rows = [&](int e) {
                if (e > L + 1)
                    return;
                const uint32_t bytes = STRIP ? 512u : (uint32_t)(W * 4);
                if (lane32 < C)
                    umma::bulk_prefetch_l2(xn + ((size_t)lane32 * H + wrap_index(sg.r0 - 2 + e, H)) * W + c0, bytes);
                const int c = lane32 - 16;
                if (c >= 0 && c < C && e >= 1 && e - 1 < L)
                    umma::bulk_prefetch_l2(gyn + ((size_t)c * H + rowY(e - 1)) * W + c0, bytes);
            };
            // producer warp: update mask of sequence row j (the strip's columns) -> MK[j % 2], then mkfull[j % 2]
            auto draw_mask = [&](int j, uint64_t sd) {
                ok = __shfl_sync(~0u, ok, 0);
                if (ok) {
                    if (STRIP)
                        row_mask_strip_warp(MK + (j & 1) * 128, sd, a.rate, n + a.n_offset, H, W, rowY(j),
                                            lane32, c0);
                    else
                        row_mask_warp(MK + (j & 1) * 128, sd, a.rate, n + a.n_offset, H, W, rowY(j), lane32);
                    __syncwarp();
                    if (lane32 == 0)
                        mbar_arrive(&mkfull[j & 1]);
                }
            };
            // ---- segment prologue. The first x rows are requested before any weight work (their slots were consumed
            // by the previous segment's last front end, which the producer waited for), so that the copies are in
            // flight while a new NCA's weights are staged. The first wait for the previous kernel on the stream (this
            // one is launched as its programmatic dependent; it may have written x or gy and adds to the same partial
            // slots) comes before them, or, when the caller declared x stable, after the weight staging.
            if (!X_STABLE && !dep_waited) {
                asm volatile("griddepcontrol.wait;" ::: "memory");
                dep_waited = true;
            }
            if (prod && !x_pre) {
                for (int e = 0; e < F::XRING; ++e)
                    issue_x(e);
                for (int e = F::XRING; e < 2 * F::XRING; ++e)
                    prefetch_rows(e);
            }
            x_pre = false;
            // a new NCA needs its weights (and the old accumulator flushed)
            if (k != cur_k) {
                group_sync();  // every warp finished the previous segment; its tensor-core work completed
                if (ok && cur_k >= 0)
                    flush(cur_k);
                stage_rows_weights<D, true>(W1s, W1T, W2T, a.w1 + (size_t)k * HID * D::PIN, a.b1 + (size_t)k * HID,
                                            a.w2 + (size_t)k * C * HID, tid, F::GROUP, F::GM0 - D::PIN);
                umma::fence_proxy_async();
                group_sync();
                cur_k = k;
            }
            if (X_STABLE && !dep_waited) {
                asm volatile("griddepcontrol.wait;" ::: "memory");
                dep_waited = true;
            }
            if (prod) {
                // ======== producer: entries 0..2 (issued above) and masks 0, 1; after every warp's FE(j): entry j + 3,
                // mask j + 2
                const uint64_t sd = *seed_sh;
                draw_mask(0, sd);
                if (L > 1)
                    draw_mask(1, sd);
                for (int j = 0; j < L; ++j) {
                    if (lane32 == 0)
                        ok &= wait_bar(fe_done, feph, abort);
                    feph ^= 1;
                    ok = __shfl_sync(~0u, ok, 0);
                    if (j + 3 <= L + 1)
                        issue_x(j + 3);
                    prefetch_rows(j + 2 * F::XRING);
                    if (j + 2 < L)
                        draw_mask(j + 2, sd);
                    // the partial slot this NCA's accumulator is added to when the segment ends: into L2 a few rows
                    // ahead, so that the flush's reads of the old values hit
                    if (a.partial_add && lane32 == 0 && j == (L > 4 ? L - 4 : 0))
                        umma::bulk_prefetch_l2(a.partial + (size_t)(blockIdx.x + k) * D::PART, (uint32_t)(D::PART * 4));
                }
            } else if (mma) {
                // ======== MMA warp: G1(0); per row DP(i), then G1(i+1)
                if (lane32 == 0) {
                    ok &= wait_bar(fe_done, feph, abort);
                    feph ^= 1;
                    if (ok) {
                        umma::fence_after_sync();
                        g1_issue(0);
                    }
                    for (int i = 0; i < L; ++i) {
                        const int b = i & 1;
                        ok &= wait_bar(ea_done, eaph, abort);
                        eaph ^= 1;
                        if (ok) {
                            umma::fence_after_sync();
                            const uint32_t tp = tmem + (b ? F::T_P1 : F::T_P0);
#pragma unroll
                            for (int ks = 0; ks < HID / 8; ++ks)
                                umma::mma_ts(tp, tmem + F::T_H + ks * 8, dW1T + (uint64_t)(ks * 2 * D::PIN), IP, ks > 0);
                            umma::commit(dpbar);
                            ++dp_issued;
                            if (i >= 1 && i <= L - 2)
                                mbar_arrive(wggo);
                        }
                        if (i + 1 < L) {
                            ok &= wait_bar(fe_done, feph, abort);
                            feph ^= 1;
                        }
                        ok &= wait_bar(dpbar, dpph, abort);  // DP(i) read H: G1(i+1) may overwrite it
                        dpph ^= 1;
                        if (ok && i + 1 < L) {
                            umma::fence_after_sync();
                            g1_issue(b ^ 1);
                        }
                    }
                }
            } else {
                // ======== compute warps
                int xwaited = 0;
                float gyA[F::CPP];  // gy of the next front end's row
                float win[F::CPP][6];  // rows Y - 1, Y (x[l], x[c], x[r]) of the last front end's channels
                auto load_gy = [&](int j) {
                    const float *src = gyn + (size_t)rowY(j) * W + gcol;
#pragma unroll
                    for (int cc = 0; cc < F::CPP; ++cc)
                        gyA[cc] = __ldg(src + (size_t)(F::CPP * part + cc) * plane);
                };
                // front end of sequence row j into buffer bj: p' and gm -> TMEM P[bj] and PSW[bj]
                auto front_end = [&](int j, int bj) {
                    ring_wait_x(xwaited, j + 2);  // x rows Y_j - 1 .. Y_j + 1
                    ok &= wait_bar(&mkfull[j & 1], (mkpar >> (j & 1)) & 1u, abort);  // the mask of row j
                    mkpar ^= 1u << (j & 1);
                    const float *rm = XR + (size_t)(j % F::XRING) * C * RS, *r0 = XR + (size_t)((j + 1) % F::XRING) * C * RS,
                                *rp = XR + (size_t)((j + 2) % F::XRING) * C * RS;
                    const bool m = MK[(j & 1) * 128 + xc] != 0;
                    float *psw = PSW + bj * D::PSW;
                    const uint32_t tp = lane + (bj ? F::T_P1 : F::T_P0);
#pragma unroll
                    for (int cc = 0; cc < F::CPP; ++cc) {  // warp-uniform channel: tcgen05.st takes one column per warp
                        const int c = F::CPP * part + cc;
                        const float *bm = rm + c * RS, *b0 = r0 + c * RS, *bp = rp + c * RS;
                        if (j == 0) {
                            win[cc][0] = bm[il]; win[cc][1] = bm[ic]; win[cc][2] = bm[ir];
                            win[cc][3] = b0[il]; win[cc][4] = b0[ic]; win[cc][5] = b0[ir];
                        }
                        const float v[3][3] = {{win[cc][0], win[cc][1], win[cc][2]}, {win[cc][3], win[cc][4], win[cc][5]},
                                               {bp[il], bp[ic], bp[ir]}};
                        win[cc][0] = v[1][0]; win[cc][1] = v[1][1]; win[cc][2] = v[1][2];
                        win[cc][3] = v[2][0]; win[cc][4] = v[2][1]; win[cc][5] = v[2][2];
                        const float4 p = perceive3x3(v);
                        const float t4[4] = {tf32_bias(p.x), tf32_bias(p.y), tf32_bias(p.z), tf32_bias(p.w)};
                        umma::tmem_st4(tp + 4 * c, t4);
                        *reinterpret_cast<float4 *>(psw + umma::sw32_offset(4 * c, x, 128) / 4) =
                            make_float4(t4[0], t4[1], t4[2], t4[3]);
                        const float gmv = (vx && m) ? tf32_bias(gyA[cc]) : 0.f;
                        umma::tmem_st1(tp + F::GM0 + c, gmv);
                        psw[umma::sw32_offset(F::GM0 + c, x, 128) / 4] = gmv;
                    }
                    umma::tmem_wait_st();
                    umma::fence_proxy_async();
                    signal(fe_done);
                };
                load_gy(0);
                front_end(0, 0);
                if (L > 1)
                    load_gy(1);
                float accm[F::CPP], acc0[F::CPP], accp[F::CPP];
#pragma unroll
                for (int cc = 0; cc < F::CPP; ++cc)
                    accm[cc] = acc0[cc] = accp[cc] = 0.f;

                for (int i = 0; i < L; ++i) {
                    const int b = i & 1, Y = rowY(i);
                    const bool owned = i >= 1 && i <= L - 2, next = i + 1 < L;
                    // gy of row Y - 1, for the final gx of that row at the end of this row's adjoint (an L2 hit: its
                    // front end read it two rows ago)
                    const bool fin = i >= 2 && vx;
                    const size_t prow = (size_t)wrap_index(Y - 1, H) * W + gcol;
                    float gprev[F::CPP];
                    auto load_gprev = [&]() {
#pragma unroll
                        for (int cc = 0; cc < F::CPP; ++cc)
                            gprev[cc] = fin ? __ldg(gyn + prow + (size_t)(F::CPP * part + cc) * plane) : 0.f;
                    };
                    // requested here, so that the loads complete under EA and FE (strips), or at the start of the
                    // adjoint (one tile per row: measured 1.3% faster, the registers are free during EA and FE; the
                    // strip instance measured 0.9% slower that way)
                    if (STRIP)
                        load_gprev();
                    // ---- EA(i): relu(h) -> RH, dh -> DH (owned rows) and TMEM H; needs G1(i) and WG(i-1)
                    ok &= wait_bar(g1bar, g1ph, abort);
                    g1ph ^= 1;
                    if (i >= 2) {
                        ok &= wait_bar(wgbar, wgph, abort);
                        wgph ^= 1;
                    }
                    umma::fence_after_sync();
#pragma unroll
                    for (int q = 0; q < F::HPP / 8; ++q) {
                        const int j0 = part * F::HPP + q * 8;
                        float h[8], d[8];
                        umma::tmem_ld8(lane + F::T_H + j0, h);
                        umma::tmem_ld8(lane + F::T_DHP + j0, d);
                        umma::tmem_wait_ld();
#pragma unroll
                        for (int e = 0; e < 8; ++e) {
                            d[e] = h[e] > 0.f ? tf32_bias(d[e]) : 0.f;
                            h[e] = tf32_bias(fmaxf(h[e], 0.f));
                        }
                        if (owned) {
                            st_sw32x8_balanced(RH, j0, x, 128, h);
                            st_sw32x8_balanced(DH, j0, x, 128, d);
                        }
                        umma::tmem_st8(lane + F::T_H + j0, d);
                    }
                    umma::tmem_wait_st();
                    umma::fence_proxy_async();
                    signal(ea_done);
                    // ---- FE(i+1)
                    if (next) {
                        front_end(i + 1, b ^ 1);
                        if (i + 2 < L)
                            load_gy(i + 2);
                    }
                    // ---- ADJ(i): dp(i) -> gx rows Y - 1, Y, Y + 1; gx(Y - 1) final
                    if (!STRIP)
                        load_gprev();
                    ok &= wait_bar(dpbar, dpph, abort);
                    dpph ^= 1;
                    umma::fence_after_sync();
                    float dpv[F::CPP][4];
#pragma unroll
                    for (int cc = 0; cc < F::CPP; ++cc)
                        umma::tmem_ld4(lane + (b ? F::T_P1 : F::T_P0) + 4 * (F::CPP * part + cc), dpv[cc]);
                    umma::tmem_wait_ld();
                    const int my_slot = lane32 == 0 ? wq : lane32 == 31 ? 4 + wq : -1;
                    // neighbour source: an edge slot, -1 a shuffle, -2 (STRIP: the strip's first and last columns)
                    // none: the other strip's term is added by the edge fix-up
                    const int lsrc = x == 0 ? (STRIP ? -2 : 8) : lane32 == 0 ? 4 + wq - 1 : -1;
                    const int rsrc = STRIP ? (x == 127 ? -2 : lane32 == 31 ? wq + 1 : -1)
                                           : (x == W - 1 ? 0 : lane32 == 31 ? wq + 1 : -1);
                    // STRIP: the edge columns of an owned row -> edge scratch [n][Y][strip][first / last][c]
                    float4 *eg = STRIP && owned && (x == 0 || x == 127)
                                     ? reinterpret_cast<float4 *>(a.dp) + ((((size_t)n * H + Y) * S + s) * 2 + (x == 127)) * C
                                     : nullptr;
#pragma unroll
                    for (int cc = 0; cc < F::CPP; ++cc) {  // edge lanes publish (sobel_x, sobel_y, laplacian) parts
                        const int c = F::CPP * part + cc;
                        const float4 t = make_float4(dpv[cc][1], dpv[cc][2], dpv[cc][3], 0.f);
                        if (my_slot >= 0)
                            EDGE[my_slot * C + c] = t;
                        if (!STRIP && x == W - 1)
                            EDGE[8 * C + c] = t;
                        if (STRIP && eg != nullptr)
                            eg[c] = t;
                    }
                    bar_sync(2 + part, 128);
#pragma unroll
                    for (int cc = 0; cc < F::CPP; ++cc) {
                        const int c = F::CPP * part + cc;
                        // neighbours x - 1 and x + 1 (circular in the row): shuffles in the warp, edge slots across warps
                        float lx = __shfl_up_sync(~0u, dpv[cc][1], 1), ly = __shfl_up_sync(~0u, dpv[cc][2], 1),
                              lz = __shfl_up_sync(~0u, dpv[cc][3], 1);
                        float rx = __shfl_down_sync(~0u, dpv[cc][1], 1), ry = __shfl_down_sync(~0u, dpv[cc][2], 1),
                              rz = __shfl_down_sync(~0u, dpv[cc][3], 1);
                        if (lsrc >= 0) {
                            const float4 e = EDGE[lsrc * C + c];
                            lx = e.x;
                            ly = e.y;
                            lz = e.z;
                        }
                        if (rsrc >= 0) {
                            const float4 e = EDGE[rsrc * C + c];
                            rx = e.x;
                            ry = e.y;
                            rz = e.z;
                        }
                        if (STRIP && lsrc == -2) {
                            lx = 0.f;
                            ly = 0.f;
                            lz = 0.f;
                        }
                        if (STRIP && rsrc == -2) {
                            rx = 0.f;
                            ry = 0.f;
                            rz = 0.f;
                        }
                        const float rsx = lx - rx;                      // horizontal transpose of sobel_x
                        const float rsy = ry + 2.f * dpv[cc][2] + ly;   // ... of sobel_y (smoothing)
                        const float rlap = lz + 2.f * dpv[cc][3] + rz;  // ... of the laplacian
                        accm[cc] += rsx - rsy + rlap;
                        acc0[cc] += 2.f * rsx + 2.f * rlap + dpv[cc][0] - 16.f * dpv[cc][3];
                        accp[cc] += rsx + rsy + rlap;
                        if (fin)
                            gxn[prow + (size_t)c * plane] = gprev[cc] + accm[cc];
                        accm[cc] = acc0[cc];
                        acc0[cc] = accp[cc];
                        accp[cc] = 0.f;
                    }
                }
            }
        }
        group_sync();  // every warp done; the last WG was waited by the compute warps at their last row
        if (ok && cur_k >= 0)
            flush(cur_k);
        if (mma && lane32 == 0) {  // this warp's MMAs are complete before the teardown
            if (g1_issued > 0)
                umma::mbar_wait(g1bar, (uint32_t)((g1_issued - 1) & 1));
            if (dp_issued > 0)
                umma::mbar_wait(dpbar, (uint32_t)((dp_issued - 1) & 1));
        }
        if (prod && lane32 == 0)  // and so are this warp's bulk copies
            for (int s2 = 0; s2 < F::XRING; ++s2)
                if (x_issued[s2] > 0)
                    umma::mbar_wait(&xfull[s2], (uint32_t)((x_issued[s2] - 1) & 1));
    }
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    if (warp == 0)
        umma::tmem_dealloc(tmem, F::TMEM);
    if (*abort || !ok)
        if (tid == 0)
            set_device_error(1);
}

// Cross-strip terms of the adjoint after bwd_rows_kernel<..., STRIP> (W = 128 S): the first column of strip s
// (x = 128 s) receives the terms of its left neighbour x - 1 (the last column of strip s - 1, circular) and the last
// column (x = 128 s + 127) those of its right neighbour x + 1 (the first column of strip s + 1), from the edge
// scratch edge[n][Y][strip][first / last][c] = (sobel_x, sobel_y, laplacian) parts of dp. With L = such a part vector
// of the left neighbour in row Y', gx(Y) += (Lx - Ly + Lz)(Y + 1) + 2 (Lx + Lz)(Y) + (Lx + Ly + Lz)(Y - 1) (rows
// circular); a right neighbour R enters as (-Rx - Ry + Rz)(Y + 1) + 2 (Rz - Rx)(Y) + (-Rx + Ry + Rz)(Y - 1): the
// horizontal transposes of sobel_x, sobel_y and the laplacian times their vertical weights, as in the row kernel's
// adjoint. One thread per (image, row, strip, side, channel).
template <int C>
__global__ void strip_edge_fixup_kernel(const float4 *__restrict__ edge, float *gx, int N, int H, int W)
{
    const int S = W / 128;
    const int64_t total = (int64_t)N * H * S * 2 * C;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int c = (int)(t % C);
        int64_t r = t / C;
        const int side = (int)(r % 2);
        r /= 2;
        const int s = (int)(r % S);
        r /= S;
        const int Y = (int)(r % H);
        const int64_t n = r / H;
        const int sn = side == 0 ? (s == 0 ? S - 1 : s - 1) : (s + 1 == S ? 0 : s + 1);  // the neighbour's strip
        auto at = [&](int yy) { return __ldg(edge + (((n * H + yy) * S + sn) * 2 + (1 - side)) * C + c); };
        const float4 up = at(Y == 0 ? H - 1 : Y - 1), mid = at(Y), dn = at(Y + 1 == H ? 0 : Y + 1);
        const float v = side == 0 ? (dn.x - dn.y + dn.z) + 2.f * (mid.x + mid.z) + (up.x + up.y + up.z)
                                  : (-dn.x - dn.y + dn.z) + 2.f * (mid.z - mid.x) + (-up.x + up.y + up.z);
        gx[((n * C + c) * H + Y) * W + 128 * s + (side ? 127 : 0)] += v;
    }
}

}  // namespace unca
