// Kernels of the fused batched NCA step for sm_100a.
//
// One step for N = K B images (image n belongs to NCA n / B), state x (N, C, H, W):
//   p = [id, sobel_x, sobel_x^T, laplacian](x) (circular 3x3, feature 4c + f), h = relu(W1 p + b1), u = W2 h,
//   y = x + u m (m = Philox update mask), growing: y *= a, a = (maxpool3(x_alpha) > .1) & (maxpool3(y_alpha) > .1).
// Reference semantics: ncaops/nca_step.cuh:1-19 (header comment), :343-691 (forward), :693-727 (alive),
// :729-1162 (backward), :1164-1193 (reduce), :1195-1263 (adjoint); oracle math ncaops/testing/test_nca.py:21-32.
//
// Design (B200-first, not the reference's warp-MMA design):
//   * persistent CTAs of 128 threads; CTA c owns the contiguous tile range [T c / G, T (c+1) / G) over all images, so
//     weights are staged once per NCA segment and weight gradients accumulate in Tensor Memory across the segment;
//   * a tile is 128 pixels (R rows x S columns); thread i owns tile pixel i and TMEM lane i;
//   * the MLP is three tcgen05.mma kind::tf32 contractions per tile in the forward (p -> h, h -> u with A = relu(h) read
//     back from TMEM) and five in the backward (h, dh, dp and the two weight-gradient contractions whose K dimension is
//     the tile's pixels, with MN-major operands so the same shared-memory tile feeds both orientations);
//   * the bias is folded into the first contraction as two TF32 columns (b1_hi + b1_lo = b1 to 2^-22 relative);
//   * weight gradients are reduced across CTAs in a fixed order (partial slot = CTA + NCA): bitwise deterministic;
//   * fp32 mode (the reference's 3xTF32 accuracy mode) runs the same tile loop with the MLP on CUDA cores in fp32.
#pragma once
#include "nca_common.cuh"
#include "umma.cuh"

namespace unca {

template <int C_, int HID_>
struct Dims {
    static constexpr int C = C_, HID = HID_;
    static constexpr int PIN = 4 * C;                    // perception features
    static constexpr int KP = PIN + 8;                   // + bias-hi, bias-lo and six zero columns
    static constexpr int CP = 16;                        // channels padded to the MMA N / K granule
    static constexpr int NP = ((KP + 15) / 16) * 16;     // N of the dW1' contraction
    static constexpr int TILE = 128;
    static constexpr int PLANE = TILE * 4;               // floats of one chunk plane of a 128-row operand
    static constexpr int XS_FLOATS = C * 390;            // (R + 2)(S + 2) <= 390 for R S <= 128
    static constexpr int HT = TILE + 1;                  // padded pixel stride of the fp32-mode transposed buffers
    // TMEM columns
    static constexpr int FWD_TMEM = (HID + 16) <= 128 ? 128 : 256;
    // backward (TF32): H, then dh (A of dp) | dh before the relu mask | p (A of p -> h), then dp | g m (A of dh) |
    // dW1' accumulator (lanes = hidden units) | dW2^T accumulator
    static constexpr int T_H = 0, T_DHP = 128, T_P = 256, T_G = 352, T_ACC1 = 384, T_ACC2 = 480, BWD_TMEM = 512;
    static constexpr int NPW = ((KP + 31) / 32) * 32;            // N of the dW1' contraction (whole 32-wide blocks)
    static_assert(T_ACC1 + NPW <= T_ACC2 && ((KP + 15) / 16) * 16 <= T_G - T_P, "backward TMEM budget");
    static_assert(HID % 32 == 0 && HID <= 128 && C <= 16 && C % 4 == 0, "supported NCA sizes");
    // shared memory (floats)
    static constexpr int W1S = HID * KP, W2S = CP * HID, P = TILE * KP, G = TILE * CP, RHDH = TILE * HID;
    static constexpr int W1T = PIN * HID, W2T = HID * CP;          // backward B operands (K-major, transposed)
    static constexpr int PSW = TILE * NPW, GSW = TILE * 32;         // backward swizzled MN-major operands
    static constexpr size_t fwd_smem() { return (size_t)(W1S + W2S + P + XS_FLOATS) * 4 + 16; }
    // TF32 backward: [W1S | W1T | W2T | pad to 1 KB] [RHDH (XS aliases it) | PSW | GSW] + barrier
    static constexpr int BWD_W = ((W1S + W1T + W2T) * 4 + 1023) / 1024 * 1024;
    // + the halo buffer of the next tile (prefetched during the current tile's contractions), positions: growing
    // (compact 8 x 16 tiles) 180, otherwise up to 390 (R S <= 128), or as many as fit in 227 KB
    static constexpr size_t BWD_BASE = 1024 + (size_t)BWD_W + (size_t)(RHDH + PSW + GSW) * 4 + 24;
    static constexpr int xs_pos(bool growing)
    {
        return growing ? 180 : (BWD_BASE + (size_t)C * 390 * 4 <= 232448 ? 390 : (int)((232448 - BWD_BASE) / (4 * C)));
    }
    static constexpr size_t bwd_smem_tc(bool growing) { return BWD_BASE + (size_t)C * xs_pos(growing) * 4; }
    static constexpr size_t bwd_smem_cc() { return (size_t)(W1S + W2S + P + G + 2 * HID * HT) * 4 + 16; }
    static constexpr int PART = HID * PIN + HID + C * HID;  // weight-gradient partial: dW1, db1, dW2
};

// Parts of 128 threads of the TF32 tile backward (bwd_kernel_tc).
constexpr int BWD_TILE_PARTS = 4;

struct StepArgs {
    const float *x, *w1, *b1, *w2;
    float *y, *alpha;              // forward outputs (alpha: growing only)
    const float *gy;               // backward
    const uint8_t *alive;          // backward, growing
    float *dp, *partial;           // backward workspaces
    float *gx;                     // backward output of the row-streaming kernel (adjoint fused)
    int N, B, H, W;
    uint64_t seed;
    float rate;
    int64_t n_offset;              // global index of image 0 (Philox counter)
    int partial_add;               // backward: add the weight-gradient partials to the slots instead of storing them
    const uint64_t *seed_dev;      // non-null: the step's seed is splitmix_step(*seed_dev, step), read at run time
    int64_t step;                  // (a launch recorded once in a CUDA graph and replayed with new rollout seeds)
    int band_s4, band_n4;          // row kernels: switch costs of the cost-balanced bands (Bands)
    uint32_t tile_perm;            // growing tile kernels: an NCA's M tiles are visited in the order u -> u tile_perm mod
                                   // M (coprime to M; 0: in order), so that the tiles of a living region, which are
                                   // consecutive, spread over the CTAs that share the NCA
    uint8_t *alive_out;            // growing forward: the alive mask of the step (N, H, W)
    int reuse;                     // growing rollout from its third step: alive_out holds this destination's map of two
                                   // steps ago (cells 0 there hold state 0)
};

// Growing forward tiles (the alive mask fused into the step): an interior of GI_R x GI_S cells is written; the MLP runs
// on the interior and its one-cell ring, an extended tile of (GI_R + 2) x (GI_S + 2) = 128 pixels (lane = extended
// pixel), so that the unmasked new alpha of every cell the interior's 3 x 3 pooling reads is at hand.
constexpr int GI_R = 6, GI_S = 14, GE_R = GI_R + 2, GE_S = GI_S + 2;
static_assert(GE_R * GE_S == 128, "extended growing tile");

// Extended-tile geometry of the fused growing forward (R, S: the extended tile; strips and tiles count interiors).
__host__ __device__ inline TileGeom make_grow_fwd_geom(int H, int W)
{
    TileGeom g;
    g.H = H; g.W = W;
    g.S = GE_S;
    g.R = GE_R;
    g.strips = (W + GI_S - 1) / GI_S;
    g.tiles_per_image = g.strips * ((H + GI_R - 1) / GI_R);
    return g;
}

// The row bands of a row-kernel launch of `a` over `G` CTAs.
__host__ __device__ inline Bands row_bands(const StepArgs &a, int G)
{
    return Bands{(int64_t)a.N * a.H, a.H, (int64_t)a.B * a.H, G, a.band_s4, a.band_n4};
}

// The update-mask seed of this launch's step.
__device__ __forceinline__ uint64_t step_seed_of(const StepArgs &a)
{
    return a.seed_dev != nullptr ? splitmix_step(*a.seed_dev, (uint64_t)a.step) : a.seed;
}

// Stage one NCA's weights: W1' (HID x KP, chunk-planar: plane f/4, row j) with the bias columns, W2 (16 x HID,
// chunk-planar: plane j/4, row c). TF32 mode rounds (b1 split into hi + lo); fp32 mode keeps fp32 and b1 in column PIN.
template <class D, bool TC>
__device__ __forceinline__ void stage_weights(float *W1s, float *W2s, const float *w1, const float *b1, const float *w2)
{
    for (int e = threadIdx.x; e < D::HID * D::KP; e += blockDim.x) {
        const int j = e / D::KP, f = e % D::KP;
        float v = 0.f;
        if (f < D::PIN)
            v = TC ? tf32_rna(w1[j * D::PIN + f]) : w1[j * D::PIN + f];
        else if (f == D::PIN)
            v = TC ? tf32_rna(b1[j]) : b1[j];
        else if (f == D::PIN + 1 && TC)
            v = tf32_rna(b1[j] - tf32_rna(b1[j]));
        W1s[(f / 4) * D::HID * 4 + j * 4 + (f % 4)] = v;
    }
    for (int e = threadIdx.x; e < D::CP * D::HID; e += blockDim.x) {
        const int c = e / D::HID, j = e % D::HID;
        const float v = c < D::C ? (TC ? tf32_rna(w2[c * D::HID + j]) : w2[c * D::HID + j]) : 0.f;
        W2s[(j / 4) * D::CP * 4 + c * 4 + (j % 4)] = v;
    }
}

__device__ __forceinline__ void cp_async4(float *dst, const float *src)
{
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(umma::smem_u32(dst)), "l"(src) : "memory");
}
// The same, with the destination zero-filled instead when !ld (nothing is read from src then).
__device__ __forceinline__ void cp_async4_zfill(float *dst, const float *src, bool ld)
{
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(umma::smem_u32(dst)), "l"(src), "r"(ld ? 4 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// State of image n around the tile at (y0, x0), with a one-pixel circular halo: XS[c][r][s], r < R+2, s < S+2, copied
// asynchronously (cp.async; the caller waits with cp_async_wait_all + a barrier). Thread t of the NT threads copies the
// halo positions t, t + NT, .. (< 390) of every channel; index arithmetic is done once per tile, not per element.
template <class D, int NT = 128>
__device__ __forceinline__ void load_halo_async(float *XS, const float *x, int n, const TileGeom &g, int y0, int x0)
{
    constexpr int NI = (390 + NT - 1) / NT;
    const int SS = g.S + 2, per = (g.R + 2) * SS;
    const size_t plane = (size_t)g.H * g.W;
    const float *xn = x + (size_t)n * D::C * plane;
    int goff[NI], soff[NI];
#pragma unroll
    for (int i = 0; i < NI; ++i) {
        const int e = threadIdx.x + NT * i;
        const int r = e / SS, s = e - r * SS;
        soff[i] = e < per ? e : -1;
        goff[i] = wrap_index(y0 - 1 + r, g.H) * g.W + wrap_index(x0 - 1 + s, g.W);
    }
#pragma unroll 4
    for (int c = 0; c < D::C; ++c)
#pragma unroll
        for (int i = 0; i < NI; ++i)
            if (soff[i] >= 0)
                cp_async4(XS + c * per + soff[i], xn + c * plane + goff[i]);
}

// Perception of tile pixel i into P (chunk-planar, plane c = the four filters of channel c, then the bias plane
// {1, 1, 0, 0} and a zero plane). Invalid pixels get an all-zero row.
template <class D, bool TC>
__device__ __forceinline__ void perceive_tile(float *P, const float *XS, const TileGeom &g, int i, bool valid, int c0 = 0,
                                              int nc = D::C, bool bias = true)
{
    const int r = i / g.S, s = i - r * g.S, SS = g.S + 2, per = (g.R + 2) * SS;
#pragma unroll 4
    for (int c = c0; c < c0 + nc; ++c) {
        float4 p = make_float4(0.f, 0.f, 0.f, 0.f);
        if (valid) {
            float v[3][3];
            const float *b = XS + c * per + r * SS + s;
#pragma unroll
            for (int dy = 0; dy < 3; ++dy)
#pragma unroll
                for (int dx = 0; dx < 3; ++dx)
                    v[dy][dx] = b[dy * SS + dx];
            p = perceive3x3(v);
            if (TC)
                p = make_float4(tf32_bias(p.x), tf32_bias(p.y), tf32_bias(p.z), tf32_bias(p.w));
        }
        *reinterpret_cast<float4 *>(P + c * D::PLANE + i * 4) = p;
    }
    if (!bias)
        return;
    *reinterpret_cast<float4 *>(P + (D::PIN / 4) * D::PLANE + i * 4) = valid ? make_float4(1.f, 1.f, 0.f, 0.f) : make_float4(0.f, 0.f, 0.f, 0.f);
    *reinterpret_cast<float4 *>(P + (D::PIN / 4 + 1) * D::PLANE + i * 4) = make_float4(0.f, 0.f, 0.f, 0.f);
}

struct TileCoord {
    int n, k, y0, x0, ty, tx;  // image, NCA, first row and column, tile row and column (strip) in the image
};

// Block-wide OR (blocks of NT threads, every thread calls it) of a 32-bit word; sw: NT / 32 words of shared memory.
template <int NT>
__device__ __forceinline__ uint32_t block_or(uint32_t v, uint32_t *sw)
{
    v = __reduce_or_sync(~0u, v);
    if ((threadIdx.x & 31) == 0)
        sw[threadIdx.x >> 5] = v;
    __syncthreads();
    uint32_t r = 0;
#pragma unroll
    for (int w = 0; w < NT / 32; ++w)
        r |= sw[w];
    __syncthreads();  // sw is reused by the next call
    return r;
}
__device__ __forceinline__ uint32_t block_or_128(uint32_t v, uint32_t *sw) { return block_or<128>(v, sw); }

// Tile t of a launch (32-bit arithmetic: the host keeps a launch's tile count below 2^31); PERM: visited in the order
// of a.tile_perm within its NCA (a separate kernel instance, so that the in-order kernels carry none of it).
template <bool PERM = false>
__device__ __forceinline__ TileCoord tile_coord(int64_t t, const TileGeom &g, const StepArgs &a)
{
    TileCoord tc;
    const uint32_t tpi = (uint32_t)g.tiles_per_image, strips = (uint32_t)g.strips, B = (uint32_t)a.B;
    uint32_t u = (uint32_t)t;
    if (PERM) {
        const uint32_t M = B * tpi, k = u / M, v = u - k * M;
        u = k * M + (uint32_t)(((uint64_t)v * a.tile_perm) % M);
    }
    const uint32_t n = u / tpi, ti = u - n * tpi, ty = ti / strips;
    tc.n = (int)n;
    tc.k = (int)(n / (uint32_t)B);
    tc.ty = (int)ty;
    tc.tx = (int)(ti - ty * strips);
    tc.y0 = tc.ty * g.R;
    tc.x0 = tc.tx * g.S;
    return tc;
}

// ================================================================ forward
// One CTA per SM slot, tiles [T c / G, T (c+1) / G). Writes y (growing: masked by the alive mask, which the epilogue
// computes and writes too).
// Growing NCAs, active tiles: the liveness of 32 consecutive tiles [t, t + 32) (tiles >= t1 count as dead), one bit per
// tile: whether some cell within two pixels of the tile's interior (no wrap: the alive pooling pads with zeros) has
// x_alpha > 0.1. If none has, every cell within one pixel of the interior is dead before the step, so the alive mask
// is 0 on the whole interior whatever the update computes: the tile writes zeros and runs no MLP. Every thread reads its
// share of each tile's (GI_R + 4) x (GI_S + 4) window, 8 tiles' worth in flight per round, then a block-wide OR; every
// thread of the block calls it.
template <int C, int NT = 128, bool PERM = false>
__device__ __forceinline__ uint32_t grow_tiles_live(const StepArgs &a, const TileGeom &g, int64_t t, int64_t t1,
                                                    uint32_t *sw)
{
    constexpr int SO = GI_S + 4, WIN = (GI_R + 4) * SO;  // 180 positions: threadIdx.x, threadIdx.x + NT, ..
    constexpr int NQ = (WIN + NT - 1) / NT;
    int dr[NQ], dc[NQ];
#pragma unroll
    for (int q = 0; q < NQ; ++q) {
        const int e = threadIdx.x + NT * q;
        dr[q] = e < WIN ? e / SO - 2 : -1000000;
        dc[q] = e < WIN ? e % SO - 2 : 0;
    }
    uint32_t mine = 0;
    for (int i0 = 0; i0 < 32; i0 += 8) {
        float v[8][NQ];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int64_t u = t + i0 + i;
            const bool tile_ok = u < t1;
            const TileCoord tc = tile_coord<PERM>(tile_ok ? u : t, g, a);
            const int iy0 = tc.ty * GI_R, ix0 = tc.tx * GI_S;
            const float *xa = a.x + ((size_t)tc.n * C + 3) * (size_t)a.H * a.W;
#pragma unroll
            for (int q = 0; q < NQ; ++q) {
                const int Y = iy0 + dr[q], X = ix0 + dc[q];
                v[i][q] = tile_ok && Y >= 0 && Y < a.H && X >= 0 && X < a.W ? __ldg(xa + (size_t)Y * a.W + X) : 0.f;
            }
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            bool lv = false;
#pragma unroll
            for (int q = 0; q < NQ; ++q)
                lv |= v[i][q] > 0.1f;
            mine |= lv ? 1u << (i0 + i) : 0u;
        }
    }
    return block_or<NT>(mine, sw);
}

// Growing NCAs, backward: a tile with no pixel alive after its forward step has gm = gy m a = 0 throughout, so it adds
// nothing to the weight gradients and its dp is 0; the backward skips it without writing its dp, and the adjoint
// reads dp at alive cells only. Tile pixel px of tile t alive (false when the pixel is outside the image).
template <bool PERM = false>
__device__ __forceinline__ bool pixel_alive(const StepArgs &a, const TileGeom &g, int64_t t, int px)
{
    const TileCoord tc = tile_coord<PERM>(t, g, a);
    const int r = px / g.S, s = px - r * g.S;
    const int Y = tc.y0 + r, X = tc.x0 + s;
    return px < g.R * g.S && Y < a.H && X < a.W && a.alive[((size_t)tc.n * a.H + Y) * a.W + X] != 0;
}

// Parts of 128 threads of the TF32 tile forward (fwd_kernel<.., true, ..>): part p runs channels [C p / NP, ..) of the
// halo perception and the epilogue and hidden units [HID p / NP, ..) of the relu pass, for its lane's pixel; two CTAs
// per SM (registers capped for it).
constexpr int FWD_TILE_PARTS = 2;

template <int C, int HID, bool TC, bool GROWING, bool PERM = false>
__global__ void __launch_bounds__(128 * (TC ? FWD_TILE_PARTS : 1), TC ? 2 : 1) fwd_kernel(StepArgs a)
{
    constexpr int NP = TC ? FWD_TILE_PARTS : 1, NT = 128 * NP, CPP = C / NP, HPP = HID / NP;
    static_assert(C % NP == 0 && HPP % 16 == 0, "forward tile parts");
    a.seed = step_seed_of(a);
    using D = Dims<C, HID>;
    extern __shared__ __align__(128) float smem[];
    float *W1s = smem, *W2s = W1s + D::W1S, *P = W2s + D::W2S, *XS = P + D::P;
    uint64_t *bar = reinterpret_cast<uint64_t *>(XS + D::XS_FLOATS);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bar + 1);

    const int tid = threadIdx.x, warp = tid / 32, part = tid / 128, lt = tid % 128;
    const TileGeom g = GROWING ? make_grow_fwd_geom(a.H, a.W) : make_geom(a.H, a.W);
    const int64_t T = (int64_t)a.N * g.tiles_per_image;
    int64_t t0, t1;
    cta_range(T, gridDim.x, blockIdx.x, &t0, &t1);
    const bool stoch = a.rate < 1.f;
    const size_t plane = (size_t)a.H * a.W;
    __shared__ uint32_t sw[NT / 32];
    __shared__ float XA[GROWING ? 128 : 1], YA[GROWING ? 128 : 1];  // growing: x_alpha and unmasked new alpha per lane
    uint32_t live_bits = 0;  // growing: liveness of tiles [live_base, live_base + 32)
    int64_t live_base = t0 - 64;

    uint32_t tmem = 0;
    if constexpr (TC) {
        if (tid == 0) {
            umma::mbar_init(bar, 1);
            umma::fence_mbar_init();
        }
        if (warp == 0) {
            umma::tmem_alloc(tmem_slot, D::FWD_TMEM);
            umma::tmem_relinquish();
        }
        umma::fence_before_sync();
        __syncthreads();
        umma::fence_after_sync();
        tmem = *tmem_slot;
    }
    uint32_t phase = 0;
    int cur_k = -1;
    bool failed = false;
    for (int64_t t = t0; t < t1 && !failed; ++t) {
        TileCoord tc = tile_coord<PERM>(t, g, a);
        if (GROWING) {  // the extended tile's origin: one cell above and left of the interior
            tc.y0 = tc.ty * GI_R - 1;
            tc.x0 = tc.tx * GI_S - 1;
        }
        const int r = lt / g.S, s = lt - r * g.S;
        const bool valid = GROWING ? tc.y0 + r >= 0 && tc.y0 + r < a.H && tc.x0 + s >= 0 && tc.x0 + s < a.W
                                   : lt < g.R * g.S && tc.y0 + r < a.H && tc.x0 + s < a.W;
        // growing: the lane's cell is in the interior (written by this tile)
        const bool inner = GROWING && valid && r >= 1 && r <= GI_R && s >= 1 && s <= GI_S;
        const size_t cell = (size_t)tc.n * plane + (size_t)(tc.y0 + r) * a.W + (tc.x0 + s);
        if (GROWING) {  // dead tile (block-uniform): no MLP, no halo copy; its interior is dead after the step
            if (t >= live_base + 32) {
                live_base = t;
                live_bits = grow_tiles_live<C, NT, PERM>(a, g, t, t1, sw);
            }
            if (!((live_bits >> (t - live_base)) & 1u)) {
                // y = 0 and alive = 0 on the interior, by part 0 (its reuse check reads the alive byte it writes); in a
                // rollout's reuse steps a cell dead in this destination two steps ago already holds both
                if (part == 0 && inner && (!a.reuse || a.alive_out[cell])) {
                    float *yn = a.y + (size_t)tc.n * C * plane + (cell - (size_t)tc.n * plane);
#pragma unroll
                    for (int c = 0; c < C; ++c)
                        yn[(size_t)c * plane] = 0.f;
                    a.alive_out[cell] = 0;
                }
                continue;
            }
        }
        if (tc.k != cur_k) {  // staged at the NCA's first live tile
            stage_weights<D, TC>(W1s, W2s, a.w1 + (size_t)tc.k * HID * D::PIN, a.b1 + (size_t)tc.k * HID,
                                 a.w2 + (size_t)tc.k * C * HID);
            cur_k = tc.k;
        }
        load_halo_async<D, NT>(XS, a.x, tc.n, g, tc.y0, tc.x0);
        cp_async_wait_all();
        __syncthreads();
        perceive_tile<D, TC>(P, XS, g, lt, valid, CPP * part, CPP, part == 0);
        float u[CPP];  // this part's channels of the update
        if constexpr (TC) {
            umma::fence_proxy_async();
            __syncthreads();
            if (tid == 0) {
                umma::fence_after_sync();
                const uint32_t pa = umma::smem_u32(P), wa = umma::smem_u32(W1s);
#pragma unroll
                for (int ks = 0; ks < D::KP / 8; ++ks)
                    umma::mma_ss(tmem, umma::smem_desc(pa + ks * 2 * D::PLANE * 4, D::PLANE * 4, 128),
                                 umma::smem_desc(wa + ks * 2 * HID * 16, HID * 16, 128), umma::idesc_tf32(128, HID, false, false),
                                 ks > 0);
                umma::commit(bar);
            }
            bool ok = umma::mbar_wait(bar, phase);
            phase ^= 1;
            if (!__syncthreads_and(ok)) {
                failed = true;
                break;
            }
            umma::fence_after_sync();
            // relu(h) back into the same TMEM columns (TF32-rounded): the A operand of h -> u (this part's columns)
#pragma unroll
            for (int cc = 0; cc < HPP / 16; ++cc) {
                float v[16];
                const uint32_t ad = umma::tmem_addr(tmem, warp, HPP * part + cc * 16);
                umma::tmem_ld16(ad, v);
                umma::tmem_wait_ld();
#pragma unroll
                for (int e = 0; e < 16; ++e)
                    v[e] = tf32_bias(fmaxf(v[e], 0.f));
                umma::tmem_st16(ad, v);
            }
            umma::tmem_wait_st();
            umma::fence_before_sync();
            __syncthreads();
            if (tid == 0) {
                umma::fence_after_sync();
                const uint32_t w2a = umma::smem_u32(W2s);
#pragma unroll
                for (int ks = 0; ks < HID / 8; ++ks)
                    umma::mma_ts(tmem + HID, tmem + ks * 8, umma::smem_desc(w2a + ks * 2 * D::CP * 16, D::CP * 16, 128),
                                 umma::idesc_tf32(128, 16, false, false), ks > 0);
                umma::commit(bar);
            }
            ok = umma::mbar_wait(bar, phase);
            phase ^= 1;
            if (!__syncthreads_and(ok)) {
                failed = true;
                break;
            }
            umma::fence_after_sync();
#pragma unroll
            for (int cc = 0; cc < CPP; ++cc)
                u[cc] = umma::tmem_ld1(umma::tmem_addr(tmem, warp, HID + CPP * part + cc));
            umma::tmem_wait_ld();  // the loaded registers are defined only after this wait
        } else {
#pragma unroll
            for (int c = 0; c < CPP; ++c)
                u[c] = 0.f;
            if (valid) {
                float p[D::PIN];
#pragma unroll
                for (int f = 0; f < D::PIN; ++f)
                    p[f] = P[(f / 4) * D::PLANE + lt * 4 + (f % 4)];
                for (int j = 0; j < HID; ++j) {
                    const float *wrow = W1s + j * 4;
                    float h = wrow[(D::PIN / 4) * HID * 4];
#pragma unroll
                    for (int f = 0; f < D::PIN; ++f)
                        h = fmaf(wrow[(f / 4) * HID * 4 + (f % 4)], p[f], h);
                    h = fmaxf(h, 0.f);
                    const float *w2c = W2s + (j / 4) * D::CP * 4 + (j % 4);
#pragma unroll
                    for (int c = 0; c < CPP; ++c)
                        u[c] = fmaf(w2c[c * 4], h, u[c]);
                }
            }
        }
        if (!GROWING && valid) {
            const int Y = tc.y0 + r, X = tc.x0 + s;
            const float m = stoch ? update_mask_at(a.seed, a.rate, tc.n + a.n_offset, a.H, a.W, Y, X) : 1.f;
            const int SS = g.S + 2, per = (g.R + 2) * SS;
            float *yn = a.y + (size_t)tc.n * C * plane + (size_t)Y * a.W + X;
#pragma unroll
            for (int cc = 0; cc < CPP; ++cc) {
                const int c = CPP * part + cc;
                const float xc = XS[c * per + (r + 1) * SS + s + 1];
                yn[(size_t)c * plane] = m != 0.f ? xc + u[cc] : xc;
            }
        }
        if constexpr (GROWING) {
            // the alive mask in the epilogue (ncaops/nca_step.cuh:693-727 semantics): a = (maxpool3(x_alpha) > 0.1) &
            // (maxpool3(unmasked new alpha) > 0.1), cells outside the grid ignored; y = a ? unmasked y : 0
            static_assert(!GROWING || CPP > 3, "the alpha channel belongs to part 0");
            const int SS = g.S + 2, per = (g.R + 2) * SS;
            float yv[CPP];
            const float m = valid && stoch ? update_mask_at(a.seed, a.rate, tc.n + a.n_offset, a.H, a.W, tc.y0 + r,
                                                            tc.x0 + s) : 1.f;
#pragma unroll
            for (int cc = 0; cc < CPP; ++cc) {
                const float xc = XS[(CPP * part + cc) * per + (r + 1) * SS + s + 1];
                yv[cc] = m != 0.f ? xc + u[cc] : xc;
            }
            if (part == 0) {
                XA[lt] = valid ? XS[3 * per + (r + 1) * SS + s + 1] : -1.f;
                YA[lt] = valid ? yv[3] : -1.f;
            }
            __syncthreads();
            if (inner) {
                float mx = -1.f, my = -1.f;
#pragma unroll
                for (int dy = -1; dy <= 1; ++dy)
#pragma unroll
                    for (int dx = -1; dx <= 1; ++dx) {
                        const int q = (r + dy) * GE_S + (s + dx);
                        mx = fmaxf(mx, XA[q]);
                        my = fmaxf(my, YA[q]);
                    }
                const bool live = mx > 0.1f && my > 0.1f;
                float *yn = a.y + ((size_t)tc.n * C + CPP * part) * plane + (cell - (size_t)tc.n * plane);
#pragma unroll
                for (int cc = 0; cc < CPP; ++cc)
                    yn[(size_t)cc * plane] = live ? yv[cc] : 0.f;
                if (part == 0)
                    a.alive_out[cell] = live ? 1 : 0;
            }
        }
        if constexpr (TC)
            umma::fence_before_sync();
        __syncthreads();  // XS, P and TMEM are reused by the next tile
    }
    if constexpr (TC) {
        __syncthreads();
        umma::fence_after_sync();
        if (warp == 0)
            umma::tmem_dealloc(tmem, D::FWD_TMEM);
        if (failed && tid == 0)
            set_device_error(1);
    }
}

// ================================================================ backward
// Per tile: recompute p and h, gm = gy m (a); dh = (gm W2) [h > 0]; dp = dh W1 -> dp scratch (N, 4C, H, W);
// dW1' += dh^T p' (column PIN of p' is 1: db1), dW2^T += relu(h)^T gm, accumulated per NCA segment (TMEM in TF32 mode,
// registers of threads j < HID in fp32 mode) and written to partial slot (CTA + NCA).
template <class D>
__device__ __forceinline__ void write_partial_row(float *out, int j, const float *dw1_row, float db1, const float *dw2_col,
                                                  bool add)
{
    if (!add) {
        for (int f = 0; f < D::PIN; ++f)
            out[j * D::PIN + f] = dw1_row[f];
        out[D::HID * D::PIN + j] = db1;
        for (int c = 0; c < D::C; ++c)
            out[D::HID * (D::PIN + 1) + c * D::HID + j] = dw2_col[c];
        return;
    }
    float o1[D::PIN], o2[D::C];  // the old values first (all in flight), then the sums
#pragma unroll
    for (int f = 0; f < D::PIN; ++f)
        o1[f] = out[j * D::PIN + f];
    const float ob = out[D::HID * D::PIN + j];
#pragma unroll
    for (int c = 0; c < D::C; ++c)
        o2[c] = out[D::HID * (D::PIN + 1) + c * D::HID + j];
#pragma unroll
    for (int f = 0; f < D::PIN; ++f)
        out[j * D::PIN + f] = o1[f] + dw1_row[f];
    out[D::HID * D::PIN + j] = ob + db1;
#pragma unroll
    for (int c = 0; c < D::C; ++c)
        out[D::HID * (D::PIN + 1) + c * D::HID + j] = o2[c] + dw2_col[c];
}

// Per tile pixel: gm = gy m (a) (growing: a = the alive mask of the forward), 16 channels, fp32. Returns whether the
// pixel is valid and (growing) alive.
template <int C, bool GROWING>
__device__ __forceinline__ bool load_gm(float (&gm)[16], const StepArgs &a, const TileCoord &tc, int Y, int X,
                                        bool valid, bool stoch)
{
#pragma unroll
    for (int c = 0; c < 16; ++c)
        gm[c] = 0.f;
    if (!valid)
        return false;
    const size_t plane = (size_t)a.H * a.W;
    float m = stoch ? update_mask_at(a.seed, a.rate, tc.n + a.n_offset, a.H, a.W, Y, X) : 1.f;
    const bool live = !GROWING || a.alive[(size_t)tc.n * plane + (size_t)Y * a.W + X];
    if (!live)
        m = 0.f;
    if (m == 0.f)
        return live;
    const float *gyn = a.gy + (size_t)tc.n * C * plane + (size_t)Y * a.W + X;
#pragma unroll
    for (int c = 0; c < C; ++c)
        gm[c] = __ldg(gyn + (size_t)c * plane);
    return live;
}

// fp32 mode: the MLP on CUDA cores in fp32, weight gradients accumulated by threads j < HID in registers.
template <int C, int HID, bool GROWING, bool PERM = false>
__global__ void __launch_bounds__(128, 1) bwd_kernel_cc(StepArgs a)
{
    a.seed = step_seed_of(a);
    using D = Dims<C, HID>;
    extern __shared__ __align__(128) float smem[];
    float *W1s = smem, *W2s = W1s + D::W1S, *P = W2s + D::W2S, *G = P + D::P;
    float *RHt = G + D::G, *DHt = RHt + D::HID * D::HT;
    float *XS = RHt;  // the halo tile is dead before RHt is written

    const int tid = threadIdx.x;
    const TileGeom g = make_geom(a.H, a.W, GROWING);
    const int64_t T = (int64_t)a.N * g.tiles_per_image;
    int64_t t0, t1;
    cta_range(T, gridDim.x, blockIdx.x, &t0, &t1);
    const bool stoch = a.rate < 1.f;
    const size_t plane = (size_t)a.H * a.W;
    float acc1[D::PIN], accb = 0.f, acc2[C];
#pragma unroll
    for (int f = 0; f < D::PIN; ++f)
        acc1[f] = 0.f;
#pragma unroll
    for (int c = 0; c < C; ++c)
        acc2[c] = 0.f;
    int cur_k = -1;
    auto flush = [&](int k) {
        if (tid < HID)
            write_partial_row<D>(a.partial + (size_t)(blockIdx.x + k) * D::PART, tid, acc1, accb, acc2, a.partial_add != 0);
#pragma unroll
        for (int f = 0; f < D::PIN; ++f)
            acc1[f] = 0.f;
#pragma unroll
        for (int c = 0; c < C; ++c)
            acc2[c] = 0.f;
        accb = 0.f;
    };
    __shared__ uint32_t sw[4];
    uint32_t live_bits = 0;  // growing: whether tiles [live_base, live_base + 32) hold an alive pixel
    int64_t live_base = t0 - 64;
    bool staged = false;
    for (int64_t t = t0; t < t1; ++t) {
        const TileCoord tc = tile_coord<PERM>(t, g, a);
        if (tc.k != cur_k) {
            if (cur_k >= 0)
                flush(cur_k);
            __syncthreads();
            cur_k = tc.k;
            staged = false;
        }
        if (GROWING) {  // dead tile (block-uniform): nothing to add, its dp is not read
            if (t >= live_base + 32) {  // the alive bytes of 32 tiles' pixels, all loads in flight together
                live_base = t;
                uint32_t mine = 0;
#pragma unroll
                for (int i = 0; i < 32; ++i)
                    mine |= t + i < t1 && pixel_alive<PERM>(a, g, t + i, tid) ? 1u << i : 0u;
                live_bits = block_or_128(mine, sw);
            }
            if (!((live_bits >> (t - live_base)) & 1u))
                continue;
        }
        if (!staged) {  // the NCA's weights, at its first live tile
            stage_weights<D, false>(W1s, W2s, a.w1 + (size_t)tc.k * HID * D::PIN, a.b1 + (size_t)tc.k * HID,
                                    a.w2 + (size_t)tc.k * C * HID);
            staged = true;
        }
        load_halo_async<D>(XS, a.x, tc.n, g, tc.y0, tc.x0);
        const int r = tid / g.S, s = tid - r * g.S;
        const bool valid = tid < g.R * g.S && tc.y0 + r < a.H && tc.x0 + s < a.W;
        const int Y = tc.y0 + r, X = tc.x0 + s;
        float gm[16];
        load_gm<C, GROWING>(gm, a, tc, Y, X, valid, stoch);
#pragma unroll
        for (int q = 0; q < 4; ++q)
            *reinterpret_cast<float4 *>(G + q * D::PLANE + tid * 4) = make_float4(gm[4 * q], gm[4 * q + 1], gm[4 * q + 2], gm[4 * q + 3]);
        cp_async_wait_all();
        __syncthreads();
        perceive_tile<D, false>(P, XS, g, tid, valid);
        __syncthreads();
        float p[D::PIN], dpv[D::PIN];
#pragma unroll
        for (int f = 0; f < D::PIN; ++f) {
            p[f] = P[(f / 4) * D::PLANE + tid * 4 + (f % 4)];
            dpv[f] = 0.f;
        }
        for (int j = 0; j < HID; ++j) {
            const float *wrow = W1s + j * 4;
            float h = wrow[(D::PIN / 4) * HID * 4];
#pragma unroll
            for (int f = 0; f < D::PIN; ++f)
                h = fmaf(wrow[(f / 4) * HID * 4 + (f % 4)], p[f], h);
            const float *w2c = W2s + (j / 4) * D::CP * 4 + (j % 4);
            float dh = 0.f;
#pragma unroll
            for (int c = 0; c < C; ++c)
                dh = fmaf(w2c[c * 4], gm[c], dh);
            dh = h > 0.f ? dh : 0.f;
            RHt[j * D::HT + tid] = valid ? fmaxf(h, 0.f) : 0.f;
            DHt[j * D::HT + tid] = dh;
#pragma unroll
            for (int f = 0; f < D::PIN; ++f)
                dpv[f] = fmaf(wrow[(f / 4) * HID * 4 + (f % 4)], dh, dpv[f]);
        }
        if (valid) {
            float *dpn = a.dp + (size_t)tc.n * D::PIN * plane + (size_t)Y * a.W + X;
#pragma unroll
            for (int f = 0; f < D::PIN; ++f)
                dpn[(size_t)f * plane] = dpv[f];
        }
        __syncthreads();
        if (tid < HID)  // weight gradients of hidden unit j = tid over the tile's pixels, fixed order
            for (int q = 0; q < D::TILE; ++q) {
                const float dh = DHt[tid * D::HT + q], rh = RHt[tid * D::HT + q];
#pragma unroll
                for (int f = 0; f < D::PIN; ++f)
                    acc1[f] = fmaf(dh, P[(f / 4) * D::PLANE + q * 4 + (f % 4)], acc1[f]);
                accb += dh;
#pragma unroll
                for (int c = 0; c < C; ++c)
                    acc2[c] = fmaf(G[(c / 4) * D::PLANE + q * 4 + (c % 4)], rh, acc2[c]);
            }
        __syncthreads();
    }
    if (cur_k >= 0)
        flush(cur_k);
}

// Stage one NCA's backward weights: W1' (HID x KP, K-major: B of p -> h), W1^T (PIN x HID, K-major: B of dh -> dp),
// W2^T (HID x 16, K-major: B of gm -> dh), all TF32, chunk-planar without swizzle.
template <class D>
__device__ __forceinline__ void stage_bwd_weights(float *W1s, float *W1T, float *W2T, const float *w1, const float *b1,
                                                  const float *w2, int t0 = threadIdx.x, int nt = blockDim.x,
                                                  int gm_off = 0)
{
    // gm_off: W2T's K index of channel 0 (the row kernel keeps gm at feature PIN + 2 of its tensor-memory operand)
    for (int e = t0; e < D::HID * D::KP; e += nt) {
        const int j = e / D::KP, f = e % D::KP;
        float v = 0.f;
        if (f < D::PIN)
            v = tf32_rna(w1[j * D::PIN + f]);
        else if (f == D::PIN)
            v = tf32_rna(b1[j]);
        else if (f == D::PIN + 1)
            v = tf32_rna(b1[j] - tf32_rna(b1[j]));
        W1s[(f / 4) * D::HID * 4 + j * 4 + (f % 4)] = v;
        if (f < D::PIN)
            W1T[(j / 4) * D::PIN * 4 + f * 4 + (j % 4)] = v;
    }
    for (int e = t0; e < D::HID * D::CP; e += nt) {
        const int j = e / D::CP, kk = e % D::CP, c = kk - gm_off;
        W2T[(kk / 4) * D::HID * 4 + j * 4 + (kk % 4)] = c >= 0 && c < D::C ? tf32_rna(w2[c * D::HID + j]) : 0.f;
    }
}

// Eight consecutive values v[0..7] of MN index mn0 (mn0 % 8 == 0) at K row k of a swizzled MN-major tile.
__device__ __forceinline__ void st_sw32x8(float *tile, int mn0, int k, int krows, const float *v)
{
    float *dst = tile + umma::sw32_offset(mn0, k, krows) / 4;
    *reinterpret_cast<float4 *>(dst) = make_float4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<float4 *>(dst + 4) = make_float4(v[4], v[5], v[6], v[7]);
}

// TF32 mode. One CTA of BWD_TILE_PARTS parts of 128 threads: thread lt of every part owns tile pixel lt (TMEM lane lt);
// the CUDA-core work of each phase is split by part (part p: channels [CPP p, CPP (p+1)) of the halo, perception and
// gm, hidden units [HPP p, HPP (p+1)) of the epilogues, dp features [4 CPP p, 4 CPP (p+1)) of the dp stores), so that
// four warps of every SM sub-partition share each phase instead of one. Thread 0 issues the contractions. Per tile:
//   1. halo tile (cp.async) and gm; p' and gm into TMEM (A operands) and into swizzled MN-major smem (weight grads);
//   2. H = p' W1'^T and DHP = gm W2 (A from TMEM);
//   3. relu(h) -> smem (swizzled), dh = DHP [h > 0] -> TMEM (A of dp);
//   4. dW2^T += relu(h)^T gm and DP = dh W1 (A from TMEM);
//   5. dh -> smem (swizzled, over relu(h)); dW1' += dh^T p' while dp is stored to the dp scratch.
// The bias features of p' (1 at PIN and PIN + 1, zeros up to the operand widths) and gm's channels C..15 are constant:
// written once.
template <int C, int HID, bool GROWING, bool PERM = false>
__global__ void __launch_bounds__(128 * BWD_TILE_PARTS, 1) bwd_kernel_tc(StepArgs a)
{
    constexpr int NP = BWD_TILE_PARTS, NT = 128 * NP, CPP = C / NP, HPP = HID / NP, PPP = 4 * CPP;
    static_assert(C % NP == 0 && HPP % 8 == 0, "tile backward parts");
    a.seed = step_seed_of(a);
    using D = Dims<C, HID>;
    constexpr int KP16 = ((D::KP + 15) / 16) * 16;  // TMEM columns of p' (A of p -> h)
    extern __shared__ __align__(128) unsigned char smem_raw[];
    unsigned char *base = smem_raw + ((1024 - (umma::smem_u32(smem_raw) & 1023)) & 1023);
    float *W1s = reinterpret_cast<float *>(base), *W1T = W1s + D::W1S, *W2T = W1T + D::W1T;
    float *RHDH = reinterpret_cast<float *>(base + D::BWD_W), *PSW = RHDH + D::RHDH, *GSW = PSW + D::PSW;
    float *XSP = GSW + D::GSW;  // the prefetched halo
    // bar: the contractions issued by thread 0; bar2: the dW2 chain, issued by thread 32 (another SM sub-partition)
    // beside thread 0's dp chain
    uint64_t *bar = reinterpret_cast<uint64_t *>(XSP + C * D::xs_pos(GROWING)), *bar2 = bar + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bar + 2);

    const int tid = threadIdx.x, warp = tid / 32, part = tid / 128, lt = tid % 128;
    const TileGeom g = make_geom(a.H, a.W, GROWING);
    const int64_t T = (int64_t)a.N * g.tiles_per_image;
    int64_t t0, t1;
    cta_range(T, gridDim.x, blockIdx.x, &t0, &t1);
    const bool stoch = a.rate < 1.f;
    const size_t plane = (size_t)a.H * a.W;

    // the swizzled gm tile holds 16 channels in a 32-wide block: zero it once (its other lanes are never written);
    // the constant features of the p' tile: 1 at PIN and PIN + 1, zeros up to NPW
    for (int e = tid; e < D::GSW; e += NT)
        GSW[e] = 0.f;
    for (int e = tid; e < 128 * (D::NPW - D::PIN); e += NT) {
        const int q = e / (D::NPW - D::PIN), f = D::PIN + e % (D::NPW - D::PIN);
        PSW[umma::sw32_offset(f, q, 128) / 4] = f < D::PIN + 2 ? 1.f : 0.f;
    }
    if (tid == 0) {
        umma::mbar_init(bar, 1);
        umma::mbar_init(bar2, 1);
        umma::fence_mbar_init();
    }
    if (warp == 0) {
        umma::tmem_alloc(tmem_slot, D::BWD_TMEM);
        umma::tmem_relinquish();
    }
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    const uint32_t lane_base = umma::tmem_addr(tmem, warp, 0);
    if (part == 0) {  // constant TMEM columns: gm channels C..15 (zeros), p' features PIN .. KP16 (1, 1, zeros)
        float z[16], pb[KP16 - D::PIN];
#pragma unroll
        for (int e = 0; e < 16; ++e)
            z[e] = 0.f;
#pragma unroll
        for (int e = 0; e < KP16 - D::PIN; ++e)
            pb[e] = e < 2 ? 1.f : 0.f;
        umma::tmem_st16(lane_base + D::T_G, z);
#pragma unroll
        for (int e = 0; e < KP16 - D::PIN; e += 8)
            umma::tmem_st8(lane_base + D::T_P + D::PIN + e, pb + e);
        umma::tmem_wait_st();
    }
    const uint32_t sW1 = umma::smem_u32(W1s), sW1T = umma::smem_u32(W1T), sW2T = umma::smem_u32(W2T);
    const uint32_t sRH = umma::smem_u32(RHDH), sP = umma::smem_u32(PSW), sG = umma::smem_u32(GSW);

    uint32_t phase = 0, phase2 = 0;
    int cur_k = -1;
    bool started = false, failed = false;
    auto wait_mma = [&](bool both = false) {  // both: the dW2 chain (bar2) too
        bool ok = umma::mbar_wait(bar, phase);
        phase ^= 1;
        if (both) {
            ok &= umma::mbar_wait(bar2, phase2);
            phase2 ^= 1;
        }
        if (!__syncthreads_and(ok))
            failed = true;
        umma::fence_after_sync();
        return !failed;
    };
    // this CTA's weight gradients of NCA k -> partial slot (blockIdx.x + k), by part 0; zeros when no tile of NCA k ran
    // here (growing: all dead)
    auto flush = [&](int k, bool have) {
        if (part != 0)
            return;
        float row[((D::PIN + 1 + 15) / 16) * 16], col[16];
#pragma unroll
        for (int cc = 0; cc < (D::PIN + 1 + 15) / 16; ++cc) {
            float v[16];
            umma::tmem_ld16(lane_base + D::T_ACC1 + cc * 16, v);
            umma::tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 16; ++e)
                row[cc * 16 + e] = have ? v[e] : 0.f;
        }
        umma::tmem_ld16(lane_base + D::T_ACC2, col);
        umma::tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 16; ++e)
            col[e] = have ? col[e] : 0.f;
        if (lt < HID)
            write_partial_row<D>(a.partial + (size_t)(blockIdx.x + k) * D::PART, lt, row, row[D::PIN], col,
                                 a.partial_add != 0);
        umma::fence_before_sync();
    };

    __shared__ uint32_t sw[NT / 32];
    uint32_t live_bits = 0;  // growing: whether tiles [live_base, live_base + 32) hold an alive pixel
    int64_t live_base = t0 - 64;
    bool staged = false;
    // every NCA this CTA's tile range overlaps gets its partial slot written (the reduction reads them all)
    const int k_last = t1 > t0 ? tile_coord<PERM>(t1 - 1, g, a).k : -1;
    if (t1 > t0)
        cur_k = tile_coord<PERM>(t0, g, a).k;
    // the lane's pixel within a tile (row, column), and whether it exists
    const int lr = lt / g.S, ls = lt - lr * g.S;
    const bool lin = lt < g.R * g.S;
    // the next tile with an alive pixel from t on (growing; a dead tile adds nothing and its dp is not read), or t1
    auto next_live = [&](int64_t t) {
        if (GROWING) {
            while (t < t1) {
                if (t >= live_base + 32) {  // the alive bytes of 32 tiles' pixels, part p the tiles p, p + NP, .., all
                    live_base = t;          // loads in flight together
                    uint32_t mine = 0;
#pragma unroll
                    for (int i = part; i < 32; i += NP) {
                        bool al = false;
                        if (lin && t + i < t1) {
                            const TileCoord tq = tile_coord<PERM>(t + i, g, a);
                            const int Yq = tq.y0 + lr, Xq = tq.x0 + ls;
                            al = Yq < a.H && Xq < a.W && a.alive[((size_t)tq.n * a.H + Yq) * a.W + Xq] != 0;
                        }
                        mine |= al ? 1u << i : 0u;
                    }
                    live_bits = block_or<NT>(mine, sw);
                }
                const uint32_t rest = live_bits >> (t - live_base);
                if (rest != 0)
                    return t + __ffs(rest) - 1;
                t = live_base + 32;
            }
        }
        return t < t1 ? t : t1;
    };
    // a tile's inputs: its halo (cp.async into XS) and this part's gm channels (registers). With the dedicated buffer
    // (the tile's halo fits it) the next tile's inputs are requested right after the current tile's perception, so
    // that they arrive during its contractions; otherwise the halo goes to RHDH at the start of its own tile.
    const bool prefetch = (g.R + 2) * (g.S + 2) <= D::xs_pos(GROWING);
    float *XS = prefetch ? XSP : RHDH;
    // The request is in two steps, so that no thread waits on memory in it: request() copies the halo, loads the
    // pixel's alive byte (growing) and draws its update mask; request_gm(), some phases later, reads that byte and
    // loads gy of this part's channels where gm = gy m a is not 0.
    float gmn[CPP];
    bool livn = false;     // the requested tile's pixel is valid and (growing) alive
    size_t gq = 0;         // ... its offset in a channel plane of gy (image base included)
    bool vq = false;       // ... is valid
    uint8_t aq = 1;        // ... alive byte (growing)
    float mq = 1.f;        // ... update mask
    auto request = [&](int64_t tn) {
        const TileCoord tq = tile_coord<PERM>(tn, g, a);
        load_halo_async<D, NT>(XS, a.x, tq.n, g, tq.y0, tq.x0);
        const int Yq = tq.y0 + lr, Xq = tq.x0 + ls;
        vq = lin && Yq < a.H && Xq < a.W;
        gq = (size_t)tq.n * C * plane + (size_t)Yq * a.W + Xq;
        if (GROWING)
            aq = vq ? a.alive[(size_t)tq.n * plane + (size_t)Yq * a.W + Xq] : 0;
        mq = vq && stoch ? update_mask_at(a.seed, a.rate, tq.n + a.n_offset, a.H, a.W, Yq, Xq) : 1.f;
    };
    auto request_gm = [&]() {
        livn = vq && (!GROWING || aq != 0);
        const bool act = livn && mq != 0.f;
        const float *gyq = a.gy + gq + (size_t)(CPP * part) * plane;
#pragma unroll
        for (int cc = 0; cc < CPP; ++cc)
            gmn[cc] = act ? __ldg(gyq + (size_t)cc * plane) : 0.f;
    };
    int64_t t = next_live(t0);
    if (prefetch && t < t1) {
        request(t);
        request_gm();
    }
    while (t < t1) {
        const TileCoord tc = tile_coord<PERM>(t, g, a);
        if (tc.k != cur_k) {
            flush(cur_k, started);
            for (int kk = cur_k + 1; kk < tc.k; ++kk)  // NCAs whose tiles here are all dead
                flush(kk, false);
            __syncthreads();
            cur_k = tc.k;
            started = false;
            staged = false;
        }
        if (!staged) {  // the NCA's weights, at its first live tile (the flush above needs none)
            stage_bwd_weights<D>(W1s, W1T, W2T, a.w1 + (size_t)tc.k * HID * D::PIN, a.b1 + (size_t)tc.k * HID,
                                 a.w2 + (size_t)tc.k * C * HID);
            staged = true;
        }
        // ---- 1. inputs (requested one tile ahead when prefetching)
        if (!prefetch) {
            request(t);
            request_gm();
        }
        const int r = lt / g.S, s = lt - r * g.S;
        const bool valid = lt < g.R * g.S && tc.y0 + r < a.H && tc.x0 + s < a.W;
        const int Y = tc.y0 + r, X = tc.x0 + s;
        // the pixel's dp is stored where the adjoint reads it: valid pixels, growing: alive ones (dp = 0 elsewhere)
        const bool store_dp = livn;
#pragma unroll
        for (int cc = 0; cc < CPP; ++cc) {  // gm of this part's channels -> TMEM G and the swizzled gm tile
            const float gv = tf32_bias(gmn[cc]);
            umma::tmem_st1(lane_base + D::T_G + CPP * part + cc, gv);
            GSW[umma::sw32_offset(CPP * part + cc, lt, 128) / 4] = gv;
        }
        cp_async_wait_all();
        __syncthreads();
        {  // p' of this part's channels -> TMEM P and the swizzled p' tile
            const int SS = g.S + 2, per = (g.R + 2) * SS;
#pragma unroll
            for (int cc = 0; cc < CPP; ++cc) {
                const int c = CPP * part + cc;
                float4 p = make_float4(0.f, 0.f, 0.f, 0.f);
                if (valid) {
                    float v[3][3];
                    const float *b = XS + c * per + r * SS + s;
#pragma unroll
                    for (int dy = 0; dy < 3; ++dy)
#pragma unroll
                        for (int dx = 0; dx < 3; ++dx)
                            v[dy][dx] = b[dy * SS + dx];
                    p = perceive3x3(v);
                }
                const float pv[4] = {tf32_bias(p.x), tf32_bias(p.y), tf32_bias(p.z), tf32_bias(p.w)};
                umma::tmem_st4(lane_base + D::T_P + 4 * c, pv);
                *reinterpret_cast<float4 *>(PSW + umma::sw32_offset(4 * c, lt, 128) / 4) = make_float4(pv[0], pv[1], pv[2], pv[3]);
            }
        }
        umma::tmem_wait_st();
        umma::fence_proxy_async();
        umma::fence_before_sync();
        __syncthreads();
        // the halo is consumed: the next live tile's inputs may land in it during this tile's contractions
        const int64_t t_next = next_live(t + 1);
        if (prefetch && t_next < t1)
            request(t_next);
        // ---- 2. H = p' W1'^T, DHP = gm W2 (A from TMEM)
        if (tid == 0) {
            umma::fence_after_sync();
#pragma unroll
            for (int ks = 0; ks < D::KP / 8; ++ks)
                umma::mma_ts(tmem + D::T_H, tmem + D::T_P + ks * 8, umma::smem_desc(sW1 + ks * 2 * HID * 16, HID * 16, 128),
                             umma::idesc_tf32(128, HID, false, false), ks > 0);
#pragma unroll
            for (int ks = 0; ks < 2; ++ks)
                umma::mma_ts(tmem + D::T_DHP, tmem + D::T_G + ks * 8, umma::smem_desc(sW2T + ks * 2 * HID * 16, HID * 16, 128),
                             umma::idesc_tf32(128, HID, false, false), ks > 0);
            umma::commit(bar);
        }
        if (!wait_mma())
            break;
        // ---- 3. relu(h) -> smem (swizzled MN-major), dh -> TMEM (this part's hidden units)
#pragma unroll
        for (int q = 0; q < HPP / 8; ++q) {
            const int j0 = HPP * part + 8 * q;
            float h[8], d[8];
            umma::tmem_ld8(lane_base + D::T_H + j0, h);
            umma::tmem_ld8(lane_base + D::T_DHP + j0, d);
            umma::tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                d[e] = h[e] > 0.f ? tf32_bias(d[e]) : 0.f;
                h[e] = tf32_bias(fmaxf(h[e], 0.f));
            }
            st_sw32x8(RHDH, j0, lt, 128, h);
            umma::tmem_st8(lane_base + D::T_H + j0, d);
        }
        umma::tmem_wait_st();
        umma::fence_proxy_async();
        umma::fence_before_sync();
        __syncthreads();
        if (prefetch && t_next < t1)  // the next tile's alive byte has arrived by now: its gy loads
            request_gm();
        // ---- 4. dW2^T += relu(h)^T gm (K = pixels, MN-major; thread 32), DP = dh W1 (A from TMEM; thread 0)
        if (tid == 32) {
            umma::fence_after_sync();
#pragma unroll
            for (int ks = 0; ks < 16; ++ks)
                umma::mma_ss(tmem + D::T_ACC2, umma::smem_desc(sRH + ks * 1024, 128 * 128, 512, umma::LAYOUT_SW128_32B),
                             umma::smem_desc(sG + ks * 1024, 128 * 128, 512, umma::LAYOUT_SW128_32B),
                             umma::idesc_tf32(128, 16, true, true), started || ks > 0);
            umma::commit(bar2);
        }
        if (tid == 0) {
            umma::fence_after_sync();
#pragma unroll
            for (int ks = 0; ks < HID / 8; ++ks)
                umma::mma_ts(tmem + D::T_P, tmem + D::T_H + ks * 8, umma::smem_desc(sW1T + ks * 2 * D::PIN * 16, D::PIN * 16, 128),
                             umma::idesc_tf32(128, D::PIN, false, false), ks > 0);
            umma::commit(bar);
        }
        if (!wait_mma(true))
            break;
        // ---- 5. dh -> smem (swizzled, over relu(h)); dW1' += dh^T p'; dp -> dp scratch
#pragma unroll
        for (int q = 0; q < HPP / 8; ++q) {
            const int j0 = HPP * part + 8 * q;
            float d[8];
            umma::tmem_ld8(lane_base + D::T_H + j0, d);
            umma::tmem_wait_ld();
            st_sw32x8(RHDH, j0, lt, 128, d);
        }
        umma::fence_proxy_async();
        umma::fence_before_sync();
        __syncthreads();
        if (tid == 0) {
            umma::fence_after_sync();
#pragma unroll
            for (int ks = 0; ks < 16; ++ks)
                umma::mma_ss(tmem + D::T_ACC1, umma::smem_desc(sRH + ks * 1024, 128 * 128, 512, umma::LAYOUT_SW128_32B),
                             umma::smem_desc(sP + ks * 1024, 128 * 128, 512, umma::LAYOUT_SW128_32B),
                             umma::idesc_tf32(128, D::NPW, true, true), started || ks > 0);
            umma::commit(bar);
        }
        started = true;
        {  // this part's dp features
            float *dpn = a.dp + (size_t)tc.n * D::PIN * plane + (size_t)Y * a.W + X;
            float v[PPP];
#pragma unroll
            for (int q = 0; q < PPP / 4; ++q)
                umma::tmem_ld4(lane_base + D::T_P + PPP * part + 4 * q, v + 4 * q);
            umma::tmem_wait_ld();
            if (store_dp)
#pragma unroll
                for (int e = 0; e < PPP; ++e)
                    dpn[(size_t)(PPP * part + e) * plane] = v[e];
        }
        umma::fence_before_sync();
        if (!wait_mma())  // dW1' done: RHDH / PSW / TMEM are free for the next tile
            break;
        t = t_next;
    }
    if (cur_k >= 0 && !failed) {
        flush(cur_k, started);
        for (int kk = cur_k + 1; kk <= k_last; ++kk)
            flush(kk, false);
    }
    cp_async_wait_all();  // a prefetch issued before a failed wait lands before the block ends
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    if (warp == 0)
        umma::tmem_dealloc(tmem, D::BWD_TMEM);
    if (failed && tid == 0)
        set_device_error(1);
}

// gx = gy a + sum_f P_f^T dp_f: the transpose of the circular perception (ncaops/nca_step.cuh:1195-1263), fp32, fixed
// tap order. Block: 32 x 8 output pixels of one image, all channels; dp halo staged in shared memory.
constexpr int ADJ_TW = 32, ADJ_TH = 8, ADJ_HALVES = 2;
template <int C, bool GROWING>
__global__ void __launch_bounds__(256) adjoint_kernel(const float *__restrict__ dp, const float *__restrict__ gy,
                                                      const uint8_t *__restrict__ alive, float *__restrict__ gx, int N,
                                                      int H, int W)
{
    // the dp halo is staged in ADJ_HALVES passes of PIN / ADJ_HALVES features (channels [c0, c0 + C / ADJ_HALVES)), so
    // that several blocks of 256 threads fit an SM (dead blocks, the common case of a growing grid, are latency-bound)
    constexpr int PIN = 4 * C, HW_ = ADJ_TW + 2, HH_ = ADJ_TH + 2, NPOS = HH_ * HW_, FH = PIN / ADJ_HALVES;
    constexpr int NQ = (NPOS + 255) / 256;  // halo positions per thread
    static_assert(C % ADJ_HALVES == 0, "adjoint feature passes");
    extern __shared__ __align__(16) float sdp[];  // [FH][HH_][HW_]
    __shared__ uint8_t sal[GROWING ? NPOS : 1];   // growing: the alive mask of the halo
    const uint32_t tiles_x = (W + ADJ_TW - 1) / ADJ_TW, per_image = tiles_x * ((H + ADJ_TH - 1) / ADJ_TH);
    const int64_t plane = (int64_t)H * W;
    const uint32_t total = (uint32_t)N * per_image;  // < 2^31 (the host checks)
    // persistent over the blocks b = blockIdx.x, blockIdx.x + gridDim.x, .. (block b: image b / per_image, tile
    // b % per_image); growing: this thread's alive bytes of the next block's halo are loaded one block ahead
    auto origin = [&](uint32_t b, int &n, int &y0, int &x0) {
        const uint32_t nn = b / per_image, tb = b - nn * per_image, ty = tb / tiles_x;
        n = (int)nn;
        y0 = (int)ty * ADJ_TH;
        x0 = (int)(tb - ty * tiles_x) * ADJ_TW;
    };
    auto halo_alive = [&](uint32_t b, uint8_t (&v)[NQ]) {
        int n, y0, x0;
        origin(b, n, y0, x0);
        const uint8_t *an = alive + (int64_t)n * plane;
#pragma unroll
        for (int q = 0; q < NQ; ++q) {
            const int e = threadIdx.x + 256 * q, r = e / HW_, s = e - r * HW_;
            v[q] = e < NPOS ? an[(int64_t)wrap_near(y0 - 1 + r, H) * W + wrap_near(x0 - 1 + s, W)] : 0;
        }
    };
    uint8_t nxt[NQ];
    if (GROWING && blockIdx.x < total)
        halo_alive(blockIdx.x, nxt);
    for (uint32_t b = blockIdx.x; b < total; b += gridDim.x) {
        int n, y0, x0;
        origin(b, n, y0, x0);
        const int r = threadIdx.x / ADJ_TW, s = threadIdx.x % ADJ_TW, Y = y0 + r, X = x0 + s;
        const bool out = Y < H && X < W;
        bool gate = false;  // growing, block with dead cells in its halo: read dp at alive cells only
        if (GROWING) {
            // dp is 0 wherever the cell is dead (gm = 0 there); the backward skips all-dead tiles without writing their
            // dp, so dp is read at alive cells only, and a block with no alive cell in its halo has gx = 0
            bool some = false, all = true;  // of this thread's halo cells
#pragma unroll
            for (int q = 0; q < NQ; ++q) {
                const int e = threadIdx.x + 256 * q;
                if (e < NPOS) {
                    sal[e] = nxt[q];
                    some |= nxt[q] != 0;
                    all &= nxt[q] != 0;
                }
            }
            if (b + gridDim.x < total)
                halo_alive(b + gridDim.x, nxt);
            const bool any_alive = __syncthreads_or(some), all_alive = __syncthreads_and(all);
            if (!any_alive) {
                if (out) {
                    float *g = gx + (int64_t)n * C * plane + (int64_t)Y * W + X;
#pragma unroll
                    for (int c = 0; c < C; ++c)
                        g[(int64_t)c * plane] = 0.f;
                }
                continue;
            }
            gate = !all_alive;
        }
        const bool live = out && (!GROWING || alive[(int64_t)n * plane + (int64_t)Y * W + X]);
#pragma unroll 1
        for (int hf = 0; hf < ADJ_HALVES; ++hf) {
            // dp halo of features [hf FH, (hf + 1) FH) -> sdp: thread t takes halo positions t, t + 256; its address is
            // computed once per position, then each feature plane is copied from it asynchronously (zeros where a
            // growing halo cell is dead)
            const float *dpn = dp + ((int64_t)n * PIN + hf * FH) * plane;
#pragma unroll
            for (int q = 0; q < NQ; ++q) {
                const int pos = threadIdx.x + 256 * q;
                if (pos < NPOS) {
                    const int hr = pos / HW_, hs = pos - hr * HW_;
                    const float *src = dpn + (int64_t)wrap_near(y0 - 1 + hr, H) * W + wrap_near(x0 - 1 + hs, W);
                    const bool ld = !gate || sal[GROWING ? pos : 0];
#pragma unroll 16
                    for (int f = 0; f < FH; ++f)
                        cp_async4_zfill(sdp + f * NPOS + pos, src + (int64_t)f * plane, ld);
                }
            }
            cp_async_wait_all();
            __syncthreads();
            if (out) {
                const int64_t pix = (int64_t)Y * W + X;
#pragma unroll 1
                for (int cl = 0; cl < C / ADJ_HALVES; ++cl) {
                    float acc = 0.f;
#pragma unroll
                    for (int f = 0; f < 4; ++f)
#pragma unroll
                        for (int i = 0; i < 3; ++i)
#pragma unroll
                            for (int j = 0; j < 3; ++j) {
                                // output (Y, X) receives tap (i, j) of the pixel (Y - (i - 1), X - (j - 1))
                                const float k = filter_tap(f, i, j);
                                if (k != 0.f)
                                    acc = fmaf(k, sdp[((4 * cl + f) * HH_ + (r + 1 - (i - 1))) * HW_ + (s + 1 - (j - 1))], acc);
                            }
                    const int64_t o = ((int64_t)n * C + hf * (C / ADJ_HALVES) + cl) * plane + pix;
                    gx[o] = (live ? gy[o] : 0.f) + acc;
                }
            }
            __syncthreads();  // sdp (and sal) are rewritten by the next pass or block
        }
    }
}

// The CTAs [c0, c1] of a launch whose unit ranges (bands bd) overlap NCA k's units [k U, (k + 1) U): c0 holds unit
// k U (first, from the uniform estimate, step down while the band starts after it, then up while it ends at or before
// it), c1 the last CTA that starts before (k + 1) U.
// blo(c): the first unit of CTA c (band_lo, or a table of it).
template <class BandLo>
__device__ __forceinline__ void nca_cta_span(const Bands &bd, int64_t U, int k, int *c0_out, int *c1_out, BandLo blo)
{
    const int64_t lo = (int64_t)k * U, hi = lo + U;
    int c0 = (int)(lo * bd.G / bd.T);
    c0 = c0 >= bd.G ? bd.G - 1 : c0;
    while (c0 > 0 && blo(c0) > lo)
        --c0;
    while (c0 + 1 < bd.G && blo(c0 + 1) <= lo)
        ++c0;
    int c1 = c0;
    while (c1 + 1 < bd.G && blo(c1 + 1) < hi)
        ++c1;
    *c0_out = c0;
    *c1_out = c1;
}
__device__ __forceinline__ void nca_cta_span(const Bands &bd, int64_t U, int k, int *c0_out, int *c1_out)
{
    nca_cta_span(bd, U, k, c0_out, c1_out, [&](int c) { return band_lo(bd, c); });
}

// Block-wide (every thread calls it): the non-empty CTAs of NCA k's span, in increasing order, into slots[0 .. n);
// returns n, or -1 (range = the span) when the span has more than cap CTAs. For a launch of at most SPAN_TABLE CTAs
// the band starts are computed in parallel (one band_lo per thread, into the shared table blo) and thread 0 lists
// from the table: band_lo of cost-balanced bands is a search of a few steps and the listing needs two per CTA, which
// serially on one thread made a reduce launch take ~27 us.
constexpr int SPAN_TABLE = 1024;
__device__ __forceinline__ int nca_span_slots(const Bands &bd, int64_t U, int k, int *slots, int cap, int64_t *blo,
                                              int *range, int *nslots)
{
    const bool table = bd.G < SPAN_TABLE;
    if (table)
        for (int c = threadIdx.x; c <= bd.G; c += blockDim.x)
            blo[c] = band_lo(bd, c);
    __syncthreads();
    if (threadIdx.x == 0) {
        auto lo_of = [&](int c) { return table ? blo[c] : band_lo(bd, c); };
        nca_cta_span(bd, U, k, &range[0], &range[1], lo_of);
        int n = 0;
        for (int c = range[0]; c <= range[1] && n < cap; ++c)
            if (lo_of(c + 1) > lo_of(c))
                slots[n++] = c;
        *nslots = range[1] - range[0] + 1 <= cap ? n : -1;
    }
    __syncthreads();
    return *nslots;
}

// Fixed-order sum of the partial slots (c + k) of the CTAs c whose tile ranges overlap NCA k -> dw1, db1, dw2
// (accumulate: added to the outputs). ncaops/nca_step.cuh:1164-1193 sums per-block partials the same way.
template <int C, int HID>
__global__ void reduce_kernel(const float *__restrict__ partial, Bands bd, int64_t tiles_per_nca,
                              float *__restrict__ dw1, float *__restrict__ db1, float *__restrict__ dw2, int accumulate)
{
    using D = Dims<C, HID>;
    constexpr int MAXS = 1024;  // slots listed in shared memory; a longer span is summed in the same order from bd
    const int k = blockIdx.y, e = blockIdx.x * blockDim.x + threadIdx.x;
    __shared__ int range[2], nslots_s;
    __shared__ int slots[MAXS];  // the non-empty CTAs of the span
    __shared__ int64_t blo[SPAN_TABLE];
    const int nslots = nca_span_slots(bd, tiles_per_nca, k, slots, MAXS, blo, range, &nslots_s);
    if (e >= D::PART)
        return;
    float s = 0.f;
    if (nslots >= 0) {
        for (int i = 0; i < nslots; ++i)
            s += partial[(size_t)(slots[i] + k) * D::PART + e];
    } else {
        for (int c = range[0]; c <= range[1]; ++c) {
            int64_t a, b;
            band_range(bd, c, &a, &b);
            if (b > a)
                s += partial[(size_t)(c + k) * D::PART + e];
        }
    }
    float *dst;
    if (e < HID * D::PIN)
        dst = dw1 + (size_t)k * HID * D::PIN + e;
    else if (e < HID * (D::PIN + 1))
        dst = db1 + (size_t)k * HID + (e - HID * D::PIN);
    else
        dst = dw2 + (size_t)k * C * HID + (e - HID * (D::PIN + 1));
    *dst = accumulate ? *dst + s : s;
}

}  // namespace unca
