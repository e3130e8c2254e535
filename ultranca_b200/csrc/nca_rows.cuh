// Row-streaming step kernels (TF32, texture NCAs, W <= 128 and W % 4 == 0): the hot path of the benchmark configs.
//
// A CTA owns a contiguous band of global rows [NH c / G, NH (c+1) / G) of the N images; one image row is one
// 128-lane MMA tile (lane = column). Rows of x (and, in the backward, gy) stream through shared-memory rings by
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
__device__ __forceinline__ void row_mask_warp(float *mk, uint64_t seed, float rate, int64_t n, int H, int W, int Y, int lane)
{
    const int quads = (W + 3) / 4;
    if (rate >= 1.f) {
        for (int x = lane; x < W; x += 32)
            mk[x] = 1.f;
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
                mk[x] = floorf(__fadd_rn(__fmul_rn((float)(words[e] >> 8), 1.0f / 16777216.0f), rate)) != 0.f ? 1.f : 0.f;
        }
    }
}

// ================================================================ forward
template <int C, int HID, int NPART>
struct FwdRows {
    using D = Dims<C, HID>;
    static constexpr int THREADS = 128 * NPART, CPP = C / NPART, HPP = HID / NPART, RING = 4;
    static constexpr int KPAD = ((D::KP + 15) / 16) * 16;
    static constexpr int T_P = 0, T_H = 128, T_U = T_H + HID, TMEM = 256;
    static_assert(C % NPART == 0 && HPP % 8 == 0 && KPAD <= T_H && T_U + 16 <= TMEM, "forward row-kernel layout");
    static constexpr size_t smem() { return (size_t)(D::W1S + D::W2S + RING * C * 128 + 2 * 128) * 4 + 8 * (RING + 1) + 16; }
};

template <int C, int HID, int NPART>
__global__ void __launch_bounds__(128 * NPART, 4 / NPART) fwd_rows_kernel(StepArgs a)
{
    using F = FwdRows<C, HID, NPART>;
    using D = typename F::D;
    extern __shared__ __align__(128) float smem[];
    float *W1s = smem, *W2s = W1s + D::W1S, *XR = W2s + D::W2S, *MK = XR + F::RING * C * 128;
    uint64_t *xfull = reinterpret_cast<uint64_t *>(MK + 2 * 128), *mbar = xfull + F::RING;
    uint32_t *tslot = reinterpret_cast<uint32_t *>(mbar + 1);

    const int tid = threadIdx.x, warp = tid / 32, part = tid / 128, x = tid % 128;
    const int lane32 = tid % 32, mask_warp = F::THREADS / 32 - 1;
    const int H = a.H, W = a.W;
    const bool vx = x < W;
    const int xc = vx ? x : 0, xl = xc == 0 ? W - 1 : xc - 1, xr = xc + 1 >= W ? 0 : xc + 1;
    int64_t g0, g1;
    cta_range((int64_t)a.N * H, gridDim.x, blockIdx.x, &g0, &g1);
    const size_t plane = (size_t)H * W;

    if (tid == 0) {
        for (int i = 0; i < F::RING; ++i)
            umma::mbar_init(&xfull[i], 1);
        umma::mbar_init(mbar, 1);
        umma::fence_mbar_init();
    }
    if (warp == 0) {
        umma::tmem_alloc(tslot, F::TMEM);
        umma::tmem_relinquish();
    }
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    const uint32_t tmem = *tslot, lane = umma::tmem_addr(tmem, warp, 0);
    if (part == 0) {  // p' columns past the channel features: bias-hi, bias-lo = 1, zeros (never overwritten)
        float v[8] = {1.f, 1.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        umma::tmem_st8(lane + F::T_P + D::PIN, v);
        const float z[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int c0 = D::PIN + 8; c0 < F::KPAD; c0 += 8)
            umma::tmem_st8(lane + F::T_P + c0, z);
        umma::tmem_wait_st();
    }
    uint32_t xpar = 0, mphase = 0;
    int cur_k = -1;
    bool ok = true;
    int64_t g = g0;
    RowSeg sg;
    while (ok && next_segment(g, g1, H, sg)) {
        const int n = sg.n, k = n / a.B, L = sg.r1 - sg.r0;
        umma::fence_before_sync();
        __syncthreads();  // the previous segment's ring, mask and TMEM reads are complete
        if (k != cur_k) {
            stage_weights<D, true>(W1s, W2s, a.w1 + (size_t)k * HID * D::PIN, a.b1 + (size_t)k * HID,
                                   a.w2 + (size_t)k * C * HID);
            umma::fence_proxy_async();
            cur_k = k;
        }
        const float *xn = a.x + (size_t)n * C * plane;
        auto issue = [&](int e) {  // x row wrap(r0 - 1 + e) -> slot e % RING
            const int slot = e % F::RING, Y = wrap_index(sg.r0 - 1 + e, H);
            umma::mbar_arrive_expect_tx(&xfull[slot], (uint32_t)(C * W * 4));
            for (int c = 0; c < C; ++c)
                umma::bulk_g2s(XR + ((size_t)slot * C + c) * W, xn + ((size_t)c * H + Y) * W, (uint32_t)(W * 4), &xfull[slot]);
        };
        if (tid == 0)
            for (int e = 0; e < min(L + 2, F::RING); ++e)
                issue(e);
        if (warp == mask_warp)
            row_mask_warp(MK, a.seed, a.rate, n + a.n_offset, H, W, sg.r0, lane32);
        int waited = 0;
        for (int i = 0; i < L && ok; ++i) {
            const int Y = sg.r0 + i;
            if (tid == 0)
                ok = ring_wait<F::RING>(xfull, waited, i + 2, xpar);
            ok = __syncthreads_and(ok);  // rows Y-1 .. Y+1 and the mask of row Y are in shared memory
            if (!ok)
                break;
            umma::fence_after_sync();
            const float *rm = XR + (size_t)(i % F::RING) * C * W, *r0 = XR + (size_t)((i + 1) % F::RING) * C * W,
                        *rp = XR + (size_t)((i + 2) % F::RING) * C * W;
#pragma unroll
            for (int cc = 0; cc < F::CPP; ++cc) {
                const int c = part + NPART * cc;
                const float *bm = rm + c * W, *b0 = r0 + c * W, *bp = rp + c * W;
                const float v[3][3] = {{bm[xl], bm[xc], bm[xr]}, {b0[xl], b0[xc], b0[xr]}, {bp[xl], bp[xc], bp[xr]}};
                const float4 p = perceive3x3(v);
                const float pv[4] = {tf32_rna(p.x), tf32_rna(p.y), tf32_rna(p.z), tf32_rna(p.w)};
                umma::tmem_st4(lane + F::T_P + 4 * c, pv);
            }
            const float m = MK[(i & 1) * 128 + xc];
            float xv[F::CPP];
#pragma unroll
            for (int cc = 0; cc < F::CPP; ++cc)
                xv[cc] = r0[(part + NPART * cc) * W + xc];
            umma::tmem_wait_st();
            umma::fence_before_sync();
            __syncthreads();  // p' complete; row Y-1 (ring entry i) is no longer read
            if (tid == 0) {
                umma::fence_after_sync();
#pragma unroll
                for (int ks = 0; ks < D::KP / 8; ++ks)
                    umma::mma_ts(tmem + F::T_H, tmem + F::T_P + ks * 8,
                                 umma::smem_desc(umma::smem_u32(W1s) + ks * 2 * HID * 16, HID * 16, 128),
                                 umma::idesc_tf32(128, HID, false, false), ks > 0);
                umma::commit(mbar);
                if (i + 4 < L + 2)
                    issue(i + 4);
                ok = umma::mbar_wait(mbar, mphase);
            }
            mphase ^= 1;
            if (warp == mask_warp && i + 1 < L)
                row_mask_warp(MK + ((i + 1) & 1) * 128, a.seed, a.rate, n + a.n_offset, H, W, Y + 1, lane32);
            ok = __syncthreads_and(ok);
            umma::fence_after_sync();
#pragma unroll
            for (int q = 0; q < F::HPP / 8; ++q) {
                float h[8];
                umma::tmem_ld8(lane + F::T_H + part * F::HPP + q * 8, h);
                umma::tmem_wait_ld();
#pragma unroll
                for (int e = 0; e < 8; ++e)
                    h[e] = tf32_rna(fmaxf(h[e], 0.f));
                umma::tmem_st8(lane + F::T_H + part * F::HPP + q * 8, h);
            }
            umma::tmem_wait_st();
            umma::fence_before_sync();
            __syncthreads();
            if (tid == 0 && ok) {
                umma::fence_after_sync();
#pragma unroll
                for (int ks = 0; ks < HID / 8; ++ks)
                    umma::mma_ts(tmem + F::T_U, tmem + F::T_H + ks * 8,
                                 umma::smem_desc(umma::smem_u32(W2s) + ks * 2 * D::CP * 16, D::CP * 16, 128),
                                 umma::idesc_tf32(128, 16, false, false), ks > 0);
                umma::commit(mbar);
                ok = umma::mbar_wait(mbar, mphase);
            }
            mphase ^= 1;
            ok = __syncthreads_and(ok);
            umma::fence_after_sync();
            float u[16];
            umma::tmem_ld16(lane + F::T_U, u);
            umma::tmem_wait_ld();
            if (vx && ok) {
                float *yn = a.y + (size_t)n * C * plane + (size_t)Y * W + x;
#pragma unroll
                for (int cc = 0; cc < F::CPP; ++cc) {
                    const int c = part + NPART * cc;
                    yn[(size_t)c * plane] = m != 0.f ? xv[cc] + u[c] : xv[cc];
                }
            }
            umma::fence_before_sync();  // the next row's barriers order these TMEM reads before its MMAs
        }
    }
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    if (warp == 0)
        umma::tmem_dealloc(tmem, F::TMEM);
    if (!ok && tid == 0)
        set_device_error(1);
}

// ================================================================ backward with the fused adjoint
template <int C, int HID, int NPART>
struct BwdRows {
    using D = Dims<C, HID>;
    static constexpr int THREADS = 128 * NPART, CPP = C / NPART, HPP = HID / NPART, XRING = 4, GRING = 4;
    static constexpr int KPAD = ((D::KP + 15) / 16) * 16;
    // TMEM: H (then dh) | DHP | p' (then dp) | gm | dW1' | dW2^T
    static constexpr int T_H = 0, T_DHP = 128, T_P = 256, T_G = 256 + KPAD, T_ACC1 = 384, T_ACC2 = 384 + D::NPW, TMEM = 512;
    static_assert(C % NPART == 0 && HPP % 8 == 0 && T_G + 16 <= T_ACC1 && T_ACC2 + 16 <= TMEM, "backward row-kernel layout");
    // shared memory, 1024-aligned base: weights | RHDH | PSW | GSW (swizzled) | XR | GR | EX | MK | barriers
    static constexpr size_t OFF_SW = (size_t)D::BWD_W;
    static constexpr size_t OFF_XR = OFF_SW + (size_t)(D::RHDH + D::PSW + D::GSW) * 4;
    static constexpr size_t OFF_GR = OFF_XR + (size_t)XRING * C * 128 * 4;
    static constexpr size_t OFF_EX = OFF_GR + (size_t)GRING * C * 128 * 4;
    static constexpr size_t OFF_MK = OFF_EX + (size_t)C * 128 * 16;
    static constexpr size_t OFF_BAR = OFF_MK + 2 * 128 * 4;
    static constexpr size_t smem() { return 1024 + OFF_BAR + 8 * (XRING + GRING + 2) + 16; }
};

template <int C, int HID, int NPART>
__global__ void __launch_bounds__(128 * NPART, 1) bwd_rows_kernel(StepArgs a)
{
    using F = BwdRows<C, HID, NPART>;
    using D = typename F::D;
    extern __shared__ __align__(128) unsigned char smem_raw[];
    unsigned char *base = smem_raw + ((1024 - (umma::smem_u32(smem_raw) & 1023)) & 1023);
    float *W1s = reinterpret_cast<float *>(base), *W1T = W1s + D::W1S, *W2T = W1T + D::W1T;
    float *RHDH = reinterpret_cast<float *>(base + F::OFF_SW), *PSW = RHDH + D::RHDH, *GSW = PSW + D::PSW;
    float *XR = reinterpret_cast<float *>(base + F::OFF_XR), *GR = reinterpret_cast<float *>(base + F::OFF_GR);
    float4 *EX = reinterpret_cast<float4 *>(base + F::OFF_EX);
    float *MK = reinterpret_cast<float *>(base + F::OFF_MK);
    uint64_t *xfull = reinterpret_cast<uint64_t *>(base + F::OFF_BAR), *gfull = xfull + F::XRING;
    uint64_t *mbar = gfull + F::GRING, *wbar = mbar + 1;
    uint32_t *tslot = reinterpret_cast<uint32_t *>(wbar + 1);

    const int tid = threadIdx.x, warp = tid / 32, part = tid / 128, x = tid % 128;
    const int lane32 = tid % 32, mask_warp = F::THREADS / 32 - 1;
    const int H = a.H, W = a.W;
    const bool vx = x < W;
    const int xc = vx ? x : 0, xl = xc == 0 ? W - 1 : xc - 1, xr = xc + 1 >= W ? 0 : xc + 1;
    int64_t g0, g1;
    cta_range((int64_t)a.N * H, gridDim.x, blockIdx.x, &g0, &g1);
    const size_t plane = (size_t)H * W;

    for (int e = tid; e < D::GSW; e += blockDim.x)
        GSW[e] = 0.f;
    for (int e = tid; e < 128 * (D::NPW - D::PIN); e += blockDim.x) {  // p' features past the channels: 1, 1, 0...
        const int q = e / (D::NPW - D::PIN), f = D::PIN + e % (D::NPW - D::PIN);
        PSW[umma::sw32_offset(f, q, 128) / 4] = f < D::PIN + 2 ? 1.f : 0.f;
    }
    if (tid == 0) {
        for (int i = 0; i < F::XRING; ++i)
            umma::mbar_init(&xfull[i], 1);
        for (int i = 0; i < F::GRING; ++i)
            umma::mbar_init(&gfull[i], 1);
        umma::mbar_init(mbar, 1);
        umma::mbar_init(wbar, 1);
        umma::fence_mbar_init();
    }
    if (warp == 0) {
        umma::tmem_alloc(tslot, F::TMEM);
        umma::tmem_relinquish();
    }
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    const uint32_t tmem = *tslot, lane = umma::tmem_addr(tmem, warp, 0);
    if (part == 0) {  // constant p' columns and zero gm columns in TMEM (never overwritten)
        float v[8] = {1.f, 1.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        umma::tmem_st8(lane + F::T_P + D::PIN, v);
        const float z[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int c0 = D::PIN + 8; c0 < F::KPAD; c0 += 8)
            umma::tmem_st8(lane + F::T_P + c0, z);
        for (int c = C; c < 16; ++c)
            umma::tmem_st1(lane + F::T_G + c, 0.f);
        umma::tmem_wait_st();
    }
    const uint32_t sW1 = umma::smem_u32(W1s), sW1T = umma::smem_u32(W1T), sW2T = umma::smem_u32(W2T);
    const uint32_t sRH = umma::smem_u32(RHDH), sP = umma::smem_u32(PSW), sG = umma::smem_u32(GSW);
    uint32_t xpar = 0, gpar = 0, mphase = 0, wphase = 0;
    bool w_pending = false, started = false, ok = true;
    int cur_k = -1;

    auto flush = [&](int k) {  // this CTA's weight gradients of NCA k -> partial slot (blockIdx.x + k); part 0 only
        if (part != 0)
            return;
        float row[((D::PIN + 1 + 15) / 16) * 16], col[16];
#pragma unroll
        for (int cc = 0; cc < (D::PIN + 1 + 15) / 16; ++cc) {
            float v[16];
            umma::tmem_ld16(lane + F::T_ACC1 + cc * 16, v);
            umma::tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 16; ++e)
                row[cc * 16 + e] = v[e];
        }
        umma::tmem_ld16(lane + F::T_ACC2, col);
        umma::tmem_wait_ld();
        if (x < HID)
            write_partial_row<D>(a.partial + (size_t)(blockIdx.x + k) * D::PART, x, row, row[D::PIN], col);
    };
    auto wait_w = [&]() {  // by thread 0: the last issued dW1' (reads RHDH and PSW) has completed
        bool r = true;
        if (w_pending && tid == 0)
            r = umma::mbar_wait(wbar, wphase);
        if (w_pending)
            wphase ^= 1;
        w_pending = false;
        return r;
    };

    int64_t g = g0;
    RowSeg sg;
    while (ok && next_segment(g, g1, H, sg)) {
        const int n = sg.n, k = n / a.B, L = sg.r1 - sg.r0 + 2;  // sequence: halo, owned rows, halo
        ok = __syncthreads_and(wait_w());  // previous segment complete (ring, EX, MK reads; dW1')
        umma::fence_after_sync();
        if (!ok)
            break;
        if (k != cur_k) {
            if (cur_k >= 0)
                flush(cur_k);
            umma::fence_before_sync();
            __syncthreads();
            stage_bwd_weights<D>(W1s, W1T, W2T, a.w1 + (size_t)k * HID * D::PIN, a.b1 + (size_t)k * HID,
                                 a.w2 + (size_t)k * C * HID);
            umma::fence_proxy_async();
            cur_k = k;
            started = false;
        }
        const float *xn = a.x + (size_t)n * C * plane, *gyn = a.gy + (size_t)n * C * plane;
        float *gxn = a.gx + (size_t)n * C * plane;
        auto issue_x = [&](int e) {  // x row wrap(r0 - 2 + e)
            const int slot = e % F::XRING, Y = wrap_index(sg.r0 - 2 + e, H);
            umma::mbar_arrive_expect_tx(&xfull[slot], (uint32_t)(C * W * 4));
            for (int c = 0; c < C; ++c)
                umma::bulk_g2s(XR + ((size_t)slot * C + c) * W, xn + ((size_t)c * H + Y) * W, (uint32_t)(W * 4), &xfull[slot]);
        };
        auto issue_g = [&](int e) {  // gy row wrap(r0 - 1 + e)
            const int slot = e % F::GRING, Y = wrap_index(sg.r0 - 1 + e, H);
            umma::mbar_arrive_expect_tx(&gfull[slot], (uint32_t)(C * W * 4));
            for (int c = 0; c < C; ++c)
                umma::bulk_g2s(GR + ((size_t)slot * C + c) * W, gyn + ((size_t)c * H + Y) * W, (uint32_t)(W * 4), &gfull[slot]);
        };
        if (tid == 0) {
            for (int e = 0; e < min(L + 2, F::XRING); ++e)
                issue_x(e);
            for (int e = 0; e < min(L, 2); ++e)  // entry i + 2 is issued during iteration i
                issue_g(e);
        }
        if (warp == mask_warp)
            row_mask_warp(MK, a.seed, a.rate, n + a.n_offset, H, W, wrap_index(sg.r0 - 1, H), lane32);
        int xwaited = 0, gwaited = 0;
        float accm[F::CPP], acc0[F::CPP], accp[F::CPP];
#pragma unroll
        for (int cc = 0; cc < F::CPP; ++cc)
            accm[cc] = acc0[cc] = accp[cc] = 0.f;
        for (int i = 0; i < L && ok; ++i) {
            const int Y = wrap_index(sg.r0 - 1 + i, H);
            const bool owned = i >= 1 && i <= L - 2;
            // ---- B1: x rows Y-1 .. Y+1, gy row Y, mask of row Y; the previous dW1' has completed
            if (tid == 0) {
                ok = ring_wait<F::XRING>(xfull, xwaited, i + 2, xpar);
                ok &= ring_wait<F::GRING>(gfull, gwaited, i, gpar);
            }
            ok &= wait_w();
            ok = __syncthreads_and(ok);
            if (!ok)
                break;
            umma::fence_after_sync();
            if (tid == 0 && i + 2 < L)
                issue_g(i + 2);  // slot of entry i - 2, last read by the finalize of iteration i - 1
            const float *rm = XR + (size_t)(i % F::XRING) * C * W, *r0 = XR + (size_t)((i + 1) % F::XRING) * C * W,
                        *rp = XR + (size_t)((i + 2) % F::XRING) * C * W, *gr = GR + (size_t)(i % F::GRING) * C * W;
            const float m = MK[(i & 1) * 128 + xc];
#pragma unroll
            for (int cc = 0; cc < F::CPP; ++cc) {
                const int c = part + NPART * cc;
                const float *bm = rm + c * W, *b0 = r0 + c * W, *bp = rp + c * W;
                const float v[3][3] = {{bm[xl], bm[xc], bm[xr]}, {b0[xl], b0[xc], b0[xr]}, {bp[xl], bp[xc], bp[xr]}};
                const float4 p = perceive3x3(v);
                const float4 pv = make_float4(tf32_rna(p.x), tf32_rna(p.y), tf32_rna(p.z), tf32_rna(p.w));
                const float gmv = (vx && m != 0.f) ? tf32_rna(gr[c * W + xc]) : 0.f;
                const float t4[4] = {pv.x, pv.y, pv.z, pv.w};
                umma::tmem_st4(lane + F::T_P + 4 * c, t4);
                *reinterpret_cast<float4 *>(PSW + umma::sw32_offset(4 * c, x, 128) / 4) = pv;
                umma::tmem_st1(lane + F::T_G + c, gmv);
                GSW[umma::sw32_offset(c, x, 128) / 4] = gmv;
            }
            umma::tmem_wait_st();
            umma::fence_proxy_async();
            umma::fence_before_sync();
            __syncthreads();  // B2: p', gm ready; x row Y-1 (entry i) no longer read
            // ---- H = p' W1'^T, DHP = gm W2 (A from TMEM)
            if (tid == 0) {
                umma::fence_after_sync();
#pragma unroll
                for (int ks = 0; ks < D::KP / 8; ++ks)
                    umma::mma_ts(tmem + F::T_H, tmem + F::T_P + ks * 8, umma::smem_desc(sW1 + ks * 2 * HID * 16, HID * 16, 128),
                                 umma::idesc_tf32(128, HID, false, false), ks > 0);
#pragma unroll
                for (int ks = 0; ks < 2; ++ks)
                    umma::mma_ts(tmem + F::T_DHP, tmem + F::T_G + ks * 8, umma::smem_desc(sW2T + ks * 2 * HID * 16, HID * 16, 128),
                                 umma::idesc_tf32(128, HID, false, false), ks > 0);
                umma::commit(mbar);
                if (i + 4 < L + 2)
                    issue_x(i + 4);
                ok = umma::mbar_wait(mbar, mphase);
            }
            mphase ^= 1;
            if (warp == mask_warp && i + 1 < L)
                row_mask_warp(MK + ((i + 1) & 1) * 128, a.seed, a.rate, n + a.n_offset, H, W, wrap_index(Y + 1, H), lane32);
            ok = __syncthreads_and(ok);  // B3
            umma::fence_after_sync();
            // ---- relu(h) -> RHDH (swizzled), dh -> TMEM (this part's hidden units)
#pragma unroll
            for (int q = 0; q < F::HPP / 8; ++q) {
                const int j0 = part * F::HPP + q * 8;
                float h[8], d[8];
                umma::tmem_ld8(lane + F::T_H + j0, h);
                umma::tmem_ld8(lane + F::T_DHP + j0, d);
                umma::tmem_wait_ld();
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    d[e] = h[e] > 0.f ? tf32_rna(d[e]) : 0.f;
                    h[e] = tf32_rna(fmaxf(h[e], 0.f));
                }
                if (owned)
                    st_sw32x8(RHDH, j0, x, 128, h);
                umma::tmem_st8(lane + F::T_H + j0, d);
            }
            umma::tmem_wait_st();
            umma::fence_proxy_async();
            umma::fence_before_sync();
            __syncthreads();  // B4
            // ---- dW2^T += relu(h)^T gm (owned rows), DP = dh W1 (A from TMEM)
            if (tid == 0 && ok) {
                umma::fence_after_sync();
                if (owned)
#pragma unroll
                    for (int ks = 0; ks < 16; ++ks)
                        umma::mma_ss(tmem + F::T_ACC2, umma::smem_desc(sRH + ks * 1024, 128 * 128, 512, umma::LAYOUT_SW128_32B),
                                     umma::smem_desc(sG + ks * 1024, 128 * 128, 512, umma::LAYOUT_SW128_32B),
                                     umma::idesc_tf32(128, 16, true, true), started || ks > 0);
#pragma unroll
                for (int ks = 0; ks < HID / 8; ++ks)
                    umma::mma_ts(tmem + F::T_P, tmem + F::T_H + ks * 8, umma::smem_desc(sW1T + ks * 2 * D::PIN * 16, D::PIN * 16, 128),
                                 umma::idesc_tf32(128, D::PIN, false, false), ks > 0);
                umma::commit(mbar);
                ok = umma::mbar_wait(mbar, mphase);
            }
            mphase ^= 1;
            ok = __syncthreads_and(ok);  // B5
            umma::fence_after_sync();
            // ---- dh -> RHDH (swizzled, over relu(h)); dp -> exchange buffer
            if (owned) {
#pragma unroll
                for (int q = 0; q < F::HPP / 8; ++q) {
                    const int j0 = part * F::HPP + q * 8;
                    float d[8];
                    umma::tmem_ld8(lane + F::T_H + j0, d);
                    umma::tmem_wait_ld();
                    st_sw32x8(RHDH, j0, x, 128, d);
                }
            }
            float dpv[F::CPP][4];
#pragma unroll
            for (int cc = 0; cc < F::CPP; ++cc)
                umma::tmem_ld4(lane + F::T_P + 4 * (part + NPART * cc), dpv[cc]);
            umma::tmem_wait_ld();
#pragma unroll
            for (int cc = 0; cc < F::CPP; ++cc)
                EX[(part + NPART * cc) * 128 + x] = vx ? make_float4(dpv[cc][1], dpv[cc][2], dpv[cc][3], 0.f)
                                                      : make_float4(0.f, 0.f, 0.f, 0.f);
            umma::fence_proxy_async();
            umma::fence_before_sync();
            __syncthreads();  // B6: dh (swizzled) and the exchange buffer are complete
            if (tid == 0 && owned && ok) {
                umma::fence_after_sync();
#pragma unroll
                for (int ks = 0; ks < 16; ++ks)
                    umma::mma_ss(tmem + F::T_ACC1, umma::smem_desc(sRH + ks * 1024, 128 * 128, 512, umma::LAYOUT_SW128_32B),
                                 umma::smem_desc(sP + ks * 1024, 128 * 128, 512, umma::LAYOUT_SW128_32B),
                                 umma::idesc_tf32(128, D::NPW, true, true), started || ks > 0);
                umma::commit(wbar);
            }
            if (owned) {
                w_pending = true;
                started = true;
            }
            // ---- adjoint: dp of row Y -> gx rows Y-1, Y, Y+1; row Y-1 is final when owned
            const bool fin = i >= 2 && vx;
            const float *gprev = GR + (size_t)((i + F::GRING - 1) % F::GRING) * C * W;
            float *gxrow = gxn + (size_t)wrap_index(Y - 1, H) * W + x;
#pragma unroll
            for (int cc = 0; cc < F::CPP; ++cc) {
                const int c = part + NPART * cc;
                const float4 el = EX[c * 128 + xl], er = EX[c * 128 + xr];
                const float rsx = el.x - er.x;                     // horizontal transpose of sobel_x
                const float rsy = er.y + 2.f * dpv[cc][2] + el.y;  // ... of sobel_y (smoothing)
                const float rlap = el.z + 2.f * dpv[cc][3] + er.z; // ... of the laplacian
                accm[cc] += rsx - rsy + rlap;
                acc0[cc] += 2.f * rsx + 2.f * rlap + dpv[cc][0] - 16.f * dpv[cc][3];
                accp[cc] += rsx + rsy + rlap;
                if (fin)
                    gxrow[(size_t)c * plane] = gprev[c * W + x] + accm[cc];
                accm[cc] = acc0[cc];
                acc0[cc] = accp[cc];
                accp[cc] = 0.f;
            }
            umma::fence_before_sync();  // the next row's barriers order these TMEM reads before its writes
        }
    }
    if (ok) {
        ok = __syncthreads_and(wait_w());
        umma::fence_after_sync();
        if (ok && cur_k >= 0)
            flush(cur_k);
    }
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    if (warp == 0)
        umma::tmem_dealloc(tmem, F::TMEM);
    if (!ok && tid == 0)
        set_device_error(1);
}

}  // namespace unca
