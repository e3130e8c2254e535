// Auxiliary kernels around the step: update mask, synthetic loss + its gradient, fused per-NCA gradient normalisation
// + Adam + MultiStepLR, and the tcgen05 operand-layout self-test.
#pragma once
#include "nca_common.cuh"
#include "umma.cuh"

namespace unca {

// mask (n, h, w) of {0, 1} (ncaops/nca_step.cuh:237-245, grid-stride).
__global__ void mask_kernel(float *__restrict__ mask, int64_t N, int H, int W, uint64_t seed, float rate, int64_t n_offset)
{
    const int64_t total = N * H * W;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int X = (int)(i % W), Y = (int)((i / W) % H);
        const int64_t n = i / ((int64_t)H * W);
        mask[i] = update_mask_at(seed, rate, n + n_offset, H, W, Y, X);
    }
}

// ---------------------------------------------------------------- synthetic loss
// Per NCA k: mean over (B, TC, H, W) of (x[:, :TC] - target_k)^2 plus overflow_weight * sum over (B, C, H, W) of
// |x - clamp(x, -1, 1)|, and its gradient gy. TC = 3 with overflow: the texture configurations (the OT loss replaced
// by an L2 to a synthetic target, train.py:67-72); TC = 4 without: the growing NCA's loss, L2 to a premultiplied RGBA
// target (train.py:97-99). Block (chunk, k) sums a fixed slice of NCA k's elements (fixed order: strided per thread,
// then a tree), writes gy for the slice; loss_final sums the chunks of each NCA in order.
constexpr int LOSS_CHUNKS = 64;

__global__ void __launch_bounds__(256) loss_kernel(const float *__restrict__ x, const float *__restrict__ target,
                                                   float *__restrict__ gy, float *__restrict__ work, int B, int C, int H,
                                                   int W, int TC, float overflow_weight)
{
    const int k = blockIdx.y, chunk = blockIdx.x;
    const int64_t plane = (int64_t)H * W, per = (int64_t)B * C * plane;
    const int64_t lo = per * chunk / LOSS_CHUNKS, hi = per * (chunk + 1) / LOSS_CHUNKS;
    const float inv = 1.f / (float)((int64_t)B * TC * plane);
    const float *xk = x + (int64_t)k * per;
    float *gk = gy + (int64_t)k * per;
    float l2 = 0.f, of = 0.f;
    for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
        const int64_t pix = i % plane, c = (i / plane) % C;
        const float v = xk[i];
        float g = 0.f;
        if (c < TC) {
            const float d = v - target[((int64_t)k * TC + c) * plane + pix];
            l2 = fmaf(d, d, l2);
            g = 2.f * d * inv;
        }
        const float o = fabsf(v - fminf(fmaxf(v, -1.f), 1.f));
        of += o;
        if (o > 0.f)
            g += overflow_weight * (v > 0.f ? 1.f : -1.f);
        gk[i] = g;
    }
    __shared__ float s1[256], s2[256];
    s1[threadIdx.x] = l2;
    s2[threadIdx.x] = of;
    __syncthreads();
    for (int w = 128; w > 0; w >>= 1) {
        if (threadIdx.x < w) {
            s1[threadIdx.x] += s1[threadIdx.x + w];
            s2[threadIdx.x] += s2[threadIdx.x + w];
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        work[((int64_t)k * LOSS_CHUNKS + chunk) * 2] = s1[0];
        work[((int64_t)k * LOSS_CHUNKS + chunk) * 2 + 1] = s2[0];
    }
}

__global__ void loss_final_kernel(const float *__restrict__ work, float *__restrict__ loss, int K, int64_t l2_count,
                                  float overflow_weight)
{
    const int k = blockIdx.x * blockDim.x + threadIdx.x;
    if (k >= K)
        return;
    float a = 0.f, b = 0.f;
    for (int c = 0; c < LOSS_CHUNKS; ++c) {
        a += work[((int64_t)k * LOSS_CHUNKS + c) * 2];
        b += work[((int64_t)k * LOSS_CHUNKS + c) * 2 + 1];
    }
    loss[k] = a / (float)l2_count + overflow_weight * b;
}

// ---------------------------------------------------------------- gradient normalisation + Adam
struct AdamTensor {
    float *p, *m, *v;
    const float *g;
    int64_t numel;  // per NCA
};

struct AdamArgs {
    AdamTensor t[3];
    const int64_t *iteration;
    float lr, beta1, beta2, eps, gamma;
    int64_t milestones[8];
    int n_milestones;
};

// g / norm_eps (norm_eps = ||g_k|| + 1e-8, train.py:139) through torch.optim.Adam's update of NCA k's slice [base,
// base + numel) of one tensor (exp_avg.lerp_(g, 1 - beta1); exp_avg_sq = beta2 v + (1 - beta2) g^2;
// p -= lr / bc1 * m / (sqrt(v) / sqrt(bc2) + eps)), with MultiStepLR's lr at the device iteration counter.
__device__ __forceinline__ void adam_apply(const AdamArgs &a, const AdamTensor &T, int64_t base, float norm_eps)
{
    const int64_t it = *a.iteration;
    int decays = 0;
    for (int i = 0; i < a.n_milestones; ++i)
        decays += a.milestones[i] <= it;
    const double lr = (double)a.lr * pow((double)a.gamma, (double)decays);
    const double step = (double)(it + 1);
    const double bc1 = 1.0 - pow((double)a.beta1, step), bc2 = 1.0 - pow((double)a.beta2, step);
    const float step_size = (float)(lr / bc1), bc2_sqrt = (float)sqrt(bc2);
    const float w1 = 1.f - a.beta1, w2 = 1.f - a.beta2;
    for (int64_t i = threadIdx.x; i < T.numel; i += blockDim.x) {
        const float g = T.g[base + i] / norm_eps;
        float m = T.m[base + i], v = T.v[base + i];
        m = m + w1 * (g - m);
        v = v * a.beta2 + w2 * g * g;
        T.m[base + i] = m;
        T.v[base + i] = v;
        const float denom = sqrtf(v) / bc2_sqrt + a.eps;
        T.p[base + i] -= step_size * m / denom;
    }
}

// Block (k, tensor): ||g_k|| in a fixed order (strided per thread, then a tree), then adam_apply.
__global__ void __launch_bounds__(256) adam_kernel(AdamArgs a)
{
    const int k = blockIdx.x;
    const AdamTensor &T = a.t[blockIdx.y];
    const int64_t base = (int64_t)k * T.numel;
    float ss = 0.f;
    for (int64_t i = threadIdx.x; i < T.numel; i += blockDim.x) {
        const float g = T.g[base + i];
        ss = fmaf(g, g, ss);
    }
    __shared__ float red[256];
    red[threadIdx.x] = ss;
    __syncthreads();
    for (int w = 128; w > 0; w >>= 1) {
        if (threadIdx.x < w)
            red[threadIdx.x] += red[threadIdx.x + w];
        __syncthreads();
    }
    adam_apply(a, T, base, sqrtf(red[0]) + 1e-8f);  // train.py:139: p.grad /= ||p.grad_k|| + 1e-8
}

__global__ void increment_kernel(int64_t *iteration) { *iteration += 1; }

// ---------------------------------------------------------------- tcgen05 layout self-test
// D (128 x N) = A (128 x K) B (N x K)^T from row-major fp32 in global memory (rounded to TF32), with the operands
// staged in one of the forms the step kernels use:
//   form 0: A, B K-major, no swizzle (chunk-planar);           form 1: A in TMEM (lane = row), B K-major;
//   form 2: A, B MN-major SW128_32B (rows = K);                 form 3: form 2 with LBO / SBO exchanged (diagnostic).
__global__ void __launch_bounds__(128, 1) umma_selftest_kernel(int form, int N, int K, const float *__restrict__ A,
                                                               const float *__restrict__ B, float *__restrict__ D)
{
    extern __shared__ __align__(128) unsigned char raw[];
    unsigned char *base = raw + ((1024 - (umma::smem_u32(raw) & 1023)) & 1023);
    float *As = reinterpret_cast<float *>(base), *Bs = As + 128 * 128;
    uint64_t *bar = reinterpret_cast<uint64_t *>(Bs + 128 * 128);
    uint32_t *slot = reinterpret_cast<uint32_t *>(bar + 1);
    const int tid = threadIdx.x, warp = tid / 32;
    const bool mn = form >= 2;
    for (int e = tid; e < 128 * 128; e += 128)
        As[e] = Bs[e] = 0.f;
    __syncthreads();
    for (int e = tid; e < 128 * K; e += 128) {
        const int m = e / K, k = e % K;
        const float v = tf32_rna(A[e]);
        if (mn)
            As[umma::sw32_offset(m, k, K) / 4] = v;
        else
            As[(k / 4) * 128 * 4 + m * 4 + (k % 4)] = v;
    }
    for (int e = tid; e < N * K; e += 128) {
        const int n = e / K, k = e % K;
        const float v = tf32_rna(B[e]);
        if (mn)
            Bs[umma::sw32_offset(n, k, K) / 4] = v;
        else
            Bs[(k / 4) * N * 4 + n * 4 + (k % 4)] = v;
    }
    if (tid == 0) {
        umma::mbar_init(bar, 1);
        umma::fence_mbar_init();
    }
    if (warp == 0) {
        umma::tmem_alloc(slot, 512);
        umma::tmem_relinquish();
    }
    umma::fence_proxy_async();
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    const uint32_t tmem = *slot;
    const int dcol = 256;
    if (form == 1) {  // A into TMEM columns [0, K): thread = lane = row m
        for (int c0 = 0; c0 < K; c0 += 16) {
            float v[16];
#pragma unroll
            for (int e = 0; e < 16; ++e)
                v[e] = c0 + e < K ? tf32_rna(A[tid * K + c0 + e]) : 0.f;
            umma::tmem_st16(umma::tmem_addr(tmem, warp, c0), v);
        }
        umma::tmem_wait_st();
        umma::fence_before_sync();
        __syncthreads();
        umma::fence_after_sync();
    }
    if (tid == 0) {
        const uint32_t aa = umma::smem_u32(As), ba = umma::smem_u32(Bs);
        const uint32_t idesc = umma::idesc_tf32(128, N, mn, mn);
        for (int ks = 0; ks < K / 8; ++ks) {
            uint64_t adesc, bdesc;
            if (mn) {
                const uint32_t lbo = form == 2 ? K * 128 : 512, sbo = form == 2 ? 512 : K * 128;
                adesc = umma::smem_desc(aa + ks * 1024, lbo, sbo, umma::LAYOUT_SW128_32B);
                bdesc = umma::smem_desc(ba + ks * 1024, lbo, sbo, umma::LAYOUT_SW128_32B);
            } else {
                adesc = umma::smem_desc(aa + ks * 2 * 128 * 16, 128 * 16, 128);
                bdesc = umma::smem_desc(ba + ks * 2 * N * 16, N * 16, 128);
            }
            if (form == 1)
                umma::mma_ts(tmem + dcol, tmem + ks * 8, bdesc, idesc, ks > 0);
            else
                umma::mma_ss(tmem + dcol, adesc, bdesc, idesc, ks > 0);
        }
        umma::commit(bar);
    }
    const bool ok = umma::mbar_wait(bar, 0);
    umma::fence_after_sync();
    if (__syncthreads_and(ok)) {
        for (int c0 = 0; c0 < N; c0 += 16) {
            float v[16];
            umma::tmem_ld16(umma::tmem_addr(tmem, warp, dcol + c0), v);
            umma::tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 16; ++e)
                if (c0 + e < N)
                    D[tid * N + c0 + e] = v[e];
        }
    } else if (tid == 0) {
        set_device_error(1);
    }
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    if (warp == 0)
        umma::tmem_dealloc(tmem, 512);
}

}  // namespace unca
