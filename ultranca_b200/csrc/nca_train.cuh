// Training-iteration glue on the device, so that one captured CUDA graph replays a whole iteration of the reference's
// group loop (train.py:126-142) with nothing read from the host:
//   control_advance  the iteration counter and the iteration's rollout seed, in a device control block;
//   pool_draw        B distinct pool entries per NCA (train.py:128, rand(K, P).argsort(1)[:, :B]);
//   pool_gather      the batch from the pool, with the seed state injected every inject_every iterations
//                    (train.py:129-131);
//   pool_store       the final states back into their pool entries (train.py:141);
//   reduce_adam      the fixed-order reduction of the rollout's weight-gradient partials fused with the per-NCA
//                    per-tensor gradient normalisation + Adam + MultiStepLR (train.py:136-140).
// The random draws are this library's own (splitmix64), not torch's generator: like the reference's, they are fresh
// random samples each iteration, reproducible from the control block's key.
#pragma once
#include "nca_common.cuh"
#include "nca_kernels.cuh"
#include "nca_aux.cuh"

namespace unca {

// Control block (4 x uint64, device memory): [0] key (set by the host), [1] iterations started, [2] index of the
// current iteration, [3] its rollout seed (step t's update masks use splitmix_step(ctl[3], t), as nca_rollout derives
// them from its seed). One thread.
__global__ void control_advance_kernel(uint64_t *ctl)
{
    const uint64_t i = ctl[1];
    ctl[1] = i + 1;
    ctl[2] = i;
    ctl[3] = splitmix_step(ctl[0], 2 * i);
}

constexpr int POOL_MAX_BATCH = 64;

// Thread k: a partial Fisher-Yates shuffle of 0 .. P - 1 (B swaps, the swapped positions kept in a small map), draw b
// uniform in [b, P) from splitmix_step(key, (k0 + k) B + b) by a 64 x 64 -> high-64 multiply (k0: global index of
// NCA 0, so that a shard draws what the whole job would); idx[k, b] = the b-th entry.
__global__ void pool_draw_kernel(int64_t *__restrict__ idx, const uint64_t *__restrict__ ctl, int K, int P, int B,
                                 int64_t k0)
{
    const int k = blockIdx.x * blockDim.x + threadIdx.x;
    if (k >= K)
        return;
    const uint64_t key = splitmix_step(ctl[0], 2 * ctl[2] + 1);
    int pos[2 * POOL_MAX_BATCH], val[2 * POOL_MAX_BATCH], n = 0;
    auto get = [&](int p) {
        for (int i = 0; i < n; ++i)
            if (pos[i] == p)
                return val[i];
        return p;
    };
    auto set = [&](int p, int v) {
        for (int i = 0; i < n; ++i)
            if (pos[i] == p) {
                val[i] = v;
                return;
            }
        pos[n] = p;
        val[n] = v;
        ++n;
    };
    for (int b = 0; b < B; ++b) {
        const uint64_t r = splitmix_step(key, (uint64_t)(k0 + k) * B + b);
        const int j = b + (int)__umul64hi(r, (uint64_t)(P - b));
        const int vb = get(b), vj = get(j);
        set(b, vj);
        set(j, vb);
        idx[(int64_t)k * B + b] = vj;
    }
}

// Seed state value of element r (channel-major C x H x W) of one image: texture zeros (train.py:58-59); growing 1 in
// channels 3.. at the centre cell (train.py:81-84).
__device__ __forceinline__ float seed_state_value(int64_t r, int H, int W, int seed_kind)
{
    if (seed_kind != 1)
        return 0.f;
    const int64_t hw = (int64_t)H * W;
    const int c = (int)(r / hw), rem = (int)(r % hw);
    return c >= 3 && rem == (H / 2) * W + W / 2 ? 1.f : 0.f;
}

// x0[k, b] = pool[k, idx[k, b]] (C H W floats each); in an injection iteration (current index % inject_every == 0)
// x0[k, 0] is the seed state instead. VEC = 4: float4 moves (C H W % 4 == 0, 16-byte aligned buffers).
template <int VEC>
__global__ void pool_gather_kernel(const float *__restrict__ pool, float *__restrict__ x0, const int64_t *__restrict__ idx,
                                   const uint64_t *__restrict__ ctl, int K, int P, int B, int H, int W, int64_t chw,
                                   int64_t inject_every, int seed_kind)
{
    const bool inject = inject_every > 0 && ctl[2] % (uint64_t)inject_every == 0;
    const int64_t per = chw / VEC, total = (int64_t)K * B * per;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t n = e / per, r = (e - n * per) * VEC;
        const int k = (int)(n / B), b = (int)(n - (int64_t)k * B);
        if (VEC == 4) {
            float4 v;
            if (inject && b == 0)
                v = make_float4(seed_state_value(r, H, W, seed_kind), seed_state_value(r + 1, H, W, seed_kind),
                                seed_state_value(r + 2, H, W, seed_kind), seed_state_value(r + 3, H, W, seed_kind));
            else
                v = *reinterpret_cast<const float4 *>(pool + ((int64_t)k * P + idx[n]) * chw + r);
            *reinterpret_cast<float4 *>(x0 + n * chw + r) = v;
        } else {
            x0[n * chw + r] = inject && b == 0 ? seed_state_value(r, H, W, seed_kind)
                                               : pool[((int64_t)k * P + idx[n]) * chw + r];
        }
    }
}

// pool[k, idx[k, b]] = x[k, b].
template <int VEC>
__global__ void pool_store_kernel(float *__restrict__ pool, const float *__restrict__ x, const int64_t *__restrict__ idx,
                                  int K, int P, int B, int64_t chw)
{
    const int64_t per = chw / VEC, total = (int64_t)K * B * per;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t n = e / per, r = (e - n * per) * VEC;
        const int k = (int)(n / B);
        float *dst = pool + ((int64_t)k * P + idx[n]) * chw + r;
        if (VEC == 4)
            *reinterpret_cast<float4 *>(dst) = *reinterpret_cast<const float4 *>(x + n * chw + r);
        else
            *dst = x[n * chw + r];
    }
}

constexpr int REDUCE_MAX_SLOTS = 4096;  // partial slots one NCA may span (CTAs of the backward grid)

// Block (k, tensor t): gradient element e of NCA k = the fixed-order sum (CTAs ascending) of the partial slots of the
// backward CTAs that covered NCA k's units (as reduce_kernel), stored into the gradient output, then ||g_k|| and the
// Adam update exactly as adam_kernel (same per-thread element order and tree over 256 threads), so the result is
// bitwise that of reduce_kernel followed by adam_kernel, in one pass over the partials. A thread keeps up to 8 slots x 4
// elements of loads in flight (the sums are then taken in slot order).
template <int C, int HID>
__global__ void __launch_bounds__(256) reduce_adam_kernel(const float *__restrict__ partial, Bands bd,
                                                          int64_t units_per_nca, AdamArgs a)
{
    using D = Dims<C, HID>;
    constexpr int U = 4, S = 8;
    const int k = blockIdx.x, t = blockIdx.y;
    const AdamTensor &Tt = a.t[t];
    const int64_t off = t == 0 ? 0 : t == 1 ? (int64_t)HID * D::PIN : (int64_t)HID * (D::PIN + 1);
    const int64_t base = (int64_t)k * Tt.numel;
    __shared__ int slots[REDUCE_MAX_SLOTS];
    __shared__ int range[2], nslots;
    __shared__ int64_t blo[SPAN_TABLE];
    // the host launches this only for grids of at most REDUCE_MAX_SLOTS CTAs, so the span always fits
    const int ns = nca_span_slots(bd, units_per_nca, k, slots, REDUCE_MAX_SLOTS, blo, range, &nslots);
    float *g = const_cast<float *>(Tt.g);
    float ss = 0.f;
    for (int64_t i0 = threadIdx.x; i0 < Tt.numel; i0 += U * blockDim.x) {
        float sum[U];
#pragma unroll
        for (int u = 0; u < U; ++u)
            sum[u] = 0.f;
        for (int cb = 0; cb < ns; cb += S) {
            float v[S][U];
#pragma unroll
            for (int j = 0; j < S; ++j)
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    const int64_t i = i0 + (int64_t)u * blockDim.x;
                    v[j][u] = cb + j < ns && i < Tt.numel ? partial[(size_t)(slots[cb + j] + k) * D::PART + off + i] : 0.f;
                }
#pragma unroll
            for (int j = 0; j < S; ++j)
#pragma unroll
                for (int u = 0; u < U; ++u)
                    if (cb + j < ns)
                        sum[u] += v[j][u];
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t i = i0 + (int64_t)u * blockDim.x;
            if (i < Tt.numel) {
                g[base + i] = sum[u];
                ss = fmaf(sum[u], sum[u], ss);
            }
        }
    }
    __shared__ float red[256];
    red[threadIdx.x] = ss;
    __syncthreads();
    for (int w = 128; w > 0; w >>= 1) {
        if (threadIdx.x < w)
            red[threadIdx.x] += red[threadIdx.x + w];
        __syncthreads();
    }
    adam_apply(a, Tt, base, sqrtf(red[0]) + 1e-8f);
}

}  // namespace unca
