// TEST INFRASTRUCTURE ONLY: a C-ABI launcher for the reference's own CUDA kernels (UltraNCA ncaops/nca_step.cuh,
// compiled unchanged from the reference checkout by oracle/build_ref.py into oracle/_ref/libncaref.so). Only the
// tests and bench.py's reference-kernel timing load it, to pin the Philox mask bitwise against the reference's
// mask_kernel and to compare with / time the reference's step kernels on the same B200.
//
// The launch parameters restate the reference's nanobind host layer, which needs nanobind and cannot be built here:
//   forward + alive: ncaops/nca_cuda.cu:94-126 (dispatch :62-77, segment sizing, split tail);
//   backward:        ncaops/nca_cuda.cu:190-216,236-323 with one launch over all images (the reference's choice for
//                    GPUs with >= 160 KB of shared memory per SM, :211-212);
//   update mask:     ncaops/nca_cuda.cu:325-331.
#include <cuda_runtime.h>
#include <algorithm>
#include <cstdint>
#include <type_traits>

#include "nca_step.cuh"

namespace {

template <int C_, int HID_, bool FP32_, bool STOCH_, bool ALIVE_>
struct Inst {
    static constexpr int C = C_, HID = HID_;
    static constexpr bool FP32 = FP32_, STOCH = STOCH_, ALIVE = ALIVE_;
};

template <typename F>
int with_bool(bool v, F &&f) { return v ? f(std::true_type{}) : f(std::false_type{}); }

template <typename F>
int dispatch(int C, int HID, bool fp32, bool stoch, bool alive, F &&f)
{
    return with_bool(fp32, [&](auto FP) { return with_bool(stoch, [&](auto ST) { return with_bool(alive, [&](auto AL) {
        if (C == 12 && HID == 96)
            return f(Inst<12, 96, decltype(FP)::value, decltype(ST)::value, decltype(AL)::value>{});
        if (C == 16 && HID == 128)
            return f(Inst<16, 128, decltype(FP)::value, decltype(ST)::value, decltype(AL)::value>{});
        return (int)cudaErrorInvalidValue;
    }); }); });
}

int ceil_div(int a, int b) { return (a + b - 1) / b; }

int sm_count()
{
    int dev, v;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    return v;
}

int bwd_blocks_per_image(int H, int W, bool stoch)
{
    const int tiles = ceil_div(W, nca_step::TILE_W) * ceil_div(H, nca_step::bwd_tile_h(stoch));
    return ceil_div(tiles, nca_step::BWD_TILES_PER_BLOCK);
}

}  // namespace

extern "C" {

int ref_update_mask(float *mask, int N, int H, int W, uint64_t seed, float rate, void *stream)
{
    const uint64_t total = (uint64_t)N * H * W;
    nca_step::mask_kernel<<<(unsigned)std::min<uint64_t>((total + 255) / 256, 65535), 256, 0, (cudaStream_t)stream>>>(
        mask, N, H, W, seed, rate);
    return (int)cudaGetLastError();
}

int ref_forward(const float *x, const float *w1, const float *b1, const float *w2, float *y, float *alpha, uint8_t *alive,
                int N, int C, int HID, int H, int W, int B, uint64_t seed, float rate, int fp32, int growing, void *stream)
{
    return dispatch(C, HID, fp32, rate < 1.f, growing, [&](auto I) {
        using D = decltype(I);
        auto kernel = nca_step::forward_kernel<D::C, D::HID, D::FP32, D::STOCH, D::ALIVE>;
        constexpr int smem = sizeof(nca_step::ForwardSmem<D::C, D::HID, D::FP32>);
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        int blocks_per_sm = 1;
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks_per_sm, kernel, nca_step::FWD_THREADS, smem);
        const int strips = ceil_div(W, nca_step::TILE_W), slots = blocks_per_sm * sm_count();
        int seg = D::ALIVE ? std::min<int>(H, 128) : H;
        while (seg > nca_step::FWD_PHASE && (size_t)N * strips * ceil_div(H, seg) < 2 * (size_t)slots)
            seg = ceil_div(seg, 2);
        const cudaStream_t st = (cudaStream_t)stream;
        if constexpr (nca_step::FWD_TAIL) {
            const int items = N * strips * ceil_div(H, seg), tail = items > slots ? items % slots : 0;
            kernel<<<items + tail, nca_step::FWD_THREADS, smem, st>>>(x, w1, b1, w2, y, alpha, nullptr, B, H, W, seed, rate,
                                                                     seg, items - tail);
        } else {
            kernel<<<dim3(strips * ceil_div(H, seg), N), nca_step::FWD_THREADS, smem, st>>>(x, w1, b1, w2, y, alpha, nullptr,
                                                                                            B, H, W, seed, rate, seg, 0);
        }
        if (D::ALIVE) {
            const uint64_t total = (uint64_t)N * H * W;
            nca_step::alive_kernel<D::C><<<(unsigned)((total + 255) / 256), 256, 0, st>>>(x, alpha, y, alive, H, W, total,
                                                                                         false);
        }
        return (int)cudaGetLastError();
    });
}

// Workspace sizes: packed bytes (all NCAs), partial floats (all images), dp floats (all images), updating bytes.
int ref_backward_workspace(int N, int K, int C, int HID, int H, int W, float rate, int fp32, int growing, int64_t *packed,
                           int64_t *partial, int64_t *dp, int64_t *updating)
{
    return dispatch(C, HID, fp32, rate < 1.f, growing, [&](auto I) {
        using D = decltype(I);
        *packed = (int64_t)K * sizeof(nca_step::BackwardWeights<D::C, D::HID, D::FP32>);
        *partial = (int64_t)N * bwd_blocks_per_image(H, W, D::STOCH) * nca_step::BwdShape<D::C, D::HID>::PARTIAL;
        *dp = (int64_t)N * H * W * 4 * C;
        *updating = (int64_t)N * H * W;
        return 0;
    });
}

int ref_backward(const float *x, const float *gy, const uint8_t *alive, const float *w1, const float *b1, const float *w2,
                 float *gx, float *dw1, float *db1, float *dw2, void *packed, float *dp, uint8_t *updating, float *partial,
                 int N, int K, int C, int HID, int H, int W, int B, uint64_t seed, float rate, int fp32, int growing,
                 void *stream)
{
    return dispatch(C, HID, fp32, rate < 1.f, growing, [&](auto I) {
        using D = decltype(I);
        using BW = nca_step::BackwardWeights<D::C, D::HID, D::FP32>;
        using BS = nca_step::BwdShape<D::C, D::HID>;
        const cudaStream_t st = (cudaStream_t)stream;
        BW *pk = reinterpret_cast<BW *>(packed);
        nca_step::pack_kernel<D::C, D::HID, D::FP32><<<K, 256, 0, st>>>(w1, b1, w2, pk);
        auto kernel = nca_step::backward_kernel<D::C, D::HID, D::FP32, D::STOCH, D::ALIVE>;
        constexpr int smem = sizeof(nca_step::BackwardSmem<D::C, D::HID, nca_step::bwd_tile_h(D::STOCH)>);
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        const int blocks = bwd_blocks_per_image(H, W, D::STOCH);
        kernel<<<dim3(blocks, N), nca_step::BWD_THREADS, smem, st>>>(x, gy, alive, pk, dp, updating, partial, 0, B, H, W,
                                                                     seed, rate);
        const dim3 adj_grid(ceil_div(W, nca_step::ADJ_PIX) * ceil_div(H, nca_step::adj_rows(D::ALIVE)), N);
        nca_step::adjoint_kernel<D::C, D::ALIVE><<<adj_grid, nca_step::ADJ_PIX * D::C / nca_step::adj_cpt(D::ALIVE), 0, st>>>(
            dp, updating, gy, alive, gx, H, W);
        nca_step::reduce_kernel<D::C, D::HID><<<dim3(ceil_div(BS::PARTIAL, 256), K), 256, 0, st>>>(partial, B * blocks, dw1,
                                                                                                 db1, dw2);
        return (int)cudaGetLastError();
    });
}

}  // extern "C"
