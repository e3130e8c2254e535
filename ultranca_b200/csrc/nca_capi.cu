// C-ABI of the fused NCA step (the drop-in boundary under ultranca_b200/nca_ops.py). Every entry point takes plain
// device pointers and sizes, launches asynchronously on the caller's stream and returns 0, or a nonzero status with the
// message in nca_last_error(). Nothing here allocates device memory: the caller passes every buffer.
//
// Mirrors the reference's nanobind module (ncaops/nca_cuda.cu:333-353): forward, rollout, backward_workspace, backward,
// update_mask, with the same argument meaning and error behaviour (shape / size mismatch and unsupported sizes are
// errors, ncaops/nca_cuda.cu:35-52,75,128-145,262-284; launch errors are checked after every launch, :23-33).
// Per-device state (SM count, kernel attributes, occupancy) is cached per device, not process-wide.
#include <cuda_runtime.h>
#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <numeric>
#include <stdexcept>
#include <utility>
#include <string>

#include "nca_kernels.cuh"
#include "nca_aux.cuh"
#include "nca_rows.cuh"
#include "nca_train.cuh"
#include "../../include/ultranca_b200.h"

namespace unca {
namespace {

thread_local std::string g_last_error;

struct Error : std::runtime_error {
    int code;
    Error(int c, const std::string &m) : std::runtime_error(m), code(c) {}
};

[[noreturn]] void fail(int code, const char *fmt, ...)
{
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    throw Error(code, buf);
}

#define CUDA_OK(call)                                                                                         \
    do {                                                                                                      \
        cudaError_t e_ = (call);                                                                              \
        if (e_ != cudaSuccess)                                                                                \
            fail(NCA_ERR_CUDA, "CUDA error at %s:%d - %s", __FILE__, __LINE__, cudaGetErrorString(e_));      \
    } while (0)

template <class F>
int guarded(F &&f)
{
    try {
        f();
        return NCA_OK;
    } catch (const Error &e) {
        g_last_error = e.what();
        return e.code;
    } catch (const std::exception &e) {
        g_last_error = e.what();
        return NCA_ERR_INTERNAL;
    }
}

// ---------------------------------------------------------------- per-device cache
constexpr int MAX_DEV = 64;
struct DeviceInfo {
    bool init = false;
    int sms = 0;
    int smem_optin = 0;
};
DeviceInfo g_dev[MAX_DEV];
std::mutex g_mutex;

int current_device()
{
    int d = 0;
    CUDA_OK(cudaGetDevice(&d));
    if (d < 0 || d >= MAX_DEV)
        fail(NCA_ERR_CUDA, "device index %d out of range", d);
    return d;
}

const DeviceInfo &device_info()
{
    const int d = current_device();
    std::lock_guard<std::mutex> lk(g_mutex);
    DeviceInfo &di = g_dev[d];
    if (!di.init) {
        CUDA_OK(cudaDeviceGetAttribute(&di.sms, cudaDevAttrMultiProcessorCount, d));
        CUDA_OK(cudaDeviceGetAttribute(&di.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, d));
        di.init = true;
    }
    return di;
}

// Resident CTAs per SM of `kernel` launched with `threads` threads and `smem` bytes of dynamic shared memory:
// min over registers (allocated per warp in units of 8 per thread), shared memory (plus the 1 KB the driver reserves
// per CTA), warps (64 per SM) and Tensor Memory columns (512 per SM). Computed from the kernel's attributes rather
// than cudaOccupancyMaxActiveBlocksPerMultiprocessor, which answers 1 for these tcgen05 kernels on this driver where
// the hardware limits (as Nsight Compute reports them) allow more. The step kernels' CTAs never wait on each other,
// so an over-estimate would only cost a second wave, never a hang. Cached per (kernel, device).
std::map<std::pair<const void *, int>, int> g_occupancy;

template <class K>
int ctas_per_sm(K kernel, size_t smem, int tmem_cols, int threads = 128)
{
    const int d = current_device();
    std::lock_guard<std::mutex> lk(g_mutex);
    const auto key = std::make_pair(reinterpret_cast<const void *>(kernel), d);
    auto it = g_occupancy.find(key);
    if (it != g_occupancy.end())
        return it->second;
    CUDA_OK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    CUDA_OK(cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
    cudaFuncAttributes fa{};
    CUDA_OK(cudaFuncGetAttributes(&fa, kernel));
    int smem_sm = 0, regs_sm = 0, warps_sm = 0;
    CUDA_OK(cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, d));
    CUDA_OK(cudaDeviceGetAttribute(&regs_sm, cudaDevAttrMaxRegistersPerMultiprocessor, d));
    CUDA_OK(cudaDeviceGetAttribute(&warps_sm, cudaDevAttrMaxThreadsPerMultiProcessor, d));
    warps_sm /= 32;
    const int warps = (threads + 31) / 32;
    const int regs_warp = ((fa.numRegs + 7) / 8) * 8 * 32;
    int b = std::min(regs_sm / (regs_warp * warps), warps_sm / warps);
    b = std::min<int>(b, (int)(smem_sm / (smem + fa.sharedSizeBytes + 1024)));
    if (tmem_cols > 0)
        b = std::min(b, 512 / tmem_cols);
    b = std::max(b, 1);
    g_occupancy[key] = b;
    return b;
}

// Sets the dynamic shared memory limit of `kernel` once per device.
template <class K>
void set_smem_once(K kernel, size_t smem)
{
    const int d = current_device();
    std::lock_guard<std::mutex> lk(g_mutex);
    const auto key = std::make_pair(reinterpret_cast<const void *>(kernel), -1 - d);
    if (g_occupancy.count(key))
        return;
    CUDA_OK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    CUDA_OK(cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
    g_occupancy[key] = 1;
}

// ---------------------------------------------------------------- dispatch
template <int C_, int HID_, bool FP32_, bool GROW_>
struct Inst {
    static constexpr int C = C_, HID = HID_;
    static constexpr bool FP32 = FP32_, GROW = GROW_;
};

template <class F>
void dispatch(int64_t C, int64_t HID, bool fp32, bool growing, F &&f)
{
    auto go = [&](auto fp, auto gr) {
        constexpr bool FP = decltype(fp)::value, GR = decltype(gr)::value;
        if (C == 12 && HID == 96)
            return f(Inst<12, 96, FP, GR>{});
        if (C == 16 && HID == 128)
            return f(Inst<16, 128, FP, GR>{});
        fail(NCA_ERR_UNSUPPORTED, "no kernel instantiated for channels=%lld, hidden=%lld", (long long)C, (long long)HID);
    };
    if (fp32) {
        if (growing)
            go(std::true_type{}, std::true_type{});
        else
            go(std::true_type{}, std::false_type{});
    } else {
        if (growing)
            go(std::false_type{}, std::true_type{});
        else
            go(std::false_type{}, std::false_type{});
    }
}

// Visiting order of an NCA's M tiles in the growing tile kernels: u -> u P mod M with P coprime to M near M times the
// golden ratio, so that consecutive tiles (a living region) land far apart and the CTAs sharing an NCA get similar
// numbers of live tiles. Only where a CTA's share of the launch is under half an image (tiles per CTA < tiles per image
// / 2): there one CTA may hold most of an image's living region while its neighbours idle. With larger shares every
// CTA already spans whole images, and the natural order keeps the locality of consecutive tiles (measured: 72 x 72
// grids at 3.5 images per CTA ran 25% slower scattered, 128 x 128 ones at 0.4 images per CTA 13% faster). 0: in order.
uint32_t tile_perm_for(int64_t M, int64_t tiles, int64_t grid, int64_t tiles_per_image)
{
    if (M <= 2 || tiles >= grid * (tiles_per_image / 2))
        return 0;
    int64_t P = std::max<int64_t>(1, (int64_t)((double)M * 0.6180339887498949));
    while (std::gcd(P, M) != 1)
        ++P;
    return (uint32_t)P;
}

// The tile kernels index a launch's tiles in 32 bits.
void check_tiles(int64_t tiles)
{
    if (tiles >= ((int64_t)1 << 31))
        fail(NCA_ERR_SHAPE, "too many tiles in one launch (%lld)", (long long)tiles);
}

void check_ptr(const void *p, const char *name)
{
    if (!p)
        fail(NCA_ERR_ARGUMENT, "%s must not be null", name);
}

struct Shape {
    int64_t N, C, H, W, K, HID, B;
};

void validate(const Shape &s, bool growing)
{
    if (s.N <= 0 || s.C <= 0 || s.H <= 0 || s.W <= 0 || s.K <= 0 || s.HID <= 0 || s.B <= 0)
        fail(NCA_ERR_SHAPE, "sizes must be positive (N=%lld C=%lld H=%lld W=%lld K=%lld hidden=%lld B=%lld)",
             (long long)s.N, (long long)s.C, (long long)s.H, (long long)s.W, (long long)s.K, (long long)s.HID, (long long)s.B);
    if (s.N != s.K * s.B)
        fail(NCA_ERR_SHAPE, "x.shape[0] must equal (number of NCAs) * batch_per_nca (%lld != %lld * %lld)", (long long)s.N,
             (long long)s.K, (long long)s.B);
    if (growing && s.C < 4)
        fail(NCA_ERR_SHAPE, "a growing NCA needs at least 4 channels (alpha = channel 3)");
    if (s.H >= (1 << 24) || s.W >= (1 << 24) || s.N >= (1 << 30))
        fail(NCA_ERR_SHAPE, "grid too large");
}

// Persistent grid size of a step kernel (tiles T): the resident CTA slots of the device, at most one CTA per tile.
int grid_for(int64_t T, int per_sm)
{
    const int slots = device_info().sms * per_sm;
    return (int)std::max<int64_t>(1, std::min<int64_t>(T, slots));
}

template <class I>
int fwd_ctas_per_sm()
{
    using D = Dims<I::C, I::HID>;
    auto kernel = I::FP32 ? fwd_kernel<I::C, I::HID, false, I::GROW> : fwd_kernel<I::C, I::HID, true, I::GROW>;
    return ctas_per_sm(kernel, D::fwd_smem(), I::FP32 ? 0 : D::FWD_TMEM, I::FP32 ? 128 : 128 * FWD_TILE_PARTS);
}

template <class I>
int bwd_ctas_per_sm()
{
    using D = Dims<I::C, I::HID>;
    if (I::FP32)
        return ctas_per_sm(bwd_kernel_cc<I::C, I::HID, I::GROW>, D::bwd_smem_cc(), 0);
    return ctas_per_sm(bwd_kernel_tc<I::C, I::HID, I::GROW>, D::bwd_smem_tc(I::GROW), D::BWD_TMEM, 128 * BWD_TILE_PARTS);
}

// Row-streaming kernels (the benchmark's hot path): TF32 texture NCAs whose rows are whole 16-byte multiples that
// fit one 128-lane tile; every other case runs the tile kernels.
constexpr int FWD_ROWS_PARTS = 2, BWD_ROWS_PARTS = 4;
bool rows_path(const Shape &s, bool fp32, bool growing)
{
    return !fp32 && !growing && s.C == 12 && s.HID == 96 && s.W <= 128 && s.W % 4 == 0;
}
// Wider rows (W a multiple of 128 from 256 on): both row kernels over column strips of 128 (the backward plus the
// edge fix-up).
bool strip_path(const Shape &s, bool fp32, bool growing)
{
    return !fp32 && !growing && s.C == 12 && s.HID == 96 && s.W >= 256 && s.W % 128 == 0;
}
// The backward runs a row kernel (one tile per row, or strips) for this shape.
bool bwd_rows_path(const Shape &s, bool fp32, bool growing) { return rows_path(s, fp32, growing) || strip_path(s, fp32, growing); }
bool aligned16(const void *p) { return ((uintptr_t)p & 15) == 0; }

// Launch of a row kernel as a programmatic dependent of the previous kernel on the stream: once every CTA of that
// kernel has started (the row kernels signal it first thing), this one is launched; its CTAs take the SMs the
// previous kernel's CTAs free and run their set-up (barriers, TMEM, update masks, the first NCA's weights) under the
// previous kernel's tail, then wait for it to complete (griddepcontrol.wait) before touching the state it writes.
// The grids are persistent (at most the resident CTA slots), so a waiting dependent never holds an SM that an
// unstarted CTA of the previous kernel needs. In a captured CUDA graph the dependency becomes a programmatic edge.
template <class Kern>
void launch_pdl(Kern kern, int grid, int threads, size_t smem, cudaStream_t st, const StepArgs &a)
{
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3((unsigned)threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    CUDA_OK(cudaLaunchKernelEx(&cfg, kern, a));
}

// Switch costs (quarter rows) of the cost-balanced row bands, measured per CTA on the B200 (config 1, per-CTA clock
// stamps against band composition): a band that crosses into another image costs the forward ~2.6 rows and the
// backward ~2.7 rows more (halo rows, pipeline drain and refill), one that crosses into another NCA ~8.9 and ~4.0
// rows in all (weights restaged; the backward also flushes its weight-gradient accumulator, by L2 reductions).
constexpr int FWD_BAND_S4 = 10, FWD_BAND_N4 = 25, BWD_BAND_S4 = 11, BWD_BAND_N4 = 5;

Bands fwd_bands(const Shape &s, int G) { return Bands{s.N * s.H, s.H, s.B * s.H, G, FWD_BAND_S4, FWD_BAND_N4}; }
Bands bwd_bands(const Shape &s, int G) { return Bands{s.N * s.H, s.H, s.B * s.H, G, BWD_BAND_S4, BWD_BAND_N4}; }

int fwd_rows_grid(const Shape &s)
{
    using FR = FwdRows<12, 96, FWD_ROWS_PARTS>;
    using FS = FwdRows<12, 96, FWD_ROWS_PARTS, true>;
    const bool strip = s.W > 128;
    const int per = strip ? ctas_per_sm(fwd_rows_kernel<12, 96, FWD_ROWS_PARTS, true>, FS::smem(), FS::TMEM, FS::THREADS)
                          : ctas_per_sm(fwd_rows_kernel<12, 96, FWD_ROWS_PARTS>, FR::smem(), FR::TMEM, FR::THREADS);
    // each CTA draws the update masks of its rows (times the column strips) into shared memory: at most MAXROWS
    const int64_t rows = s.N * s.H, maxrows = strip ? FS::MAXROWS / (s.W / 128) : FR::MAXROWS;
    int64_t G = std::max<int64_t>(grid_for(rows, per), std::min<int64_t>((rows + maxrows - 1) / maxrows, rows));
    // a band holds at most cost(T) / (4 G) + (4 + s4 + n4) / 4 + 1 rows: grow the grid until that fits
    while (G < rows && band_cost(fwd_bands(s, (int)G), rows) / (4 * G) + (4 + FWD_BAND_S4 + FWD_BAND_N4) / 4 + 1 >
                           maxrows)
        ++G;
    return (int)G;
}
int bwd_rows_grid(const Shape &s)
{
    using BR = BwdRows<12, 96, BWD_ROWS_PARTS>;
    const int per = ctas_per_sm(bwd_rows_kernel<12, 96, BWD_ROWS_PARTS, false>, BR::smem(), BR::TMEM, BR::THREADS);
    return grid_for(s.N * s.H, per);
}

// seed_dev != nullptr: the kernels read the rollout seed there and derive step `step`'s seed themselves.
// Growing: the forward computes the alive mask in its epilogue and writes alive (alpha is not used). reuse (growing
// rollouts from their third step): alive holds this destination's map of two steps ago, and dead tiles skip the cells
// that were dead there (they already hold state 0 and alive 0).
void launch_forward(const float *x, const float *w1, const float *b1, const float *w2, float *y, float *alpha,
                    uint8_t *alive, const Shape &s, uint64_t seed, float rate, bool fp32, bool growing, int64_t n_offset,
                    cudaStream_t stream, const uint64_t *seed_dev = nullptr, int64_t step = 0, bool reuse = false)
{
    StepArgs a{};
    a.alive_out = alive;
    a.reuse = reuse ? 1 : 0;
    a.x = x; a.w1 = w1; a.b1 = b1; a.w2 = w2; a.y = y; a.alpha = alpha;
    a.N = (int)s.N; a.B = (int)s.B; a.H = (int)s.H; a.W = (int)s.W;
    a.seed = seed; a.rate = rate; a.n_offset = n_offset;
    a.seed_dev = seed_dev; a.step = step;
    if (rows_path(s, fp32, growing) && aligned16(x) && aligned16(y)) {
        using FR = FwdRows<12, 96, FWD_ROWS_PARTS>;
        a.band_s4 = FWD_BAND_S4;
        a.band_n4 = FWD_BAND_N4;
        launch_pdl(fwd_rows_kernel<12, 96, FWD_ROWS_PARTS>, fwd_rows_grid(s), FR::THREADS, FR::smem(), stream, a);
        CUDA_OK(cudaGetLastError());
        return;
    }
    if (strip_path(s, fp32, growing) && aligned16(x) && aligned16(y)) {  // column strips of 128
        using FS = FwdRows<12, 96, FWD_ROWS_PARTS, true>;
        a.band_s4 = FWD_BAND_S4;
        a.band_n4 = FWD_BAND_N4;
        const int grid = fwd_rows_grid(s);  // sets the kernel's shared-memory limit (occupancy query) first
        launch_pdl(fwd_rows_kernel<12, 96, FWD_ROWS_PARTS, true>, grid, FS::THREADS, FS::smem(), stream, a);
        CUDA_OK(cudaGetLastError());
        return;
    }
    dispatch(s.C, s.HID, fp32, growing, [&](auto I) {
        using II = decltype(I);
        using D = Dims<II::C, II::HID>;
        const TileGeom g = II::GROW ? make_grow_fwd_geom((int)s.H, (int)s.W) : make_geom((int)s.H, (int)s.W);
        check_tiles(s.N * g.tiles_per_image);
        const int G = grid_for(s.N * g.tiles_per_image, fwd_ctas_per_sm<II>());
        a.tile_perm = II::GROW ? tile_perm_for(s.B * g.tiles_per_image, s.N * g.tiles_per_image, G, g.tiles_per_image) : 0;
        // (the scattered tile order is a kernel instance of its own; growing NCAs only)
        auto go = [&](auto kern, int threads) {
            set_smem_once(kern, D::fwd_smem());
            kern<<<G, threads, D::fwd_smem(), stream>>>(a);
        };
        if constexpr (II::GROW) {
            if (a.tile_perm != 0) {
                if (II::FP32)
                    go(fwd_kernel<II::C, II::HID, false, true, true>, 128);
                else
                    go(fwd_kernel<II::C, II::HID, true, true, true>, 128 * FWD_TILE_PARTS);
                CUDA_OK(cudaGetLastError());
                return;
            }
        }
        if (II::FP32)
            fwd_kernel<II::C, II::HID, false, II::GROW><<<G, 128, D::fwd_smem(), stream>>>(a);
        else
            fwd_kernel<II::C, II::HID, true, II::GROW><<<G, 128 * FWD_TILE_PARTS, D::fwd_smem(), stream>>>(a);
        CUDA_OK(cudaGetLastError());
    });
}

// Workspaces of backward(): dp floats, partial floats (both exact), grid size.
struct BwdWork {
    int64_t dp_floats, partial_floats;
    int grid;
};

BwdWork backward_work(const Shape &s, bool fp32, bool growing)
{
    BwdWork w{};
    dispatch(s.C, s.HID, fp32, growing, [&](auto I) {
        using II = decltype(I);
        using D = Dims<II::C, II::HID>;
        const TileGeom g = make_geom((int)s.H, (int)s.W, II::GROW);
        check_tiles(s.N * g.tiles_per_image);
        w.grid = grid_for(s.N * g.tiles_per_image, bwd_ctas_per_sm<II>());
        w.dp_floats = s.N * D::PIN * s.H * s.W;
        int slots = w.grid;
        if (bwd_rows_path(s, fp32, growing))  // either kernel may run (the row kernel needs 16-byte aligned rows);
            slots = std::max(slots, bwd_rows_grid(s));  // the strip kernel's edge scratch fits in the dp scratch
        w.partial_floats = (int64_t)(slots + s.K - 1) * D::PART;
    });
    return w;
}

AdamArgs make_adam_args(float *param0, float *param1, float *param2, const float *grad0, const float *grad1,
                        const float *grad2, float *m0, float *m1, float *m2, float *v0, float *v1, float *v2, int64_t K,
                        int64_t numel0, int64_t numel1, int64_t numel2, int64_t *iteration, float lr, float beta1,
                        float beta2, float eps, float gamma, const int64_t *milestones, int n_milestones)
{
    float *p[3] = {param0, param1, param2}, *m[3] = {m0, m1, m2}, *v[3] = {v0, v1, v2};
    const float *g[3] = {grad0, grad1, grad2};
    const int64_t ne[3] = {numel0, numel1, numel2};
    if (K <= 0)
        fail(NCA_ERR_SHAPE, "K must be positive");
    if (n_milestones < 0 || n_milestones > 8 || (n_milestones > 0 && !milestones))
        fail(NCA_ERR_ARGUMENT, "at most 8 milestones");
    check_ptr(iteration, "iteration");
    AdamArgs a{};
    for (int i = 0; i < 3; ++i) {
        check_ptr(p[i], "param"); check_ptr(g[i], "grad"); check_ptr(m[i], "m"); check_ptr(v[i], "v");
        if (ne[i] <= 0)
            fail(NCA_ERR_SHAPE, "numel must be positive");
        a.t[i] = AdamTensor{p[i], m[i], v[i], g[i], ne[i]};
    }
    a.iteration = iteration;
    a.lr = lr; a.beta1 = beta1; a.beta2 = beta2; a.eps = eps; a.gamma = gamma;
    a.n_milestones = n_milestones;
    for (int i = 0; i < n_milestones; ++i)
        a.milestones[i] = milestones[i];
    return a;
}

int grid_stride_blocks(int64_t work)
{
    const int64_t cap = (int64_t)device_info().sms * 8;
    return (int)std::max<int64_t>(1, std::min<int64_t>(cap, (work + 255) / 256));
}

}  // namespace
}  // namespace unca

using namespace unca;

extern "C" {

const char *nca_last_error(void) { return g_last_error.c_str(); }

int nca_version(void) { return NCA_ABI_VERSION; }

int nca_forward(const float *x, const float *w1, const float *b1, const float *w2, float *y, float *alpha, uint8_t *alive,
                int64_t N, int64_t C, int64_t H, int64_t W, int64_t K, int64_t hidden, uint32_t batch_per_nca,
                uint64_t seed, float update_rate, int fp32, int growing, int64_t image_offset, void *stream)
{
    return guarded([&] {
        const Shape s{N, C, H, W, K, hidden, (int64_t)batch_per_nca};
        validate(s, growing);
        check_ptr(x, "x"); check_ptr(w1, "w1"); check_ptr(b1, "b1"); check_ptr(w2, "w2"); check_ptr(y, "y");
        if (growing)
            check_ptr(alive, "alive");  // alpha: unused (the alive mask is computed in the step's epilogue)
        launch_forward(x, w1, b1, w2, y, alpha, alive, s, seed, update_rate, fp32, growing, image_offset,
                       static_cast<cudaStream_t>(stream));
    });
}

int nca_forward_dseed(const float *x, const float *w1, const float *b1, const float *w2, float *y, float *alpha,
                      uint8_t *alive, int64_t N, int64_t C, int64_t H, int64_t W, int64_t K, int64_t hidden,
                      uint32_t batch_per_nca, const uint64_t *seed_dev, int64_t step, float update_rate, int fp32,
                      int growing, int64_t image_offset, void *stream)
{
    return guarded([&] {
        const Shape s{N, C, H, W, K, hidden, (int64_t)batch_per_nca};
        validate(s, growing);
        check_ptr(x, "x"); check_ptr(w1, "w1"); check_ptr(b1, "b1"); check_ptr(w2, "w2"); check_ptr(y, "y");
        check_ptr(seed_dev, "seed_dev");
        if (step < 0)
            fail(NCA_ERR_ARGUMENT, "step must be >= 0");
        if (growing)
            check_ptr(alive, "alive");  // alpha: unused (the alive mask is computed in the step's epilogue)
        launch_forward(x, w1, b1, w2, y, alpha, alive, s, 0, update_rate, fp32, growing, image_offset,
                       static_cast<cudaStream_t>(stream), seed_dev, step);
    });
}

int nca_rollout(const float *x, const float *w1, const float *b1, const float *w2, float *y, float *tmp, float *alpha,
                uint8_t *alive, int64_t N, int64_t C, int64_t H, int64_t W, int64_t K, int64_t hidden, uint32_t steps,
                uint32_t batch_per_nca, uint64_t seed, float update_rate, int fp32, int growing, int64_t image_offset,
                void *stream)
{
    return guarded([&] {
        const Shape s{N, C, H, W, K, hidden, (int64_t)batch_per_nca};
        validate(s, growing);
        check_ptr(x, "x"); check_ptr(w1, "w1"); check_ptr(b1, "b1"); check_ptr(w2, "w2"); check_ptr(y, "y");
        if (steps > 1)
            check_ptr(tmp, "tmp");
        if (growing)
            check_ptr(alive, "alive");  // alpha: unused (the alive mask is computed in the step's epilogue)
        const auto st = static_cast<cudaStream_t>(stream);
        if (steps == 0)
            CUDA_OK(cudaMemcpyAsync(y, x, (size_t)(N * C * H * W) * sizeof(float), cudaMemcpyDeviceToDevice, st));
        const float *src = x;
        for (uint32_t i = 0; i < steps; ++i) {  // ping-pong so that the result ends in y (x is not modified)
            float *dst = (steps - i) % 2 ? y : tmp;
            // growing: one alive map per destination buffer (steps of the same parity write the same buffer)
            uint8_t *map = growing ? alive + (size_t)(i % 2) * (size_t)(N * H * W) : alive;
            launch_forward(src, w1, b1, w2, dst, alpha, map, s, nca_step_seed(seed, i), update_rate, fp32, growing,
                           image_offset, st, nullptr, 0, growing && i >= 2);
            src = dst;
        }
    });
}

uint64_t nca_step_seed(uint64_t seed, uint64_t i) { return splitmix_step(seed, i); }

int nca_backward_workspace(int64_t C, int64_t hidden, int fp32, int64_t N, int64_t H, int64_t W, int64_t K,
                           float update_rate, int growing, int64_t *dp_floats, int64_t *partial_floats, int64_t *chunk)
{
    (void)update_rate;
    return guarded([&] {
        const Shape s{N, C, H, W, K, hidden, K > 0 ? N / K : 0};
        validate(s, growing);
        const BwdWork w = backward_work(s, fp32, growing);
        if (dp_floats)
            *dp_floats = w.dp_floats;
        if (partial_floats)
            *partial_floats = w.partial_floats;
        if (chunk)
            *chunk = N;  // one launch over all images (B200: the reference also picks one launch, nca_cuda.cu:211-212)
    });
}

}  // extern "C"

namespace {
int backward_stages_impl(const float *x, const float *gy, const uint8_t *alive, const float *w1, const float *b1,
                         const float *w2, float *gx, float *dw1, float *db1, float *dw2, float *dp, int64_t dp_floats,
                         float *partial, int64_t partial_floats, int64_t N, int64_t C, int64_t H, int64_t W, int64_t K,
                         int64_t hidden, uint32_t batch_per_nca, uint64_t seed, const uint64_t *seed_dev, int64_t step,
                         float update_rate, int fp32, int growing, int64_t image_offset, int accumulate, int stages,
                         void *stream)
{
    return guarded([&] {
        const Shape s{N, C, H, W, K, hidden, (int64_t)batch_per_nca};
        validate(s, growing);
        if ((stages & 15) == 0 || stages > 31)
            fail(NCA_ERR_ARGUMENT, "stages must be a mask of NCA_STAGE_* bits with at least one stage");
        if ((stages & NCA_STAGE_PARTIAL_ADD) && !(stages & NCA_STAGE_MAIN))
            fail(NCA_ERR_ARGUMENT, "NCA_STAGE_PARTIAL_ADD applies to NCA_STAGE_MAIN");
        check_ptr(x, "x"); check_ptr(gy, "gy"); check_ptr(w1, "w1"); check_ptr(b1, "b1"); check_ptr(w2, "w2");
        check_ptr(gx, "gx"); check_ptr(dw1, "dw1"); check_ptr(db1, "db1"); check_ptr(dw2, "dw2"); check_ptr(dp, "dp");
        check_ptr(partial, "partial");
        if (growing)
            check_ptr(alive, "alive");
        const BwdWork w = backward_work(s, fp32, growing);
        if (dp_floats < w.dp_floats)
            fail(NCA_ERR_SHAPE, "dp workspace too small: %lld floats, need %lld", (long long)dp_floats, (long long)w.dp_floats);
        if (partial_floats < w.partial_floats)
            fail(NCA_ERR_SHAPE, "partial workspace too small: %lld floats, need %lld", (long long)partial_floats,
                 (long long)w.partial_floats);
        const auto st = static_cast<cudaStream_t>(stream);
        dispatch(C, hidden, fp32, growing, [&](auto I) {
            using II = decltype(I);
            using D = Dims<II::C, II::HID>;
            StepArgs a{};
            a.x = x; a.w1 = w1; a.b1 = b1; a.w2 = w2; a.gy = gy; a.alive = alive; a.dp = dp; a.partial = partial;
            a.N = (int)N; a.B = (int)batch_per_nca; a.H = (int)H; a.W = (int)W;
            a.seed = seed; a.rate = update_rate; a.n_offset = image_offset;
            a.seed_dev = seed_dev; a.step = step;
            a.partial_add = (stages & NCA_STAGE_PARTIAL_ADD) ? 1 : 0;
            const TileGeom g = make_geom((int)H, (int)W, II::GROW);
            a.tile_perm = II::GROW ? tile_perm_for((int64_t)batch_per_nca * g.tiles_per_image, N * g.tiles_per_image, w.grid,
                                                   g.tiles_per_image)
                                   : 0;
            const bool strip = strip_path(s, fp32, growing) && aligned16(x) && aligned16(gy) && aligned16(gx) &&
                               aligned16(dp);
            const bool rows = strip || (rows_path(s, fp32, growing) && aligned16(x) && aligned16(gy) && aligned16(gx));
            int64_t units = N * g.tiles_per_image, units_per_nca = (int64_t)batch_per_nca * g.tiles_per_image;
            int grid = w.grid;
            Bands bands{units, 1, 1, grid, 0, 0};  // tile path: the uniform split
            if (rows) {  // one launch: backward + fused adjoint; the dp scratch is not used
                using BR = BwdRows<12, 96, BWD_ROWS_PARTS>;
                grid = bwd_rows_grid(s);
                bands = bwd_bands(s, grid);
                a.band_s4 = BWD_BAND_S4;
                a.band_n4 = BWD_BAND_N4;
                units = N * H;
                units_per_nca = (int64_t)batch_per_nca * H;
                a.gx = gx;
                if (strip) {  // column strips; the adjoint stage adds the cross-strip terms from the edge scratch (dp)
                    using BS = BwdRows<12, 96, BWD_ROWS_PARTS, true>;
                    if (stages & NCA_STAGE_MAIN) {
                        if (stages & NCA_STAGE_X_STABLE) {
                            set_smem_once(bwd_rows_kernel<12, 96, BWD_ROWS_PARTS, true, true>, BS::smem());
                            launch_pdl(bwd_rows_kernel<12, 96, BWD_ROWS_PARTS, true, true>, grid, BS::THREADS,
                                       BS::smem(), st, a);
                        } else {
                            set_smem_once(bwd_rows_kernel<12, 96, BWD_ROWS_PARTS, false, true>, BS::smem());
                            launch_pdl(bwd_rows_kernel<12, 96, BWD_ROWS_PARTS, false, true>, grid, BS::THREADS,
                                       BS::smem(), st, a);
                        }
                        CUDA_OK(cudaGetLastError());
                    }
                    if (stages & NCA_STAGE_ADJOINT) {
                        const int64_t total = N * H * (W / 128) * 2 * 12;
                        const int blocks = (int)std::min<int64_t>((total + 255) / 256, (int64_t)device_info().sms * 8);
                        strip_edge_fixup_kernel<12><<<blocks, 256, 0, st>>>(reinterpret_cast<const float4 *>(dp), gx,
                                                                           (int)N, (int)H, (int)W);
                        CUDA_OK(cudaGetLastError());
                    }
                } else if (stages & NCA_STAGE_MAIN) {
                    if (stages & NCA_STAGE_X_STABLE) {
                        set_smem_once(bwd_rows_kernel<12, 96, BWD_ROWS_PARTS, true>, BR::smem());
                        launch_pdl(bwd_rows_kernel<12, 96, BWD_ROWS_PARTS, true>, grid, BR::THREADS, BR::smem(), st, a);
                    } else {
                        launch_pdl(bwd_rows_kernel<12, 96, BWD_ROWS_PARTS, false>, grid, BR::THREADS, BR::smem(), st,
                                   a);
                    }
                    CUDA_OK(cudaGetLastError());
                }
            } else {
                if ((stages & NCA_STAGE_MAIN) && II::GROW && a.tile_perm != 0) {  // the scattered tile order
                    if constexpr (II::GROW) {
                        if (II::FP32) {
                            set_smem_once(bwd_kernel_cc<II::C, II::HID, true, true>, D::bwd_smem_cc());
                            bwd_kernel_cc<II::C, II::HID, true, true><<<w.grid, 128, D::bwd_smem_cc(), st>>>(a);
                        } else {
                            set_smem_once(bwd_kernel_tc<II::C, II::HID, true, true>, D::bwd_smem_tc(true));
                            bwd_kernel_tc<II::C, II::HID, true, true><<<w.grid, 128 * BWD_TILE_PARTS, D::bwd_smem_tc(true), st>>>(a);
                        }
                    }
                    CUDA_OK(cudaGetLastError());
                } else if (stages & NCA_STAGE_MAIN) {
                    if (II::FP32)
                        bwd_kernel_cc<II::C, II::HID, II::GROW><<<w.grid, 128, D::bwd_smem_cc(), st>>>(a);
                    else
                        bwd_kernel_tc<II::C, II::HID, II::GROW><<<w.grid, 128 * BWD_TILE_PARTS, D::bwd_smem_tc(II::GROW), st>>>(a);
                    CUDA_OK(cudaGetLastError());
                }
                if (stages & NCA_STAGE_ADJOINT) {
                    const size_t adj_smem = (size_t)(D::PIN / ADJ_HALVES) * (ADJ_TH + 2) * (ADJ_TW + 2) * sizeof(float);
                    set_smem_once(adjoint_kernel<II::C, II::GROW>, adj_smem);
                    // persistent: the resident blocks loop over the 8 x 32 blocks of all images
                    const int64_t blocks = N * (int64_t)(((W + ADJ_TW - 1) / ADJ_TW) * ((H + ADJ_TH - 1) / ADJ_TH));
                    check_tiles(blocks);
                    const int per = ctas_per_sm(adjoint_kernel<II::C, II::GROW>, adj_smem, 0, 256);
                    const int agrid = (int)std::min<int64_t>(blocks, (int64_t)device_info().sms * per);
                    adjoint_kernel<II::C, II::GROW><<<agrid, ADJ_TW * ADJ_TH, adj_smem, st>>>(dp, gy, alive, gx, (int)N, (int)H,
                                                                                           (int)W);
                    CUDA_OK(cudaGetLastError());
                }
            }
            if (stages & NCA_STAGE_REDUCE) {
                reduce_kernel<II::C, II::HID><<<dim3((D::PART + 255) / 256, (unsigned)K), 256, 0, st>>>(
                    partial, bands, units_per_nca, dw1, db1, dw2, accumulate);
                CUDA_OK(cudaGetLastError());
            }
        });
    });
}
}  // namespace

extern "C" {

int nca_backward_stages(const float *x, const float *gy, const uint8_t *alive, const float *w1, const float *b1,
                        const float *w2, float *gx, float *dw1, float *db1, float *dw2, float *dp, int64_t dp_floats,
                        float *partial, int64_t partial_floats, int64_t N, int64_t C, int64_t H, int64_t W, int64_t K,
                        int64_t hidden, uint32_t batch_per_nca, uint64_t seed, float update_rate, int fp32, int growing,
                        int64_t image_offset, int accumulate, int stages, void *stream)
{
    return backward_stages_impl(x, gy, alive, w1, b1, w2, gx, dw1, db1, dw2, dp, dp_floats, partial, partial_floats, N,
                                C, H, W, K, hidden, batch_per_nca, seed, nullptr, 0, update_rate, fp32, growing,
                                image_offset, accumulate, stages, stream);
}

int nca_backward_stages_dseed(const float *x, const float *gy, const uint8_t *alive, const float *w1, const float *b1,
                              const float *w2, float *gx, float *dw1, float *db1, float *dw2, float *dp,
                              int64_t dp_floats, float *partial, int64_t partial_floats, int64_t N, int64_t C, int64_t H,
                              int64_t W, int64_t K, int64_t hidden, uint32_t batch_per_nca, const uint64_t *seed_dev,
                              int64_t step, float update_rate, int fp32, int growing, int64_t image_offset,
                              int accumulate, int stages, void *stream)
{
    if (!seed_dev)
        return guarded([] { fail(NCA_ERR_ARGUMENT, "seed_dev is null"); });
    return backward_stages_impl(x, gy, alive, w1, b1, w2, gx, dw1, db1, dw2, dp, dp_floats, partial, partial_floats, N,
                                C, H, W, K, hidden, batch_per_nca, 0, seed_dev, step, update_rate, fp32, growing,
                                image_offset, accumulate, stages, stream);
}

int nca_backward(const float *x, const float *gy, const uint8_t *alive, const float *w1, const float *b1, const float *w2,
                 float *gx, float *dw1, float *db1, float *dw2, float *dp, int64_t dp_floats, float *partial,
                 int64_t partial_floats, int64_t N, int64_t C, int64_t H, int64_t W, int64_t K, int64_t hidden,
                 uint32_t batch_per_nca, uint64_t seed, float update_rate, int fp32, int growing, int64_t image_offset,
                 int accumulate, void *stream)
{
    return nca_backward_stages(x, gy, alive, w1, b1, w2, gx, dw1, db1, dw2, dp, dp_floats, partial, partial_floats, N, C,
                               H, W, K, hidden, batch_per_nca, seed, update_rate, fp32, growing, image_offset, accumulate,
                               NCA_STAGE_MAIN | NCA_STAGE_ADJOINT | NCA_STAGE_REDUCE, stream);
}

int nca_launch_info(int64_t C, int64_t hidden, int fp32, int growing, int64_t N, int64_t H, int64_t W, int64_t K,
                    int32_t *info)
{
    return guarded([&] {
        check_ptr(info, "info");
        const Shape s{N, C, H, W, K, hidden, K > 0 ? N / K : 0};
        validate(s, growing);
        const bool rows = rows_path(s, fp32, growing), brows = bwd_rows_path(s, fp32, growing);
        const BwdWork w = backward_work(s, fp32, growing);
        int fwd_grid = 0, fwd_per = 0;
        dispatch(C, hidden, fp32, growing, [&](auto I) {
            using II = decltype(I);
            const TileGeom g = II::GROW ? make_grow_fwd_geom((int)H, (int)W) : make_geom((int)H, (int)W);
            fwd_per = fwd_ctas_per_sm<II>();
            fwd_grid = grid_for(N * g.tiles_per_image, fwd_per);
        });
        info[0] = rows ? 1 : brows ? 2 : 0;
        info[1] = brows ? fwd_rows_grid(s) : fwd_grid;
        info[2] = brows ? FwdRows<12, 96, FWD_ROWS_PARTS>::THREADS : 128;
        info[3] = brows ? bwd_rows_grid(s) : w.grid;
        info[4] = brows ? BwdRows<12, 96, BWD_ROWS_PARTS>::THREADS : 128;
        info[5] = device_info().sms;
        info[6] = fwd_per;
        info[7] = w.grid;
        // raw occupancy-query results of the row-streaming forward kernel (diagnostic)
        using FR = FwdRows<12, 96, FWD_ROWS_PARTS>;
        int b = -1;
        CUDA_OK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, fwd_rows_kernel<12, 96, FWD_ROWS_PARTS>, FR::THREADS, FR::smem()));
        info[8] = b;
        cudaFuncAttributes fa{};
        CUDA_OK(cudaFuncGetAttributes(&fa, fwd_rows_kernel<12, 96, FWD_ROWS_PARTS>));
        info[9] = fa.numRegs;
        info[10] = fa.maxDynamicSharedSizeBytes;
        info[11] = fa.preferredShmemCarveout;
    });
}

int nca_device_error(int *code, int reset)
{
    return guarded([&] {
        int v = 0;
        CUDA_OK(cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)));
        if (code)
            *code = v;
        if (reset) {
            const int z = 0;
            CUDA_OK(cudaMemcpyToSymbol(g_device_error, &z, sizeof(int)));
        }
    });
}

int nca_update_mask(float *mask, int64_t n, int64_t h, int64_t w, uint64_t seed, float update_rate, int64_t image_offset,
                    void *stream)
{
    return guarded([&] {
        check_ptr(mask, "mask");
        if (n <= 0 || h <= 0 || w <= 0)
            fail(NCA_ERR_SHAPE, "mask sizes must be positive");
        const int64_t total = n * h * w;
        const unsigned blocks = (unsigned)std::min<int64_t>((total + 255) / 256, 65535);
        mask_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(mask, n, (int)h, (int)w, seed, update_rate,
                                                                            image_offset);
        CUDA_OK(cudaGetLastError());
    });
}

int nca_task_loss(const float *x, const float *target, float *gy, float *loss, float *work, int64_t K, int64_t B,
                  int64_t C, int64_t H, int64_t W, int64_t target_channels, float overflow_weight, void *stream)
{
    return guarded([&] {
        check_ptr(x, "x"); check_ptr(target, "target"); check_ptr(gy, "gy"); check_ptr(loss, "loss"); check_ptr(work, "work");
        if (K <= 0 || B <= 0 || H <= 0 || W <= 0 || target_channels < 1 || C < target_channels)
            fail(NCA_ERR_SHAPE, "loss sizes must be positive with 1 <= target_channels <= C (got C=%lld, target "
                 "channels %lld)", (long long)C, (long long)target_channels);
        const auto st = static_cast<cudaStream_t>(stream);
        loss_kernel<<<dim3(LOSS_CHUNKS, (unsigned)K), 256, 0, st>>>(x, target, gy, work, (int)B, (int)C, (int)H, (int)W,
                                                                   (int)target_channels, overflow_weight);
        CUDA_OK(cudaGetLastError());
        loss_final_kernel<<<(unsigned)((K + 127) / 128), 128, 0, st>>>(work, loss, (int)K, B * target_channels * H * W,
                                                                      overflow_weight);
        CUDA_OK(cudaGetLastError());
    });
}

int nca_synthetic_loss(const float *x, const float *target, float *gy, float *loss, float *work, int64_t K, int64_t B,
                       int64_t C, int64_t H, int64_t W, float overflow_weight, void *stream)
{
    return nca_task_loss(x, target, gy, loss, work, K, B, C, H, W, 3, overflow_weight, stream);
}

int nca_adam_step(float *param0, float *param1, float *param2, const float *grad0, const float *grad1, const float *grad2,
                  float *m0, float *m1, float *m2, float *v0, float *v1, float *v2, int64_t K, int64_t numel0,
                  int64_t numel1, int64_t numel2, int64_t *iteration, float lr, float beta1, float beta2, float eps,
                  float gamma, const int64_t *milestones, int n_milestones, void *stream)
{
    return guarded([&] {
        const AdamArgs a = make_adam_args(param0, param1, param2, grad0, grad1, grad2, m0, m1, m2, v0, v1, v2, K, numel0,
                                          numel1, numel2, iteration, lr, beta1, beta2, eps, gamma, milestones,
                                          n_milestones);
        const auto st = static_cast<cudaStream_t>(stream);
        adam_kernel<<<dim3((unsigned)K, 3), 256, 0, st>>>(a);
        CUDA_OK(cudaGetLastError());
        increment_kernel<<<1, 1, 0, st>>>(iteration);
        CUDA_OK(cudaGetLastError());
    });
}

int nca_control_advance(uint64_t *ctl, void *stream)
{
    return guarded([&] {
        check_ptr(ctl, "ctl");
        control_advance_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(ctl);
        CUDA_OK(cudaGetLastError());
    });
}

int nca_pool_sample(const float *pool, float *x0, int64_t *idx, const uint64_t *ctl, int64_t K, int64_t P, int64_t B,
                    int64_t C, int64_t H, int64_t W, int64_t inject_every, int seed_kind, int64_t nca_offset,
                    void *stream)
{
    return guarded([&] {
        check_ptr(pool, "pool"); check_ptr(x0, "x0"); check_ptr(idx, "idx"); check_ptr(ctl, "ctl");
        if (K <= 0 || C <= 0 || H <= 0 || W <= 0 || K > INT32_MAX)
            fail(NCA_ERR_SHAPE, "K, C, H, W must be positive");
        if (B < 1 || B > POOL_MAX_BATCH || P < B || P > INT32_MAX)
            fail(NCA_ERR_ARGUMENT, "need 1 <= B <= %d and B <= pool size (B=%lld, P=%lld)", POOL_MAX_BATCH, (long long)B,
                 (long long)P);
        if (seed_kind != 0 && seed_kind != 1)
            fail(NCA_ERR_ARGUMENT, "seed_kind: 0 texture (zeros), 1 growing (centre cell)");
        if (inject_every < 0 || nca_offset < 0)
            fail(NCA_ERR_ARGUMENT, "inject_every and nca_offset must be >= 0 (inject_every 0: never)");
        const auto st = static_cast<cudaStream_t>(stream);
        const int64_t chw = C * H * W;
        pool_draw_kernel<<<(unsigned)((K + 127) / 128), 128, 0, st>>>(idx, ctl, (int)K, (int)P, (int)B, nca_offset);
        CUDA_OK(cudaGetLastError());
        const bool v4 = chw % 4 == 0 && aligned16(pool) && aligned16(x0);
        const int blocks = grid_stride_blocks(K * B * chw / (v4 ? 4 : 1));
        if (v4)
            pool_gather_kernel<4><<<blocks, 256, 0, st>>>(pool, x0, idx, ctl, (int)K, (int)P, (int)B, (int)H, (int)W,
                                                          chw, inject_every, seed_kind);
        else
            pool_gather_kernel<1><<<blocks, 256, 0, st>>>(pool, x0, idx, ctl, (int)K, (int)P, (int)B, (int)H, (int)W,
                                                          chw, inject_every, seed_kind);
        CUDA_OK(cudaGetLastError());
    });
}

int nca_pool_store(float *pool, const float *x, const int64_t *idx, int64_t K, int64_t P, int64_t B, int64_t C,
                   int64_t H, int64_t W, void *stream)
{
    return guarded([&] {
        check_ptr(pool, "pool"); check_ptr(x, "x"); check_ptr(idx, "idx");
        if (K <= 0 || B <= 0 || P < B || C <= 0 || H <= 0 || W <= 0 || K > INT32_MAX || P > INT32_MAX)
            fail(NCA_ERR_SHAPE, "need positive K, B <= P, C, H, W");
        const auto st = static_cast<cudaStream_t>(stream);
        const int64_t chw = C * H * W;
        const bool v4 = chw % 4 == 0 && aligned16(pool) && aligned16(x);
        const int blocks = grid_stride_blocks(K * B * chw / (v4 ? 4 : 1));
        if (v4)
            pool_store_kernel<4><<<blocks, 256, 0, st>>>(pool, x, idx, (int)K, (int)P, (int)B, chw);
        else
            pool_store_kernel<1><<<blocks, 256, 0, st>>>(pool, x, idx, (int)K, (int)P, (int)B, chw);
        CUDA_OK(cudaGetLastError());
    });
}

int nca_reduce_adam_step(const float *partial, int64_t partial_floats, int64_t N, int64_t C, int64_t H, int64_t W,
                         int64_t K, int64_t hidden, uint32_t batch_per_nca, int fp32, int growing, float *dw1,
                         float *db1, float *dw2, float *w1, float *b1, float *w2, float *m0, float *m1, float *m2,
                         float *v0, float *v1, float *v2, int64_t *iteration, float lr, float beta1, float beta2,
                         float eps, float gamma, const int64_t *milestones, int n_milestones, void *stream)
{
    return guarded([&] {
        const Shape s{N, C, H, W, K, hidden, (int64_t)batch_per_nca};
        validate(s, growing);
        check_ptr(partial, "partial");
        const BwdWork w = backward_work(s, fp32, growing);
        if (partial_floats < w.partial_floats)
            fail(NCA_ERR_SHAPE, "partial workspace too small: %lld floats, need %lld", (long long)partial_floats,
                 (long long)w.partial_floats);
        const AdamArgs a = make_adam_args(w1, b1, w2, dw1, db1, dw2, m0, m1, m2, v0, v1, v2, K, hidden * 4 * C, hidden,
                                          C * hidden, iteration, lr, beta1, beta2, eps, gamma, milestones, n_milestones);
        const auto st = static_cast<cudaStream_t>(stream);
        dispatch(C, hidden, fp32, growing, [&](auto I) {
            using II = decltype(I);
            // the unit decomposition of the backward launches that wrote the partials (the row kernel when its shape
            // qualifies: those launches had 16-byte-aligned x, gy and gx)
            const TileGeom g = make_geom((int)H, (int)W, II::GROW);
            const bool rows = bwd_rows_path(s, fp32, growing);
            const int64_t units = rows ? N * H : N * g.tiles_per_image;
            const int64_t per = rows ? (int64_t)batch_per_nca * H : (int64_t)batch_per_nca * g.tiles_per_image;
            const int grid = rows ? bwd_rows_grid(s) : w.grid;
            if (grid > REDUCE_MAX_SLOTS)
                fail(NCA_ERR_UNSUPPORTED, "backward grid of %d CTAs exceeds the fused reduction's %d slots", grid,
                     REDUCE_MAX_SLOTS);
            const Bands bands = rows ? bwd_bands(s, grid) : Bands{units, 1, 1, grid, 0, 0};
            reduce_adam_kernel<II::C, II::HID><<<dim3((unsigned)K, 3), 256, 0, st>>>(partial, bands, per, a);
            CUDA_OK(cudaGetLastError());
        });
        increment_kernel<<<1, 1, 0, st>>>(iteration);
        CUDA_OK(cudaGetLastError());
    });
}

int nca_umma_selftest(int form, int N, int K, const float *A, const float *B, float *D, void *stream)
{
    return guarded([&] {
        if (form < 0 || form > 3)
            fail(NCA_ERR_ARGUMENT, "self-test form must be 0..3");
        if (N < 16 || N > 128 || N % 16 || K < 8 || K > 128 || K % 8)
            fail(NCA_ERR_ARGUMENT, "self-test sizes: N in 16..128 (multiple of 16), K in 8..128 (multiple of 8)");
        check_ptr(A, "A"); check_ptr(B, "B"); check_ptr(D, "D");
        const size_t smem = 2 * 128 * 128 * sizeof(float) + 1024 + 16;
        set_smem_once(umma_selftest_kernel, smem);
        umma_selftest_kernel<<<1, 128, smem, static_cast<cudaStream_t>(stream)>>>(form, N, K, A, B, D);
        CUDA_OK(cudaGetLastError());
    });
}

int nca_wait_selftest(int64_t limit_ns, unsigned long long *out, void *stream)
{
    return guarded([&] {
        if (limit_ns <= 0 || limit_ns > 1000000000ll)
            fail(NCA_ERR_ARGUMENT, "wait self-test limit must be in (0, 1 s], got %lld ns", (long long)limit_ns);
        check_ptr(out, "out");
        wait_selftest_kernel<<<1, 64, 0, static_cast<cudaStream_t>(stream)>>>((uint64_t)limit_ns, out);
        CUDA_OK(cudaGetLastError());
    });
}

}  // extern "C"

// ---------------------------------------------------------------- backward with library-owned scratch
// nca_backward_static_scratch: the row-streaming backward (bwd_rows_kernel + reduce_kernel) with its only scratch, the
// per-CTA weight-gradient partials, in the file-scope array below instead of a caller-passed workspace. It is for
// callers that cannot allocate device memory at the point where they run the backward: a host runtime whose memory
// is owned by another allocator (a foreign-language binding that only holds the buffers it was given), or code that
// must not grow the device footprint between set-up and the timed or captured loop. The array is part of the loaded
// module: every device that loads this library holds NCA_STATIC_SCRATCH_FLOATS floats (16 MiB) until the process
// exits, whether or not the entry point is ever called.
namespace unca {
namespace {

static __device__ __align__(256) float g_static_scratch[NCA_STATIC_SCRATCH_FLOATS];

// Device address of g_static_scratch on the current device, looked up once per device (in host code the array's
// name stands for the symbol, not for a device address). The lookup may load the module on that device, so the
// first call on a device must come before any stream capture on it.
float *static_scratch_ptr()
{
    const int d = current_device();
    static std::map<int, float *> ptrs;
    std::lock_guard<std::mutex> lk(g_mutex);
    auto it = ptrs.find(d);
    if (it != ptrs.end())
        return it->second;
    float *p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void **>(&p), g_static_scratch);
    if (e != cudaSuccess || p == nullptr)
        fail(NCA_ERR_CUDA, "cudaGetSymbolAddress of the static scratch failed on device %d: %s", d,
             cudaGetErrorString(e));
    ptrs[d] = p;
    return p;
}

}  // namespace
}  // namespace unca

extern "C" int nca_backward_static_scratch(const float *x, const float *gy, const float *w1, const float *b1,
                                           const float *w2, float *gx, float *dw1, float *db1, float *dw2, int64_t N,
                                           int64_t C, int64_t H, int64_t W, int64_t K, int64_t hidden,
                                           uint32_t batch_per_nca, uint64_t seed, float update_rate,
                                           int64_t image_offset, int accumulate, void *stream)
{
    return guarded([&] {
        const Shape s{N, C, H, W, K, hidden, (int64_t)batch_per_nca};
        validate(s, false);
        check_ptr(x, "x"); check_ptr(gy, "gy"); check_ptr(w1, "w1"); check_ptr(b1, "b1"); check_ptr(w2, "w2");
        check_ptr(gx, "gx"); check_ptr(dw1, "dw1"); check_ptr(db1, "db1"); check_ptr(dw2, "dw2");
        if (!rows_path(s, false, false))
            fail(NCA_ERR_UNSUPPORTED, "static-scratch backward: only the TF32 texture row kernel (12 channels, hidden 96, "
                 "W <= 128 and a multiple of 4); got C=%lld hidden=%lld W=%lld", (long long)C, (long long)hidden,
                 (long long)W);
        if (!aligned16(x) || !aligned16(gy) || !aligned16(gx))
            fail(NCA_ERR_ARGUMENT, "static-scratch backward: x, gy and gx must be 16-byte aligned");
        using D = Dims<12, 96>;
        using BR = BwdRows<12, 96, BWD_ROWS_PARTS>;
        const int grid = bwd_rows_grid(s);
        const int64_t need = (int64_t)(grid + K - 1) * D::PART;
        if (need > NCA_STATIC_SCRATCH_FLOATS)
            fail(NCA_ERR_SHAPE, "static-scratch backward: %lld NCAs over %d CTAs need %lld floats of scratch, the static "
                 "array holds %lld (use nca_backward with a caller-allocated workspace)", (long long)K, grid,
                 (long long)need, (long long)NCA_STATIC_SCRATCH_FLOATS);
        float *partial = static_scratch_ptr();
        const auto st = static_cast<cudaStream_t>(stream);
        StepArgs a{};
        a.x = x; a.w1 = w1; a.b1 = b1; a.w2 = w2; a.gy = gy; a.gx = gx; a.partial = partial;
        a.N = (int)N; a.B = (int)batch_per_nca; a.H = (int)H; a.W = (int)W;
        a.seed = seed; a.rate = update_rate; a.n_offset = image_offset;
        a.band_s4 = BWD_BAND_S4;
        a.band_n4 = BWD_BAND_N4;
        // every partial slot the reduction reads is written by the row kernel of the same call: nothing to clear
        bwd_rows_kernel<12, 96, BWD_ROWS_PARTS, false><<<grid, BR::THREADS, BR::smem(), st>>>(a);
        CUDA_OK(cudaGetLastError());
        reduce_kernel<12, 96><<<dim3((D::PART + 255) / 256, (unsigned)K), 256, 0, st>>>(
            partial, bwd_bands(s, grid), (int64_t)batch_per_nca * H, dw1, db1, dw2, accumulate);
        CUDA_OK(cudaGetLastError());
    });
}
