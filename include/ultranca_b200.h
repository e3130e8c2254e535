/*
 * UltraNCA-B200: C-ABI of the fused batched NCA step for NVIDIA B200 (sm_100a).
 *
 * K NCAs with B images each are stacked as N = K B images of C x H x W fp32 state (image n belongs to NCA n / B);
 * weights w1 (K, hidden, 4C), b1 (K, hidden), w2 (K, C, hidden), all C-contiguous device memory.
 * Supported (C, hidden): (12, 96) texture and (16, 128) growing NCAs, as in the reference.
 *
 * Conventions (the reference's nanobind layer, ncaops/nca_cuda.cu, raises RuntimeError; this layer returns codes):
 *   - every function returns NCA_OK (0) or an NCA_ERR_* code, with the message in nca_last_error() (thread-local);
 *   - work is enqueued asynchronously on `stream` (a cudaStream_t; NULL = the legacy default stream);
 *   - no function allocates device memory; workspaces are sized by nca_backward_workspace();
 *   - `fp32` = 0 runs the MLP on TF32 tensor cores (tcgen05), 1 in fp32 (the reference's FP32 accuracy mode);
 *   - `image_offset` is the global index of image 0 (a shard of a multi-GPU job passes its first image, so that the
 *     Philox update mask equals the single-GPU mask); 0 for a single-GPU call.
 */
#ifndef ULTRANCA_B200_H
#define ULTRANCA_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NCA_ABI_VERSION 1

enum {
    NCA_OK = 0,
    NCA_ERR_ARGUMENT = 1,    /* null pointer or invalid scalar */
    NCA_ERR_SHAPE = 2,       /* shape / size mismatch (reference: std::runtime_error from validate_array_shape) */
    NCA_ERR_UNSUPPORTED = 3, /* no kernel for this (channels, hidden) */
    NCA_ERR_CUDA = 4,        /* a CUDA runtime error (launch or API) */
    NCA_ERR_INTERNAL = 5
};

/* Message of the last failed call on this thread (empty if none). */
const char *nca_last_error(void);

/* NCA_ABI_VERSION of the loaded library. */
int nca_version(void);

/* One NCA step x -> y.
 * Replaces nca_cuda.forward (ncaops/nca_cuda.cu:147-155, bound at :335-340).
 * x, y: (N, C, H, W); growing: alive (N, H, W) uint8 output (the alive mask the backward needs), computed in the step
 * kernel's epilogue; alpha is unused (the reference's alpha workspace; may be NULL); alive may be NULL when
 * growing = 0. update_rate >= 1: every cell updates. */
int nca_forward(const float *x, const float *w1, const float *b1, const float *w2, float *y, float *alpha, uint8_t *alive,
                int64_t N, int64_t C, int64_t H, int64_t W, int64_t K, int64_t hidden, uint32_t batch_per_nca,
                uint64_t seed, float update_rate, int fp32, int growing, int64_t image_offset, void *stream);

/* `steps` forward steps from x into y without gradients; step i uses seed nca_step_seed(seed, i); x is not modified;
 * steps = 0 copies x. tmp: workspace like x when steps > 1 (ping-pong). Growing: alive (2N, H, W): one alive map
 * per ping-pong buffer, so that from the third step on a dead tile leaves the cells that were dead in the destination
 * two steps ago untouched (they hold state 0 and alive 0 there); alpha is unused and may be NULL.
 * Replaces nca_cuda.rollout (ncaops/nca_cuda.cu:166-188, bound at :341-344). */
int nca_rollout(const float *x, const float *w1, const float *b1, const float *w2, float *y, float *tmp, float *alpha,
                uint8_t *alive, int64_t N, int64_t C, int64_t H, int64_t W, int64_t K, int64_t hidden, uint32_t steps,
                uint32_t batch_per_nca, uint64_t seed, float update_rate, int fp32, int growing, int64_t image_offset,
                void *stream);

/* splitmix64 seed of rollout step i (ncaops/nca_cuda.cu:157-164). */
uint64_t nca_step_seed(uint64_t seed, uint64_t i);

/* nca_forward whose step seed is read from device memory when the kernels run: nca_step_seed(*seed_dev, step), so
 * that a launch recorded once in a CUDA graph replays with each iteration's rollout seed (seed_dev: a device uint64,
 * e.g. word 3 of a control block, see nca_control_advance). Otherwise identical to nca_forward. No reference
 * counterpart (the reference launches every step from the host). */
int nca_forward_dseed(const float *x, const float *w1, const float *b1, const float *w2, float *y, float *alpha,
                      uint8_t *alive, int64_t N, int64_t C, int64_t H, int64_t W, int64_t K, int64_t hidden,
                      uint32_t batch_per_nca, const uint64_t *seed_dev, int64_t step, float update_rate, int fp32,
                      int growing, int64_t image_offset, void *stream);

/* Workspace sizes of nca_backward for this shape on the current device: dp_floats (the dp scratch, fp32 elements),
 * partial_floats (weight-gradient partials, fp32 elements) and chunk (images per backward launch: always N).
 * Replaces nca_cuda.backward_workspace (ncaops/nca_cuda.cu:235-254, bound at :345-346), whose tuple was
 * (packed bytes per NCA, partial floats per image, images per chunk). */
int nca_backward_workspace(int64_t C, int64_t hidden, int fp32, int64_t N, int64_t H, int64_t W, int64_t K,
                           float update_rate, int growing, int64_t *dp_floats, int64_t *partial_floats, int64_t *chunk);

/* Gradients of one step (same seed, update_rate and, growing, alive mask as its forward): gx (N, C, H, W),
 * dw1 (K, hidden, 4C), db1 (K, hidden), dw2 (K, C, hidden); weight gradients are reduced in a fixed order (bitwise
 * deterministic). accumulate = 1 adds them to dw1 / db1 / dw2 instead of overwriting (a rollout's backward can then
 * sum its steps without extra launches). dp, partial: workspaces of at least the sizes nca_backward_workspace gives.
 * Replaces nca_cuda.backward (ncaops/nca_cuda.cu:256-323, bound at :347-350). */
int nca_backward(const float *x, const float *gy, const uint8_t *alive, const float *w1, const float *b1, const float *w2,
                 float *gx, float *dw1, float *db1, float *dw2, float *dp, int64_t dp_floats, float *partial,
                 int64_t partial_floats, int64_t N, int64_t C, int64_t H, int64_t W, int64_t K, int64_t hidden,
                 uint32_t batch_per_nca, uint64_t seed, float update_rate, int fp32, int growing, int64_t image_offset,
                 int accumulate, void *stream);

/* The three stages of nca_backward, separately: NCA_STAGE_MAIN (recompute p, h; dh, dp into the dp scratch; per-CTA
 * weight-gradient partials), NCA_STAGE_ADJOINT (gx from dp and gy), NCA_STAGE_REDUCE (fixed-order sum of the partials
 * into dw1 / db1 / dw2). Issued in this order on one stream, any subset equals the matching part of nca_backward, so a
 * caller can time or interleave the stages. No reference counterpart: the reference launches them only together,
 * inside nca_cuda.backward (ncaops/nca_cuda.cu:285-322). */
#define NCA_STAGE_MAIN 1
#define NCA_STAGE_ADJOINT 2
#define NCA_STAGE_REDUCE 4
/* With NCA_STAGE_MAIN: add this call's weight-gradient partials to the partial workspace instead of replacing them.
 * A run of calls of one shape (a rollout's backward steps) then needs a single NCA_STAGE_REDUCE at its end; the caller
 * zeroes the partial workspace before the run's first call. No reference counterpart (the reference reduces the
 * weight gradients of every step, ncaops/nca_cuda.cu:285-322). */
#define NCA_STAGE_PARTIAL_ADD 8
/* The row kernels are launched as programmatic dependents of the previous kernel on the stream: their set-up overlaps
 * the tail of a previous step kernel, and they wait for it before touching the state it may write. With this bit
 * the caller declares that x was written before the last launch on this stream of a kernel other than this library's
 * step kernels (for a rollout's saved states: the loss kernel, or the zeroing of the partial workspace, came later),
 * so the backward may start copying x before that wait. No reference counterpart. */
#define NCA_STAGE_X_STABLE 16
int nca_backward_stages(const float *x, const float *gy, const uint8_t *alive, const float *w1, const float *b1,
                        const float *w2, float *gx, float *dw1, float *db1, float *dw2, float *dp, int64_t dp_floats,
                        float *partial, int64_t partial_floats, int64_t N, int64_t C, int64_t H, int64_t W, int64_t K,
                        int64_t hidden, uint32_t batch_per_nca, uint64_t seed, float update_rate, int fp32, int growing,
                        int64_t image_offset, int accumulate, int stages, void *stream);

/* nca_backward_stages with the step seed read from device memory (nca_step_seed(*seed_dev, step)), as
 * nca_forward_dseed. */
int nca_backward_stages_dseed(const float *x, const float *gy, const uint8_t *alive, const float *w1, const float *b1,
                              const float *w2, float *gx, float *dw1, float *db1, float *dw2, float *dp,
                              int64_t dp_floats, float *partial, int64_t partial_floats, int64_t N, int64_t C, int64_t H,
                              int64_t W, int64_t K, int64_t hidden, uint32_t batch_per_nca, const uint64_t *seed_dev,
                              int64_t step, float update_rate, int fp32, int growing, int64_t image_offset,
                              int accumulate, int stages, void *stream);

/* nca_backward for the TF32 texture row kernel (C = 12, hidden = 96, W <= 128 and a multiple of 4; x, gy, gx
 * 16-byte aligned; growing = 0, fp32 = 0) with its scratch held by the library: the weight-gradient partials live in
 * a file-scope device array of NCA_STATIC_SCRATCH_FLOATS floats (16 MiB) that every device which loads this library
 * holds until the process exits. For callers that cannot allocate device memory where they run the backward (a
 * binding that only holds buffers it was handed, or a loop that must not grow the device footprint after set-up);
 * the call allocates nothing. Needs (backward grid + K - 1) x 5856 floats: larger K is rejected with NCA_ERR_SHAPE
 * (about 560 NCAs on 148 SMs); other shapes or modes with NCA_ERR_UNSUPPORTED. The first call on a device looks up
 * the array's address (cudaGetSymbolAddress, which may load the module): make it before any stream capture on that
 * device. Every call shares the one array and nothing in it needs to start at zero; calls that overlap on the GPU
 * (other streams, other host threads) race on it and must be serialised by the caller. Outputs and accumulate as
 * nca_backward. No counterpart in the reference (its backward always takes caller-allocated workspaces). */
#define NCA_STATIC_SCRATCH_FLOATS (4 * 1024 * 1024)
int nca_backward_static_scratch(const float *x, const float *gy, const float *w1, const float *b1, const float *w2,
                                float *gx, float *dw1, float *db1, float *dw2, int64_t N, int64_t C, int64_t H,
                                int64_t W, int64_t K, int64_t hidden, uint32_t batch_per_nca, uint64_t seed,
                                float update_rate, int64_t image_offset, int accumulate, void *stream);

/* mask (n, h, w) = the {0, 1} update mask the kernels use for `seed` (Philox4x32-10; image index image_offset + i).
 * Replaces nca_cuda.update_mask (ncaops/nca_cuda.cu:325-331, bound at :351-352). */
int nca_update_mask(float *mask, int64_t n, int64_t h, int64_t w, uint64_t seed, float update_rate, int64_t image_offset,
                    void *stream);

/* Synthetic loss of the benchmark configurations, per NCA k:
 *   loss[k] = mean over (B, 3, H, W) of (x[k, :, :3] - target[k])^2 + overflow_weight * sum over (B, C, H, W) of
 *             |x - clamp(x, -1, 1)|,
 * and gy = d(sum_k loss[k]) / dx (N, C, H, W). target (K, 3, H, W); work: K * 128 floats of scratch.
 * Replaces the task loss the reference's training loop calls (train.py:67-72 / :97-99, Texture / Growing.loss);
 * deterministic (fixed-order reductions). */
int nca_synthetic_loss(const float *x, const float *target, float *gy, float *loss, float *work, int64_t K, int64_t B,
                       int64_t C, int64_t H, int64_t W, float overflow_weight, void *stream);

/* The same loss over the first target_channels channels (target: K x target_channels x H x W): per NCA the mean
 * squared error to the target plus overflow_weight x the summed overflow. target_channels = 4 with overflow_weight = 0
 * is the growing NCA's loss, L2 to a premultiplied RGBA target (train.py:97-99, Growing.loss); nca_synthetic_loss is
 * target_channels = 3. */
int nca_task_loss(const float *x, const float *target, float *gy, float *loss, float *work, int64_t K, int64_t B,
                  int64_t C, int64_t H, int64_t W, int64_t target_channels, float overflow_weight, void *stream);

/* Per-NCA, per-tensor gradient normalisation followed by Adam with a MultiStepLR schedule, for the three weight
 * tensors at once, in one launch (train.py:120-122 and :136-141: g /= ||g_k||_2 + 1e-8; torch.optim.Adam; lr x gamma
 * at each milestone). param_i / grad_i / m_i / v_i: K x numel_i fp32 (i = 0, 1, 2 for w1, b1, w2). iteration: device
 * int64, the 0-based iteration index (step = iteration + 1 for the bias corrections); the call increments it.
 * milestones: up to 8 iteration indices (host array), n_milestones of them. */
int nca_adam_step(float *param0, float *param1, float *param2, const float *grad0, const float *grad1, const float *grad2,
                  float *m0, float *m1, float *m2, float *v0, float *v1, float *v2, int64_t K, int64_t numel0,
                  int64_t numel1, int64_t numel2, int64_t *iteration, float lr, float beta1, float beta2, float eps,
                  float gamma, const int64_t *milestones, int n_milestones, void *stream);

/* The weight-gradient reduction of a rollout fused with nca_adam_step: one launch sums, per NCA and in a fixed order,
 * the partials that backward calls of this shape (NCA_STAGE_MAIN | NCA_STAGE_PARTIAL_ADD, 16-byte-aligned x, gy and
 * gx) accumulated in `partial`, stores the gradients into dw1 / db1 / dw2, and applies the per-NCA per-tensor
 * normalisation + Adam + MultiStepLR to w1 / b1 / w2 with moments m_i / v_i (then a one-thread launch increments
 * iteration). Bitwise equal to nca_backward_stages(NCA_STAGE_REDUCE, accumulate = 0) followed by nca_adam_step.
 * Replaces the gradient reduction of nca_cuda.backward plus train.py:136-141. */
int nca_reduce_adam_step(const float *partial, int64_t partial_floats, int64_t N, int64_t C, int64_t H, int64_t W,
                         int64_t K, int64_t hidden, uint32_t batch_per_nca, int fp32, int growing, float *dw1,
                         float *db1, float *dw2, float *w1, float *b1, float *w2, float *m0, float *m1, float *m2,
                         float *v0, float *v1, float *v2, int64_t *iteration, float lr, float beta1, float beta2,
                         float eps, float gamma, const int64_t *milestones, int n_milestones, void *stream);

/* Training-iteration glue on the device (train.py:126-142), for a loop captured once as a CUDA graph.
 * Control block ctl: 4 device uint64: [0] key (written by the caller once), [1] iterations started, [2] index of the
 * current iteration, [3] its rollout seed. nca_control_advance starts the next iteration: [2] = [1]++, [3] =
 * nca_step_seed([0], 2 [2]); the rollout's step t then uses nca_step_seed([3], t) (nca_*_dseed with seed_dev =
 * ctl + 3). */
int nca_control_advance(uint64_t *ctl, void *stream);

/* Batch of the current iteration from the pool: idx (K, B) int64 = B distinct entries of 0..P-1 per NCA (a partial
 * Fisher-Yates shuffle driven by nca_step_seed(ctl[0], 2 ctl[2] + 1), NCA k's draws indexed by nca_offset + k, the
 * global index a shard passes; train.py:128 draws them as rand(K, P).argsort(1)[:, :B]), x0 (K, B, C, H, W) =
 * pool (K, P, C, H, W) [k, idx[k, b]]; when inject_every > 0 and ctl[2] % inject_every == 0, x0[k, 0] is the seed
 * state instead (train.py:130-131): seed_kind 0 zeros (Texture.seed), 1 the growing seed, 1 in channels 3.. at
 * (H / 2, W / 2) (Growing.seed). 1 <= B <= 64, B <= P. */
int nca_pool_sample(const float *pool, float *x0, int64_t *idx, const uint64_t *ctl, int64_t K, int64_t P, int64_t B,
                    int64_t C, int64_t H, int64_t W, int64_t inject_every, int seed_kind, int64_t nca_offset,
                    void *stream);

/* pool[k, idx[k, b]] = x[k, b] (train.py:141). */
int nca_pool_store(float *pool, const float *x, const int64_t *idx, int64_t K, int64_t P, int64_t B, int64_t C,
                   int64_t H, int64_t W, void *stream);

/* Launch configuration the step kernels use for this shape on the current device, into info[0..11]: row-streaming
 * path (1), row kernels over column strips of 128 (2: W a multiple of 128 from 256 on) or tile path (0), forward
 * grid, forward threads per CTA, backward grid, backward threads per CTA, SM count,
 * tile-path forward CTAs per SM, tile-path backward grid, and the occupancy query, registers, dynamic shared memory
 * limit and carveout of the row-streaming forward kernel. Diagnostic; no reference counterpart. */
int nca_launch_info(int64_t C, int64_t hidden, int fp32, int growing, int64_t N, int64_t H, int64_t W, int64_t K,
                    int32_t *info);

/* Reads (and, reset = 1, clears) the device error word of the current device: 0, or 1 when a kernel gave up waiting
 * for its tensor-core work (a bounded wait ran out; the kernel returned instead of hanging). Synchronous. */
int nca_device_error(int *code, int reset);

/* Tensor-core layout self-test: D (128 x N) = A (128 x K) B (N x K)^T on tcgen05 (kind::tf32) with the operands
 * staged in one of the forms the step kernels use: form 0: A and B K-major without swizzle; 1: A in Tensor Memory,
 * B K-major; 2: A and B MN-major with the 128-byte / 32-byte-atom swizzle; 3: form 2 with the two descriptor strides
 * exchanged (a diagnostic that must NOT match). A, B, D row-major fp32 device memory (A, B rounded to TF32 inside);
 * N in 16..128 (multiple of 16), K in 8..128 (multiple of 8). No reference counterpart (the reference has no
 * tcgen05 path). */
int nca_umma_selftest(int form, int N, int K, const float *A, const float *B, float *D, void *stream);

/* Failure-detection self-test of the kernels' bounded waits: one CTA waits on an mbarrier that nothing arrives on,
 * one warp with a limit of limit_ns (in (0, 1 s]) and a second warp with the step kernels' 2 s limit; the second must
 * give up as soon as the first has (the shared abort word). The kernel then frees its Tensor Memory, sets the device
 * error word to 1 (as a step kernel whose wait ran out does) and returns: no trap, the context stays usable.
 * out (4 x u64, device memory): nanoseconds each warp waited and whether its wait reported success (0 expected).
 * No reference counterpart (the reference's kernels have no bounded waits). */
int nca_wait_selftest(int64_t limit_ns, unsigned long long *out, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* ULTRANCA_B200_H */
