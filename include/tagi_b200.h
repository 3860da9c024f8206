/*
 * tagi_b200.h — C ABI of libtagi_b200.so, the sm_100a implementation of the
 * TAGI moment hot path (fused mean/variance contractions, their elementwise
 * neighbours and the capped closed-form update).
 *
 * Conventions
 *   - Every entry point returns TAGI_OK (0) or a negative TAGI_E* status and
 *     never aborts; tagi_last_error() gives a message for the calling thread.
 *   - All tensors are float32 device pointers. Sizes and strides are int64
 *     element counts. `stream` is a cudaStream_t passed as void* (NULL = the
 *     legacy default stream). Work is enqueued asynchronously; nothing here
 *     synchronises the device.
 *   - Outputs are caller-allocated. Entry points that need scratch memory take
 *     (workspace, workspace_bytes) and have a *_workspace_size() query.
 *   - A "row-split" operand dimension maps an index i to the element offset
 *       (i / div) * outer + (i % div) * stride        (div <= 0: i * stride)
 *     which lets one GEMM view an NCHW tensor as an (N*H*W) x C matrix.
 *
 * Each declaration names the reference function it replaces
 * (paths relative to the triton-tagi project root).
 */
#ifndef TAGI_B200_H
#define TAGI_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    TAGI_OK = 0,
    TAGI_E_BAD_ARG = -1,      /* null pointer, negative size, inconsistent shape */
    TAGI_E_ALIGNMENT = -2,    /* pointer/stride alignment required by a fast path */
    TAGI_E_LAUNCH = -3,       /* CUDA launch or runtime error */
    TAGI_E_WORKSPACE = -4,    /* workspace missing or too small */
    TAGI_E_UNSUPPORTED = -5,  /* configuration outside what the kernels implement */
    TAGI_E_TIMEOUT = -6       /* a bounded device-side wait ran out */
};

/* Library identification and diagnostics. */
int tagi_version(void);                  /* (major << 16) | (minor << 8) | patch */
const char* tagi_last_error(void);       /* message of the last failing call (this thread) */
int tagi_device_arch(int device);        /* SM version of `device` (e.g. 100), <0 on error */
uint64_t tagi_kernel_launches(void);     /* kernels this library has launched (process-wide) */
uint64_t tagi_tc_launches(void);         /* of those, tcgen05 tensor-core contractions */
uint64_t tagi_tma_launches(void);        /* of those, weight sums fed by tensor-map copies */
/* Error word of the tensor-core kernels on the current device: 0, or the code of
 * the first bounded wait that ran out (the kernel then skipped its remaining work
 * and released its tensor memory). Synchronises the device; `reset` clears it. */
int tagi_device_status(int reset);
/* Limit, in nanoseconds, of the tensor-core kernels' waits that give up a tile
 * when they run out (default 2 s; 0 restores it), on the current device. A
 * diagnostic hook: values below 1000 (a test's) also make every tensor-core
 * launch give up its tiles at the start, as a wait that ran out would (error
 * word 2), so that the abort path runs: the other warps of both CTAs see the
 * pair's abort flag, stop, the kernel waits for its own copies and MMAs in
 * flight (those keep the fixed 2 s limit), frees its tensor memory and returns.
 * No reference counterpart (the reference's Triton kernels do not wait). */
int tagi_set_wait_limit_ns(uint64_t ns);

/* ---------------------------------------------------------------------------
 * Small all-reduces over NVLink peer memory (data-parallel SyncBN statistics)
 * ------------------------------------------------------------------------- */

/* Bytes of one rank's exchange buffer for `world` ranks (at most 32) and
 * vectors of at most max_elems doubles: 256 bytes of flags, then two parity
 * sets of world slots. */
size_t tagi_peer_buffer_bytes(int world, int64_t max_elems);
/* Allocates and zeroes one rank's exchange buffer on the current device and
 * writes its CUDA IPC handle (64 bytes) to ipc_handle; the other ranks open it
 * with tagi_peer_buffer_open. */
int tagi_peer_buffer_create(size_t bytes, void** ptr, void* ipc_handle);
int tagi_peer_buffer_open(const void* ipc_handle, void** ptr);
/* Frees an own buffer (own != 0) or unmaps a peer's. */
int tagi_peer_buffer_close(void* ptr, int own);
/* In place: data[0:n] <- the sum over ranks of every rank's data[0:n], added in
 * rank order (bit-identical on every rank). peer_bufs: device array of the
 * world buffer addresses as this rank sees them (its own at [rank]); counter:
 * a device uint64 (zero at the start) that the kernel advances, so the launch
 * may be replayed from a CUDA graph. Every rank must issue the same sequence
 * of calls on buffers created together. Replaces, for the SyncBN statistics,
 * the NCCL all-reduce of the host package (no reference counterpart: the
 * reference is single-GPU). A wait that runs out (2 s, a rank that stopped)
 * leaves data unreduced and sets the word read by tagi_peer_status. */
int tagi_peer_allreduce_f64(double* data, int64_t n, void* const* peer_bufs, int rank, int world,
                            int64_t max_elems, uint64_t* counter, void* stream);
/* 0, or 1 if a peer exchange wait ran out; synchronises; `reset` clears it. */
int tagi_peer_status(int reset);

/* ---------------------------------------------------------------------------
 * Dense moment contractions
 * ------------------------------------------------------------------------- */

/* Sz = ma^2 @ Sw + Sa @ (mw^2 + Sw) + Sb  (Sb: N floats).
 * Replaces triton_fused_var_forward, triton_tagi/kernels/common.py:170-210. */
int tagi_fused_var_forward(const float* ma, const float* Sa, const float* mw, const float* Sw,
                           const float* Sb, float* Sz, int64_t M, int64_t N, int64_t K,
                           int64_t stride_am, int64_t stride_ak, int64_t stride_wk,
                           int64_t stride_wn, int64_t stride_cm, int64_t stride_cn, void* stream);

/* mz = ma @ mw + mb and Sz = ma^2 @ Sw + Sa @ (mw^2 + Sw) + Sb in one pass.
 * Rows of ma/Sa and of mz/Sz are row-split views (see header comment);
 * mw/Sw are K x N with row stride ldw; mb/Sb hold N floats (may be NULL).
 * Replaces the mean matmul + variance kernel pair of Linear.forward
 * (triton_tagi/layers/linear.py:95-100) and Conv2D.forward
 * (triton_tagi/layers/conv2d.py:301-308, output written directly in NCHW). */
int tagi_moment_forward(const float* ma, const float* Sa, int64_t a_div, int64_t a_outer,
                        int64_t a_stride, int64_t a_kstride, const float* mw, const float* Sw,
                        int64_t ldw, const float* mb, const float* Sb, float* mz, float* Sz,
                        int64_t c_div, int64_t c_outer, int64_t c_stride, int64_t c_nstride,
                        int64_t M, int64_t N, int64_t K, void* stream);

/* d_ma = dmz @ mw^T, d_Sa = dSz @ (mw^2)^T.
 * Replaces triton_fused_backward_delta, triton_tagi/kernels/common.py:287-327. */
int tagi_fused_backward_delta(const float* dmz, const float* dSz, const float* mw, float* d_ma,
                              float* d_Sa, int64_t M, int64_t K, int64_t N, int64_t stride_dm,
                              int64_t stride_dn, int64_t stride_wk, int64_t stride_wn,
                              int64_t stride_cm, int64_t stride_ck, void* stream);

/* Same contraction with row-split views on dmz/dSz rows (so an NCHW delta can
 * be read in place) and on the output rows. Used by Conv2D.backward
 * (triton_tagi/layers/conv2d.py:338-357). */
int tagi_backward_delta_view(const float* dmz, const float* dSz, int64_t d_div, int64_t d_outer,
                             int64_t d_stride, int64_t d_nstride, const float* mw, int64_t ldw,
                             float* d_ma, float* d_Sa, int64_t c_div, int64_t c_outer,
                             int64_t c_stride, int64_t c_kstride, int64_t M, int64_t K,
                             int64_t N, void* stream);

/* Conv2D forward without a patch matrix: the contraction gathers the patches
 * of (ma, Sa) (N x C x H x W, NCHW) itself and writes mz, Sz (N x Co x Ho x Wo,
 * NCHW). mw, Sw: (C*k*k) x Co with rows (c, kh, kw); mb, Sb: Co.
 * Replaces Conv2D.forward's patch extraction and fused moment product,
 * triton_tagi/layers/conv2d.py:254-309 (padding_type 1: symmetric padding;
 * 2: `padding` on the right/bottom edge only). nhwc != 0: ma, Sa are given
 * channels-last (N x H x W x C, e.g. from tagi_nchw_to_nhwc), which lets the
 * contraction load a tap's channels 32 bytes at a time when C is a multiple
 * of 8; the outputs stay NCHW. */
int tagi_conv2d_forward(const float* ma, const float* Sa, const float* mw, const float* Sw,
                        const float* mb, const float* Sb, float* mz, float* Sz, int64_t N,
                        int64_t C, int64_t H, int64_t W, int64_t Co, int64_t k, int64_t stride,
                        int64_t padding, int64_t padding_type, int nhwc, void* workspace,
                        size_t workspace_bytes, void* stream);

/* Conv2D input deltas, written in NCHW (N x C x H x W). The reference forms the
 * patch-space deltas dP = dmz @ mw^T, dP_S = dSz @ (mw^2)^T (rows (n, oh, ow),
 * columns (c, kh, kw)) and folds them back with its col2im gather
 * (triton_tagi/layers/conv2d.py:338-357, _col2im_kernel 119-130). This entry sums
 * the same terms in one contraction over (tap, co): for input pixel (h, w) and
 * tap (kh, kw) it gathers the deltas at the output position the gather maps to,
 * times mw[c*k*k + tap][co]. col2im_mode 0 reproduces the reference's gather
 * (for stride > 1 it does not test the column offset for divisibility, with
 * truncating division); 1 is the exact adjoint of the patches. dmz, dSz:
 * N x Co x Ho x Wo (N x Ho x Wo x Co with nhwc != 0); mw: (C*k*k) x Co;
 * padding_type as tagi_conv2d_forward. */
int tagi_conv2d_backward_delta(const float* dmz, const float* dSz, const float* mw, float* d_ma,
                               float* d_Sa, int64_t N, int64_t C, int64_t H, int64_t W,
                               int64_t Co, int64_t k, int64_t stride, int64_t padding,
                               int64_t padding_type, int col2im_mode, int nhwc, void* workspace,
                               size_t workspace_bytes, void* stream);

/* Optional workspace of the entries above and below that write an M x N output
 * through a reduction of length K (tagi_linear_forward: M, N, K; its backward
 * delta: M, K, N; tagi_conv2d_forward: N*Ho*Wo, Co, C*k*k; tagi_conv2d_backward_delta:
 * N*H*W, C, Co*k*k). It holds (1) the partial sums of a split reduction, when the
 * output grid leaves SMs idle (added in split order), and (2) the weight-side
 * operand prepared once per call as tf32 hi/lo tiles, which the tensor-core kernel
 * copies with bulk asynchronous copies instead of forming them in every output
 * tile. With less workspace the prepared tiles are dropped first, then the split;
 * with none the contraction runs unsplit. Host only; 0 when neither applies. */
size_t tagi_store_workspace_size(int64_t M, int64_t N, int64_t K);

/* Linear forward: mz = ma @ mw + mb, Sz = ma^2 @ Sw + Sa @ (mw^2 + Sw) + Sb for
 * row-major ma, Sa (M x K), mw, Sw (K x N), mb, Sb (N); workspace as above.
 * Replaces Linear.forward, triton_tagi/layers/linear.py:92-104. */
int tagi_linear_forward(const float* ma, const float* Sa, const float* mw, const float* Sw,
                        const float* mb, const float* Sb, float* mz, float* Sz, int64_t M,
                        int64_t K, int64_t N, void* workspace, size_t workspace_bytes,
                        void* stream);

/* Linear input deltas: d_ma = dmz @ mw^T, d_Sa = dSz @ (mw^2)^T for row-major dmz,
 * dSz (M x N) and mw (K x N); workspace as above. Replaces the delta part of
 * Linear.backward, triton_tagi/layers/linear.py:118-136. */
int tagi_linear_backward_delta(const float* dmz, const float* dSz, const float* mw, float* d_ma,
                               float* d_Sa, int64_t M, int64_t K, int64_t N, void* workspace,
                               size_t workspace_bytes, void* stream);

/* grad_mw = a^T @ dmz, grad_Sw = (a^2)^T @ dSz  (K x N outputs).
 * Replaces triton_fused_weight_grad, triton_tagi/kernels/common.py:410-451. */
size_t tagi_fused_weight_grad_workspace_size(int64_t M, int64_t K, int64_t N);
int tagi_fused_weight_grad(const float* a, const float* dmz, const float* dSz, float* grad_mw,
                           float* grad_Sw, int64_t M, int64_t K, int64_t N, int64_t stride_am,
                           int64_t stride_ak, int64_t stride_dm, int64_t stride_dn,
                           int64_t stride_km, int64_t stride_kn, void* workspace,
                           size_t workspace_bytes, void* stream);

/* Same contraction and the same results as tagi_fused_weight_grad, for callers
 * that cannot allocate device memory: a host runtime that reaches this library
 * only through a C FFI and owns no CUDA allocator, or an application whose
 * device memory is a fixed pool that a plugin may not grow. Instead of a caller
 * workspace, the split-reduction partial sums go to one array of
 * TAGI_STATIC_SCRATCH_BYTES that lives in the library's device image: every
 * GPU that loads the library holds it until the process exits. When room is
 * left after the partials, the tensor-core kernel's prepared delta tiles go
 * there too (as they would into a large enough workspace). Shapes whose split
 * partials alone need more than the array return TAGI_E_WORKSPACE. The first call on a
 * device looks up that device's copy of the array (cudaGetSymbolAddress on
 * the current device), so make the first call before any stream capture.
 * All calls share the array: calls that overlap on the GPU (e.g. on two
 * streams at once) race. Nothing needs clearing between calls, because each
 * call writes every scratch element it reads. No counterpart in the
 * reference. */
#define TAGI_STATIC_SCRATCH_BYTES (16u << 20)
int tagi_fused_weight_grad_static(const float* a, const float* dmz, const float* dSz,
                                  float* grad_mw, float* grad_Sw, int64_t M, int64_t K, int64_t N,
                                  int64_t stride_am, int64_t stride_ak, int64_t stride_dm,
                                  int64_t stride_dn, int64_t stride_km, int64_t stride_kn,
                                  void* stream);

/* Parameter side of Linear/Conv2D backward + update over a batch of M rows.
 *   g_m[k,n] = sum_r a[r,k] dmz[r,n],   g_S[k,n] = sum_r a[r,k]^2 dSz[r,n]
 *   (row k == K, when has_bias, is the bias: a == 1)
 * a is M x K (row stride lda, contiguous columns); dmz/dSz rows are a
 * row-split view with column stride d_nstride.
 * mode TAGI_WGRAD_SUMS   : out_m/out_S <- raw sums, (K+has_bias) x N, row stride N
 * mode TAGI_WGRAD_DELTAS : out_m/out_S <- Sw*g_m, Sw^2*g_S (delta_mw/delta_Sw of
 *                          triton_tagi/layers/linear.py:138-151 and
 *                          conv2d.py:344-354); bias deltas to out_mb/out_Sb
 * mode TAGI_WGRAD_UPDATE : applies the capped update to mw,Sw (and mb,Sb) in
 *                          place, as update_parameters after backward
 *                          (triton_tagi/update/parameters.py:58-128). */
enum { TAGI_WGRAD_SUMS = 0, TAGI_WGRAD_DELTAS = 1, TAGI_WGRAD_UPDATE = 2 };
size_t tagi_param_grad_workspace_size(int64_t M, int64_t K, int64_t N, int has_bias);
int tagi_param_grad(const float* a, int64_t lda, const float* dmz, const float* dSz,
                    int64_t d_div, int64_t d_outer, int64_t d_stride, int64_t d_nstride,
                    int64_t M, int64_t K, int64_t N, int has_bias, int mode, float* mw,
                    float* Sw, float* mb, float* Sb, float* out_m, float* out_S, float* out_mb,
                    float* out_Sb, float cap_factor, void* workspace, size_t workspace_bytes,
                    void* stream);

/* tagi_param_grad with the activations given transposed: at is K x M (row
 * stride ldat, the M reduction elements of each row contiguous), e.g. the
 * transposed patches of tagi_im2col_t. Same modes, outputs and workspace. */
int tagi_param_grad_t(const float* at, int64_t ldat, const float* dmz, const float* dSz,
                      int64_t d_div, int64_t d_outer, int64_t d_stride, int64_t d_nstride,
                      int64_t M, int64_t K, int64_t N, int has_bias, int mode, float* mw,
                      float* Sw, float* mb, float* Sb, float* out_m, float* out_S, float* out_mb,
                      float* out_Sb, float cap_factor, void* workspace, size_t workspace_bytes,
                      void* stream);

/* tagi_param_grad (transposed = 0) or tagi_param_grad_t (transposed = 1) of a
 * layer with a bias whose two column sums are already known: bias_sums holds
 * 2*N float64 values, sum of dmz per column then sum of dSz (e.g. the
 * delta_sums of tagi_bn_backward for the convolution feeding that BatchNorm).
 * The bias row (row K) is taken from them (the same three modes), so the
 * contraction covers the K weight rows only. Replaces the bias part of
 * conv2d.py:344-354 (sum of the output deltas per channel). */
int tagi_param_grad_bias_given(const float* a, int64_t lda, int transposed, const float* dmz,
                               const float* dSz, int64_t d_div, int64_t d_outer,
                               int64_t d_stride, int64_t d_nstride, int64_t M, int64_t K,
                               int64_t N, const double* bias_sums, int mode, float* mw, float* Sw,
                               float* mb, float* Sb, float* out_m, float* out_S, float* out_mb,
                               float* out_Sb, float cap_factor, void* workspace,
                               size_t workspace_bytes, void* stream);

/* Apply all-reduced raw sums (layout of TAGI_WGRAD_SUMS) as the capped update:
 * m += cap(S*g_m), S += cap(S^2*g_S), floor 1e-5 (parameters.py:77-96). */
int tagi_apply_param_sums(const float* g_m, const float* g_S, int64_t K, int64_t N, int has_bias,
                          float* mw, float* Sw, float* mb, float* Sb, float cap_factor,
                          void* stream);

/* ---------------------------------------------------------------------------
 * Batched attention products (leading dims flattened to `batch`; each operand
 * has a batch stride and two matrix strides, so transpose views need no copy)
 * ------------------------------------------------------------------------- */

/* var[n,m,l] = scale_sq * sum_k var_a (mu_b^2 + var_b) + mu_a^2 var_b.
 * If mean != NULL also mean[n,m,l] = scale * sum_k mu_a mu_b (fused mean).
 * Replaces bmm_tagi_var, triton_tagi/kernels/attention.py:149-201. */
int tagi_bmm_tagi_var(const float* mu_a, const float* var_a, const float* mu_b,
                      const float* var_b, float* mean, float* var, int64_t batch, int64_t M,
                      int64_t L, int64_t K, int64_t sa_n, int64_t sa_m, int64_t sa_k,
                      int64_t sb_n, int64_t sb_k, int64_t sb_l, int64_t so_n, int64_t so_m,
                      int64_t so_l, float scale, float scale_sq, void* stream);

/* mean = scale * a_mean @ b, var = scale^2 * a_var @ b^2.
 * Replaces bmm_shared_right, triton_tagi/kernels/attention.py:286-336
 * (bmm_shared_left, attention.py:339-374, is the same call on transposed views). */
int tagi_bmm_shared_right(const float* a_mean, const float* a_var, const float* b, float* mean,
                          float* var, int64_t batch, int64_t M, int64_t L, int64_t K,
                          int64_t sa_n, int64_t sa_m, int64_t sa_k, int64_t sb_n, int64_t sb_k,
                          int64_t sb_l, int64_t so_n, int64_t so_m, int64_t so_l, float scale,
                          void* stream);

/* mean = scale * a @ b_mean, var = scale^2 * (a*a) @ b_var, batched like
 * tagi_bmm_shared_right, with the deterministic operand on the left (its
 * squares taken in the contraction). Replaces bmm_shared_left,
 * triton_tagi/kernels/attention.py:339-374, without its transpose identity:
 * the value deltas of attention, a = scores^T (a transposed view), run with
 * the score rows as the output rows (M = S) instead of the head dimension. */
int tagi_bmm_shared_left(const float* a, const float* b_mean, const float* b_var, float* mean,
                         float* var, int64_t batch, int64_t M, int64_t L, int64_t K, int64_t sa_n,
                         int64_t sa_m, int64_t sa_k, int64_t sb_n, int64_t sb_k, int64_t sb_l,
                         int64_t so_n, int64_t so_m, int64_t so_l, float scale, void* stream);

/* ---------------------------------------------------------------------------
 * Elementwise / row kernels
 * ------------------------------------------------------------------------- */

/* In-place capped update. Replaces update_parameters,
 * triton_tagi/update/parameters.py:104-128. */
int tagi_capped_update(float* m, float* S, const float* delta_m, const float* delta_S, int64_t n,
                       float cap_factor, void* stream);

/* delta_mu = (y - mu)/(var + sv2), delta_var = -1/(var + sv2).
 * Replaces the dense branch of compute_innovation,
 * triton_tagi/update/observation.py:119-163 (dense branch 149-161). */
int tagi_innovation(const float* y, const float* mu, const float* var, float* delta_mu,
                    float* delta_var, int64_t n, float sigma_v_sq, void* stream);

/* Rectified-Gaussian moments and Jacobian. Replaces bayesian_relu,
 * triton_tagi/layers/relu.py:94-122. */
int tagi_relu_forward(const float* mz, const float* Sz, float* ma, float* Sa, float* J, int64_t n,
                      void* stream);

/* out_m = dm * J, out_S = dS * J^2 (ReLU.backward relu.py:152-169,
 * Remax.backward remax.py:185-188). */
int tagi_jacobian_backward(const float* dm, const float* dS, const float* J, float* out_m,
                           float* out_S, int64_t n, void* stream);

/* Row-wise Remax over K classes. Replaces triton_remax,
 * triton_tagi/layers/remax.py:122-164. The same moments as the reference's
 * log-normal closed form, evaluated through exact rational forms without its
 * cancelling exp/log pairs (float32 with float64 row sums, hardware
 * approximations for exp, sqrt and divisions): within ~1e-5 relative of a
 * float64 evaluation of the reference's formulas. */
int tagi_remax_forward(const float* mz, const float* Sz, float* ma, float* Sa, float* J,
                       int64_t rows, int64_t K, int64_t row_stride, void* stream);

/* a_m += b_m, a_S += b_S. Replaces triton_add_shortcut / triton_delta_merge,
 * triton_tagi/layers/resblock.py:138-175. */
int tagi_add_inplace(float* a_m, float* a_S, const float* b_m, const float* b_S, int64_t n,
                     void* stream);

/* Average pooling with window = stride = k. Replaces the AvgPool2D kernels,
 * triton_tagi/layers/avgpool2d.py:158-239. */
int tagi_avgpool_forward(const float* ma, const float* Sa, float* ma_out, float* Sa_out,
                         int64_t N, int64_t C, int64_t H, int64_t W, int64_t k, float var_scale,
                         void* stream);
int tagi_avgpool_backward(const float* dm, const float* dS, float* dm_out, float* dS_out,
                          int64_t N, int64_t C, int64_t H, int64_t W, int64_t k, float var_scale,
                          void* stream);

/* Gaussian embedding lookup: token t (ids as floats, truncated toward zero as
 * the reference's ma.long()) gets rows (mw[id], Sw[id]) of the (V x D)
 * tables; ids outside [0, V) and padding_idx (-1: none) give zero rows.
 * Replaces Embedding.forward, triton_tagi/layers/embedding.py:88-110. */
int tagi_embedding_forward(const float* idx, const float* mw, const float* Sw, float* mz,
                           float* Sz, int64_t n_tokens, int64_t V, int64_t D,
                           int64_t padding_idx, void* stream);

/* Per-row parameter sums of the embedding over its tokens, in token order
 * (deterministic): mode TAGI_WGRAD_SUMS writes sum dmz, sum dSz (V x D, for an
 * all-reduce); TAGI_WGRAD_DELTAS writes sum dmz*Sw[id] and sum dSz*Sw[id]^2
 * (delta_mw, delta_Sw). Every row is written (zeros where no token maps to it);
 * padding and out-of-range ids contribute nothing.
 * Replaces Embedding.backward, triton_tagi/layers/embedding.py:112-151. */
int tagi_embedding_backward(const float* idx, const float* dmz, const float* dSz,
                            const float* Sw, int64_t n_tokens, int64_t V, int64_t D,
                            int64_t padding_idx, int mode, float* out_m, float* out_S,
                            void* stream);

/* out[r][d] = ma[r][d] + pe[r % S][d] for the rows of a (B*S, D) tensor (the
 * variances pass through unchanged). Replaces PositionalEncoding.forward,
 * triton_tagi/layers/positional_encoding.py:57-62. */
int tagi_positional_add(const float* ma, const float* pe, float* out, int64_t rows, int64_t S,
                        int64_t D, void* stream);

/* ---------------------------------------------------------------------------
 * Convolution helpers (NCHW; padding_type 2 = right/bottom only)
 * ------------------------------------------------------------------------- */

/* patches[(n,oh,ow), (c,kh,kw)] for mean and variance in one pass (xS and pS
 * both null: the mean patches only).
 * Replaces _triton_im2col, triton_tagi/layers/conv2d.py:140-152, 280-297. */
int tagi_im2col(const float* xm, const float* xS, float* pm, float* pS, int64_t N, int64_t C,
                int64_t H, int64_t W, int64_t k, int64_t stride, int64_t padding,
                int64_t padding_type, void* stream);

/* Transposed mean patches: pt is (C*k*k) x (N*Ho*Wo), row (c, kh, kw) holding
 * x[n][c][oh*stride - pad + kh][ow*stride - pad + kw] (0 outside) at column
 * (n, oh, ow); padding_type as tagi_im2col. For tagi_param_grad_t. */
int tagi_im2col_t(const float* x, float* pt, int64_t N, int64_t C, int64_t H, int64_t W,
                  int64_t k, int64_t stride, int64_t padding, int64_t padding_type, void* stream);

/* NCHW -> NHWC copy of a tensor pair (yS, xS may both be NULL): y[n][p][c] =
 * x[n][c][p] for p < HW, for the channels-last gathers of the Conv2D entries. */
int tagi_nchw_to_nhwc(const float* xm, const float* xS, float* ym, float* yS, int64_t N,
                      int64_t C, int64_t HW, void* stream);

/* Gather patch-space deltas back to NCHW. mode 0 reproduces the reference's
 * gather exactly (_col2im_kernel, conv2d.py:85-132, 155-181, 361-370);
 * mode 1 is the true adjoint of im2col. */
int tagi_col2im(const float* cm, const float* cS, float* dm, float* dS, int64_t N, int64_t C,
                int64_t H, int64_t W, int64_t k, int64_t stride, int64_t padding,
                int64_t padding_type, int mode, void* stream);

/* ---------------------------------------------------------------------------
 * Normalisation
 * ------------------------------------------------------------------------- */

/* Per-channel raw sums over (N, H*W) of an NCHW tensor pair:
 * sums[0:C] = sum mz, sums[C:2C] = sum Sz, sums[2C:3C] = sum mz^2 (float64).
 * Replaces the three _channel_mean_kernel launches of
 * triton_tagi/layers/batchnorm2d.py:307-339 (one pass, no mz*mz temporary). */
int tagi_bn_channel_sums(const float* mz, const float* Sz, double* sums, int64_t N, int64_t C,
                         int64_t HW, void* stream);

/* From (possibly all-reduced) sums over `count` = N_global*H*W elements:
 * mean, Bessel-corrected var; running-stat init (first != 0, with optional
 * mw = sqrt(var + eps) when preserve_var) or EMA with `momentum`
 * (batchnorm2d.py:336-355). */
int tagi_bn_finalize(const double* sums, int64_t C, double count, float* mean, float* var,
                     float* running_mean, float* running_var, float* mw, int first,
                     int preserve_var, float momentum, float eps, void* stream);

/* Normalise + Gaussian affine; caches m_hat (S_hat if non-NULL).
 * Replaces _batchnorm_fwd_kernel, batchnorm2d.py:59-126, 388-431. */
int tagi_bn_forward(const float* mz, const float* Sz, const float* mean, const float* var,
                    const float* mg, const float* Sg, const float* mb, const float* Sb, float* ma,
                    float* Sa, float* m_hat, float* S_hat, int64_t N, int64_t C, int64_t HW,
                    float eps, void* stream);

/* Training-mode forward of one process in one launch: the channel sums, the
 * finalisation (mean, Bessel-corrected variance, running statistics and the
 * first-call scale, as tagi_bn_finalize with count = N*H*W) and the normalised
 * affine (as tagi_bn_forward with m_hat cached), each channel on one thread-
 * block cluster. mean, var receive the statistics. add_m, add_S (both or
 * neither; same layout as ma, Sa): a residual stream added to the outputs, as
 * tagi_add_inplace after this layer would (the ResBlock shortcut,
 * triton_tagi/layers/resblock.py:138-154). Data-parallel SyncBN, which
 * all-reduces the sums between the passes, uses the three entries above. */
int tagi_bn_train_forward(const float* mz, const float* Sz, float* mean, float* var,
                          float* running_mean, float* running_var, float* mg, const float* Sg,
                          const float* mb, const float* Sb, float* ma, float* Sa, float* m_hat,
                          const float* add_m, const float* add_S, int64_t N, int64_t C,
                          int64_t HW, int first, int preserve_var, float momentum, float eps,
                          void* stream);

/* Data-parallel training forward after the statistics exchange: from the
 * all-reduced channel sums (tagi_bn_channel_sums layout, `count` elements over
 * all ranks) every channel is finalised as tagi_bn_finalize does and
 * normalised as tagi_bn_train_forward does (residual stream add_m, add_S
 * optional), in one launch. Replaces, for SyncBN, batchnorm2d.py:336-355 and
 * 388-431 together with the shortcut add of resblock.py:138-154. */
int tagi_bn_sync_forward(const float* mz, const float* Sz, const double* sums, double count,
                         float* mean, float* var, float* running_mean, float* running_var,
                         float* mg, const float* Sg, const float* mb, const float* Sb, float* ma,
                         float* Sa, float* m_hat, const float* add_m, const float* add_S,
                         int64_t N, int64_t C, int64_t HW, int first, int preserve_var,
                         float momentum, float eps, void* stream);

/* Delta propagation plus per-channel raw sums (float64)
 * grads[0:C]=sum dma*m_hat, [C:2C]=sum dSa*m_hat^2, [2C:3C]=sum dma, [3C:4C]=sum dSa.
 * relu_J (NULL: none): Jacobian of a ReLU that produced this layer's input;
 * the outgoing deltas are then multiplied by J and J^2 as the ReLU's backward
 * (triton_tagi/layers/relu.py:152-169) would. cap_factor > 0: the capped update
 * of gamma (mg, Sw) and beta (mb, Sb) is also applied from the sums, as
 * tagi_bn_apply_grads in update mode would (mg is updated in place after every
 * block has read it); cap_factor <= 0 leaves the parameters alone.
 * delta_sums (NULL: not computed; else 2*C float64): [0:C] = sum of the
 * outgoing dmz, [C:2C] = sum of the outgoing dSz per channel, i.e. the bias
 * sums of the convolution that produced this layer's input (through the ReLU
 * given by relu_J, if any), for tagi_param_grad_bias_given.
 * Replaces batchnorm2d.py:436-513 (torch sums + _batchnorm_bwd_kernel). */
int tagi_bn_backward(const float* dma, const float* dSa, const float* m_hat, const float* var,
                     float* mg, float* dmz, float* dSz, const float* relu_J, double* grads,
                     double* delta_sums, int64_t N, int64_t C, int64_t HW, float eps, float* Sw,
                     float* mb, float* Sb, float cap_factor, void* stream);

/* Apply per-channel sums (tagi_bn_backward layout, possibly all-reduced):
 * mode TAGI_WGRAD_DELTAS writes the four delta vectors, TAGI_WGRAD_UPDATE
 * applies the capped update to (mw,Sw,mb,Sb) in place. */
int tagi_bn_apply_grads(const double* grads, int64_t C, int mode, float* mw, float* Sw, float* mb,
                        float* Sb, float* d_mw, float* d_Sw, float* d_mb, float* d_Sb,
                        float cap_factor, void* stream);

/* RMSNorm over the last dim (rows x ni). Replaces RMSNorm.forward/backward,
 * triton_tagi/layers/rms_norm.py:93-137. Backward writes propagated deltas
 * and the raw gamma sums (float64) sum_mu[ni], sum_var[ni]. */
int tagi_rmsnorm_forward(const float* ma, const float* Sa, const float* mw, const float* Sw,
                         float* mz, float* Sz, float* inv_rms, int64_t rows, int64_t ni,
                         float eps, void* stream);
int tagi_rmsnorm_backward(const float* dmz, const float* dSz, const float* ma,
                          const float* inv_rms, const float* mw, float* dma, float* dSa,
                          double* sums, int64_t rows, int64_t ni, void* stream);

/* Capped update from float64 raw sums with a per-element prior scale:
 * m += cap(S*g_m), S += cap(S^2*g_S). Used for RMSNorm gamma and any vector
 * parameter whose sums were reduced in float64 (and all-reduced). */
int tagi_apply_vector_sums(const double* g_m, const double* g_S, int64_t n, int mode, float* m,
                           float* S, float* d_m, float* d_S, float cap_factor, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TAGI_B200_H */
