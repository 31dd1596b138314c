/*
 * rapidalign_b200.h -- C ABI of the B200 (sm_100a) KDE/MMD library.
 *
 * Gaussian-kernel MMD sums between point clouds,
 *     k(u, v) = exp(-|u - v|^2 / (2 sigma^2)),
 *     Kxx = sum_ij a_i a_j k(x_i, x_j),  Kyy = sum_ij b_i b_j k(y_i, y_j),
 *     Kxy = sum_ij a_i b_j k(x_i, y_j),
 * for single pairs, ragged (ptr-segmented) batches and padded dense batches,
 * with their gradients.
 *
 * Conventions for every entry point:
 *  - all array arguments are DEVICE pointers to contiguous row-major data on
 *    the current CUDA device, except where a comment says "host";
 *  - work is enqueued on `stream` and is asynchronous; nothing synchronises
 *    the host;
 *  - the library never allocates device memory: scratch space is a caller
 *    owned `workspace` of at least the size the matching *_workspace_bytes
 *    function returns (256-byte aligned).  The one exception is
 *    ra_kde_mmd_forward_segmented_noalloc, whose scratch is a fixed array
 *    inside the library (see its comment);
 *  - the return value is an ra_status code; ra_status_string() names it.
 *    Argument errors are reported synchronously.  Data-dependent errors
 *    (bad ptr offsets, non-positive weight sums) are detected on the device
 *    and reported by ra_kde_check(), which reads one int back and therefore
 *    synchronises `stream`;
 *  - calls on different streams with different workspaces are independent.
 *    The library's only global mutable state is the no-alloc entry point's
 *    scratch array (shared by its calls, see there) and a process-wide
 *    launch counter (ra_kernel_launch_count, diagnostics only).
 */
#ifndef RAPIDALIGN_B200_H
#define RAPIDALIGN_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define RA_API __attribute__((visibility("default")))
#else
#define RA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *ra_stream_t; /* == cudaStream_t */

/* ---- status codes ------------------------------------------------------ */
enum ra_status {
  RA_OK = 0,
  RA_ERR_INVALID_ARGUMENT = 1,    /* null pointer, bad size, unsupported dim */
  RA_ERR_SIGMA = 2,               /* sigma must be positive */
  RA_ERR_WORKSPACE = 3,           /* workspace too small or misaligned */
  RA_ERR_CUDA = 4,                /* a CUDA runtime call or launch failed */
  /* device-detected data errors (returned by ra_kde_check) */
  RA_ERR_PTR_START = 16,          /* ptr must start at 0 */
  RA_ERR_PTR_END = 17,            /* ptr[-1] must equal number of nodes */
  RA_ERR_PTR_ORDER = 18,          /* ptr offsets must be non-decreasing */
  RA_ERR_WEIGHT_SUM = 19,         /* weights must sum to a positive value per segment */
  RA_ERR_STATE = 20,              /* backward called without a matching forward state */
  RA_ERR_SCRATCH_LIMIT = 21,      /* problem needs more than the fixed no-alloc scratch */
  RA_ERR_DEVICE_TIMEOUT = 22,     /* a bounded wait inside a kernel expired (reported, not hung) */
  /* RA_ERR_SIGMA is also returned by ra_kde_check for a per-pair sigma <= 0 */
};

/* Human-readable name of a status code (static string). */
RA_API const char *ra_status_string(int status);

/* ---- the general problem description (fused forward / backward) -------- */

enum ra_layout {
  RA_LAYOUT_RAGGED = 0, /* points of pair p are rows ptr[p]..ptr[p+1] */
  RA_LAYOUT_DENSE = 1   /* pair p = row p of a (B, Nmax, D) tensor plus a (B, Nmax) mask */
};

enum ra_weights {
  RA_WEIGHTS_RAW = 0,         /* a_i = w_i as given (w == NULL: 1); mask applied if dense */
  RA_WEIGHTS_SUM = 1,         /* a_i = w_i / sum_seg w; error if a segment sum <= 0
                                 (rapidalign/kde.py:20-27, 169-199) */
  RA_WEIGHTS_SUM_CLAMPED = 2, /* a_i = w_i m_i / max(sum_seg w m, 1e-8)  (kde.py:115-121);
                                 w == NULL means w = 1 */
  RA_WEIGHTS_UNIFORM = 3      /* a_i = 1 / count_seg; w ignored (kde.py:183-188) */
};

/* Kernel family for the generic (dim >= 4) layout. */
enum ra_engine {
  RA_ENGINE_AUTO = 0,
  RA_ENGINE_SIMT = 1,   /* one thread per row, columns staged in shared memory */
  RA_ENGINE_TENSOR = 2  /* tcgen05 (3xTF32) Gram and weighted-sum GEMMs */
};

typedef struct ra_kde_desc {
  int64_t num_pairs;   /* P (ragged) or B (dense) */
  int32_t dim;         /* D >= 1 */
  int32_t layout;      /* enum ra_layout */
  int64_t num_x;       /* ragged: rows of x; dense: B * nmax_x */
  int64_t num_y;       /* ragged: rows of y; dense: B * nmax_y */
  int64_t nmax_x;      /* dense only: padded length of a row of x */
  int64_t nmax_y;      /* dense only */
  int32_t weights_x;   /* enum ra_weights */
  int32_t weights_y;
  int32_t center;      /* 1: subtract the weighted centroid of each cloud first */
  int32_t need_grad;   /* 1: keep per-point state in the workspace for ra_kde_backward */
  int32_t need_sigma_grad; /* 1: also accumulate the sigma derivative */
  int32_t shard_index; /* splitting one problem over shard_count processes (GPUs): */
  int32_t shard_count; /* this process evaluates work items shard_index, shard_index +
                          shard_count, ...; 0 or 1 = no split (see ra_kde_forward) */
  double sigma;        /* bandwidth, > 0 */
  int32_t engine;      /* kernel family for dim >= 4 (enum ra_engine): RA_ENGINE_AUTO =
                          tensor cores when the padded dim is 32, 64 or 128, else SIMT;
                          RA_ENGINE_TENSOR on another padded dim is
                          RA_ERR_INVALID_ARGUMENT.  Ignored for dim <= 3. */
  int32_t skip_weight_sums; /* 1: no weight gradient will be asked for, so the forward may
                          leave out per-point sums that only grad_wx / grad_wy need
                          (dim <= 3: one FP32 operation per kernel term); a backward
                          that asks for them is then RA_ERR_STATE.  0: keep them. */
  int32_t deterministic; /* 1: gradients bitwise independent of scheduling.  dim <= 3
                          then evaluates every kernel term in both orientations with
                          plain stores instead of adding column sums atomically (about
                          1.5x the FP32 work).  dim >= 4 is deterministic either way;
                          K and the losses always are. */
  int32_t test_hooks;  /* 0 in normal use.  Bits of enum ra_test_hook, for tests of the
                          library's own failure paths only. */
} ra_kde_desc;

/* Test hooks (ra_kde_desc.test_hooks).  RA_TEST_NO_MMA: the tensor-core kernels
 * (dim >= 4 on the tensor-core engine) issue no MMA at all and bound each wait
 * to 4096 polls, so their first wait for a GEMM expires with nothing in flight:
 * the kernel records the timeout, frees its tensor memory and returns, and
 * ra_kde_check reports RA_ERR_DEVICE_TIMEOUT.  RA_TEST_RING_IDLE: the O(N)
 * passes that stream rows by bulk copies (padded dim 32-128, equal weights, no
 * mask) copy nothing and bound each wait to 4096 polls, so their consumers'
 * first wait expires: the same status, from the forward (sums and packing)
 * or the backward (write pass).  The results of such a call are invalid. */
enum ra_test_hook { RA_TEST_NO_MMA = 1, RA_TEST_RING_IDLE = 2 };

typedef struct ra_kde_inputs {
  const float *x;        /* [num_x * D] */
  const float *y;        /* [num_y * D] */
  const float *w_x;      /* [num_x] or NULL */
  const float *w_y;      /* [num_y] or NULL */
  const int64_t *ptr_x;  /* ragged: [P + 1] */
  const int64_t *ptr_y;  /* ragged: [P + 1] */
  const uint8_t *mask_x; /* dense: [num_x] (nonzero = valid) */
  const uint8_t *mask_y; /* dense: [num_y] */
  const double *sigma_pairs; /* [P] per-pair bandwidths (all > 0), or NULL: desc->sigma
                                for every pair.  Several bandwidths of one pair of clouds
                                in one call = the clouds repeated as P pairs. */
} ra_kde_inputs;

typedef struct ra_kde_grads {
  float *grad_x;      /* [num_x * D] or NULL */
  float *grad_y;      /* [num_y * D] or NULL */
  double *grad_wx;    /* [num_x] or NULL: d/dw of the given weights (incl. normalisation) */
  double *grad_wy;    /* [num_y] or NULL */
  double *grad_sigma; /* [P] per-pair d/dsigma or NULL (needs need_sigma_grad) */
} ra_kde_grads;

/* Workspace bytes for ra_kde_forward (+ ra_kde_backward) on `desc`. */
RA_API size_t ra_kde_workspace_bytes(const ra_kde_desc *desc);

/*
 * Fused forward.  Replaces the three forward launches of
 * csrc/kde_similarity.cu:84-192 / :283-381 and the normalisation and
 * centering of rapidalign/kde.py:115-121, 169-208, 241-253.  Writes
 * K[0..P) = Kxx, K[P..2P) = Kyy, K[2P..3P) = Kxy (fp64) and, if
 * desc->need_grad, leaves in `workspace` what ra_kde_backward needs.
 */
RA_API int ra_kde_forward(const ra_kde_desc *desc, const ra_kde_inputs *in, double *K,
                   void *workspace, size_t workspace_bytes, ra_stream_t stream);

/*
 * ra_kde_forward in two phases on the same stream, for callers that read the
 * device error word (ra_kde_status_of_error_word) without stopping the GPU:
 * ra_kde_forward_prepare enqueues everything before the tile kernels
 * (segments and ptr checks, weight sums, centroids, work plan, packing), after
 * which the workspace's error word holds every data error the inputs have;
 * ra_kde_forward_compute enqueues the tile kernels and forms K, exactly as
 * ra_kde_forward would.  A caller can copy the word to host memory between the
 * two and wait for that copy while the tile kernels run.  (The tensor-core
 * kernels can still set RA_ERR_DEVICE_TIMEOUT during the compute phase.)
 */
RA_API int ra_kde_forward_prepare(const ra_kde_desc *desc, const ra_kde_inputs *in,
                                  void *workspace, size_t workspace_bytes, ra_stream_t stream);
RA_API int ra_kde_forward_compute(const ra_kde_desc *desc, const ra_kde_inputs *in, double *K,
                                  void *workspace, size_t workspace_bytes, ra_stream_t stream);

/*
 * Backward of the fused forward: given coef[0..P) = dL/dKxx, coef[P..2P) =
 * dL/dKyy, coef[2P..3P) = dL/dKxy (fp64, device), writes the requested
 * gradients including the centering and weight-normalisation Jacobians.
 * Replaces csrc/kde_similarity.cu:607-712 (and generalises it from the MMD
 * coefficients (1, 1, -2) to any).  Must follow ra_kde_forward with the same
 * desc, inputs and workspace and desc->need_grad = 1.
 */
RA_API int ra_kde_backward(const ra_kde_desc *desc, const ra_kde_inputs *in, const double *coef,
                    const ra_kde_grads *grads, void *workspace, size_t workspace_bytes,
                    ra_stream_t stream);

/*
 * Split evaluation of one problem over several GPUs (e.g. a single very large
 * pair).  With desc->shard_count > 1, ra_kde_forward evaluates only this
 * shard's work items and stops before forming K: every process then sums the
 * two partial buffers reported by ra_kde_partials over the group (an
 * all-reduce of fp64 and fp32 data, in place), and calls
 * ra_kde_forward_finish to form K (and the backward state).  Inputs must be
 * identical on all shards.  No counterpart in the reference (its kernels put a
 * whole pair on one thread block, csrc/kde_similarity.cu:196-279).
 */
RA_API int ra_kde_partials(const ra_kde_desc *desc, void *workspace, size_t workspace_bytes,
                           double **f64_buf, size_t *f64_count, float **f32_buf,
                           size_t *f32_count);
RA_API int ra_kde_forward_finish(const ra_kde_desc *desc, double *K, void *workspace,
                                 size_t workspace_bytes, ra_stream_t stream);

/*
 * ra_kde_forward with timing of the hot tile kernel: records two CUDA events
 * on `stream` around that single launch, synchronises on the second and
 * writes the elapsed milliseconds to *tiles_ms.  For measurement only.
 */
RA_API int ra_kde_forward_profiled(const ra_kde_desc *desc, const ra_kde_inputs *in, double *K,
                                   void *workspace, size_t workspace_bytes, ra_stream_t stream,
                                   float *tiles_ms);

/* Reads the device error word of `workspace` (synchronises `stream`). */
RA_API int ra_kde_check(const void *workspace, ra_stream_t stream);

/* The status a device error word stands for (RA_OK for 0): for callers that
 * copy the word themselves (the first 4 bytes of the workspace, an int) to
 * read it without synchronising the stream. */
RA_API int ra_kde_status_of_error_word(int word);

/* Enqueues on `stream` the copy of the workspace's error word into host[0]
 * and, when nflags > 0, of the int32 flags[0..nflags) (ra_ptr_from_batch)
 * into host[1..nflags]; `host` should be page-locked for the copies to stay
 * asynchronous.  For a status read on a side stream that waits for the
 * preparation (an event) while the tile kernels run.  Replaces the
 * reference's host reads behind its ptr, batch and weight checks
 * (rapidalign/kde.py:136-151, 198: .item() calls that stop the stream). */
RA_API int ra_kde_error_word_async(const void *workspace, const int32_t *flags, int32_t nflags,
                                   int32_t *host, ra_stream_t stream);

/* ---- the loss and the outputs in one launch -----------------------------
 * From the P-pair sums K = (Kxx | Kyy | Kxy) (float64 [3P]) write the
 * per-pair loss and the three sums in the caller's dtype: out_f64 = 1 for
 * float64 outputs, 0 for float32.  The loss is Kxx + Kyy - 2 Kxy, or with
 * cosine = 1, 1 - Kxy / sqrt(max(Kxx Kyy, eps)) (rapidalign/kde.py:103-107,
 * 265-268, 368-371), evaluated in float64 in the order the reference
 * writes it.  Replaces the reference's tensor expressions after
 * _cuda.kde_mmd_forward* (kde.py:265-274, 368-377). */
RA_API int ra_mmd_outputs(const double *K, int64_t P, int cosine, double eps, int out_f64,
                          void *loss, void *Kxx, void *Kyy, void *Kxy, ra_stream_t stream);
/* Its derivative: coef (float64 [3P]) = dL/dK from the gradients of the four
 * outputs (each nullable = zero; float32 or float64 as out_f64 says), for
 * ra_kde_backward. */
RA_API int ra_mmd_outputs_backward(const double *K, int64_t P, int cosine, double eps,
                                   int out_f64, const void *g_loss, const void *g_Kxx,
                                   const void *g_Kyy, const void *g_Kxy, double *coef,
                                   ra_stream_t stream);

/* ---- legacy operator set: one entry point per op of csrc/bindings.cpp ---- */

/*
 * Dense masked forward.  Replaces kde_mmd_forward (csrc/bindings.cpp:35-45,
 * csrc/kde_similarity.cu:84-192): x [B, Nx, D], y [B, Ny, D], w_x [B, Nx],
 * w_y [B, Ny] (raw weights), mask_x [B, Nx], mask_y [B, Ny] (uint8),
 * outputs Kxx, Kyy, Kxy [B] fp64.
 */
RA_API size_t ra_kde_mmd_forward_workspace_bytes(int64_t B, int64_t Nx, int64_t Ny, int32_t D);
RA_API int ra_kde_mmd_forward(const float *x, const float *y, const float *w_x, const float *w_y,
                       const uint8_t *mask_x, const uint8_t *mask_y, int64_t B, int64_t Nx,
                       int64_t Ny, int32_t D, double sigma, double *Kxx, double *Kyy,
                       double *Kxy, void *workspace, size_t workspace_bytes, ra_stream_t stream);

/*
 * Ragged forward.  Replaces kde_mmd_forward_segmented (csrc/bindings.cpp:47-57,
 * csrc/kde_similarity.cu:283-381): x [NX, D], y [NY, D], raw weights w_x [NX],
 * w_y [NY], ptr_x/ptr_y int64 [P + 1]; outputs Kxx, Kyy, Kxy [P] fp64.
 */
RA_API size_t ra_kde_mmd_forward_segmented_workspace_bytes(int64_t P, int64_t NX, int64_t NY,
                                                    int32_t D);
RA_API int ra_kde_mmd_forward_segmented(const float *x, const float *y, const float *w_x,
                                 const float *w_y, const int64_t *ptr_x, const int64_t *ptr_y,
                                 int64_t P, int64_t NX, int64_t NY, int32_t D, double sigma,
                                 double *Kxx, double *Kyy, double *Kxy, void *workspace,
                                 size_t workspace_bytes, ra_stream_t stream);

/*
 * Ragged backward.  Replaces kde_mmd_backward_segmented (csrc/bindings.cpp:59-70,
 * csrc/kde_similarity.cu:607-712): gradients of sum_p grad_loss[p] *
 * (Kxx + Kyy - 2 Kxy)[p] w.r.t. x (f32 [NX, D]), y (f32 [NY, D]), the raw
 * weights (f64 [NX], [NY]) and sigma (f64 [P], per pair).  Valid for any D
 * (the reference kernels are limited to D <= 3).
 */
RA_API size_t ra_kde_mmd_backward_segmented_workspace_bytes(int64_t P, int64_t NX, int64_t NY,
                                                     int32_t D);
RA_API int ra_kde_mmd_backward_segmented(const float *x, const float *y, const float *w_x,
                                  const float *w_y, const int64_t *ptr_x, const int64_t *ptr_y,
                                  int64_t P, int64_t NX, int64_t NY, int32_t D,
                                  const double *grad_loss, double sigma, float *grad_x,
                                  float *grad_y, double *grad_wx, double *grad_wy,
                                  double *grad_sigma_pairs, void *workspace,
                                  size_t workspace_bytes, ra_stream_t stream);

/*
 * Ragged forward that allocates nothing.  No counterpart in the reference.
 *
 * Same arguments and results as ra_kde_mmd_forward_segmented, minus the
 * workspace: the scratch comes from a fixed 64 MiB array that the library
 * keeps in device memory (every GPU that loads the library holds it until the
 * process exits).  Meant for callers that cannot call cudaMalloc: hosts whose
 * plugin contract leaves all device memory to their own pool and hand a
 * library nothing but input and output buffers, and loops that must not
 * allocate (or synchronise the device, as an allocation may) once running.
 *
 * Limits and rules:
 *  - problems whose workspace (ra_kde_mmd_forward_segmented_workspace_bytes)
 *    exceeds 64 MiB are rejected with RA_ERR_SCRATCH_LIMIT before any work
 *    is enqueued;
 *  - the first call on a device looks up that device's address of the
 *    scratch array (with the device current); make that first call before
 *    any stream capture;
 *  - all calls on a device share the one array and it keeps the previous
 *    call's contents; the call clears what must start at zero, but calls
 *    whose GPU work overlaps (other streams, other host threads) race on it:
 *    serialise them;
 *  - every call looks the array's device address up again (which allocates
 *    nothing), so a device reset between calls does not leave a stale
 *    address behind;
 *  - data errors found on the device (bad ptr offsets, a non-positive weight
 *    sum, a tensor-core wait that expired) are read back by
 *    ra_kde_check_noalloc, as ra_kde_check does for a caller's workspace.
 */
RA_API int ra_kde_mmd_forward_segmented_noalloc(const float *x, const float *y,
                                                const float *w_x, const float *w_y,
                                                const int64_t *ptr_x, const int64_t *ptr_y,
                                                int64_t P, int64_t NX, int64_t NY, int32_t D,
                                                double sigma, double *Kxx, double *Kyy,
                                                double *Kxy, ra_stream_t stream);

/* The device error word of the no-alloc scratch on the current device, as a
 * status (the same codes as ra_kde_check; synchronises `stream`).  Reports on
 * the last ra_kde_mmd_forward_segmented_noalloc enqueued on this device. */
RA_API int ra_kde_check_noalloc(ra_stream_t stream);

/* ---- batch vectors ----------------------------------------------------- */

/* ptr offsets of a sorted batch vector, on the device: replaces the ptr
 * construction of rapidalign/kde.py:142-156 (there: sort check, bincount,
 * cumsum and host reads).  batch [n] int64 (device), num_graphs = the number
 * of graphs the caller expects (batch[n - 1] + 1); writes ptr [num_graphs + 1]
 * (device) and *flags (a device int, zeroed first) with bits of enum
 * ra_batch_flag.  Nothing is read back: the caller checks the flags when it
 * reads them.  ptr is exact when flags == 0. */
enum ra_batch_flag {
  RA_BATCH_UNSORTED = 1, /* "batch indices must be sorted for contiguous blocks" */
  RA_BATCH_NEGATIVE = 2, /* the first graph id is negative */
  RA_BATCH_COUNT = 4     /* batch[n - 1] + 1 != num_graphs */
};
RA_API int ra_ptr_from_batch(const int64_t *batch, int64_t n, int64_t num_graphs, int64_t *ptr,
                             int *flags, ra_stream_t stream);

/* ---- diagnostics ------------------------------------------------------- */

/* Number of kernel launches this library has issued in the calling process
 * (a process-wide counter; used to report launch counts in benchmarks). */
RA_API unsigned long long ra_kernel_launch_count(void);

/* Times a pure packed-FP32-FMA kernel on the current device (one warm-up
 * launch, then one timed launch of `iters` inner iterations) and returns the
 * FP32 lane-operation rate (an FMA counts one) in *ops_per_s.  `scratch` is a
 * device buffer of at least (multiprocessors * 8 * 256) floats.  Synchronises
 * `stream`.  Used as the measured FP32 roofline peak. */
RA_API int ra_probe_fp32_peak(float *scratch, int64_t scratch_floats, int iters, double *ops_per_s,
                       ra_stream_t stream);

/* ---- float64 verification path --------------------------------------- */
/* Replaces rapidalign/kde_gradients.py:39-193 (kde_mmd_forward_cpu,
 * kde_mmd_backward_cpu, kde_mmd_backward_ragged_cpu): closed-form sums and
 * gradients of the raw-weight loss L = Kxx + Kyy - 2 Kxy per pair, every
 * term in double precision (exp, direct differences), for verification on
 * small problems (O(N^2 D) per pair, one thread per point).
 *
 * x [NX, D], y [NY, D], w_x [NX], w_y [NY], ptr_x / ptr_y [P + 1]: device
 * arrays.  Outputs (device, caller-allocated): Kxx, Kyy, Kxy [P] (required);
 * loss [P], grad_x [NX, D], grad_y [NY, D], grad_wx [NX], grad_wy [NY],
 * grad_sigma [P] (each may be NULL).  The workspace (256-byte aligned) holds
 * at least ra_kde_exact_workspace_bytes(NX, NY).  The call synchronises
 * `stream` once to read the ptr checks (RA_ERR_PTR_*), which must pass
 * before any segment is walked. */
RA_API size_t ra_kde_exact_workspace_bytes(int64_t NX, int64_t NY);
RA_API int ra_kde_exact_f64(const double *x, const double *y, const double *w_x,
                            const double *w_y, const int64_t *ptr_x, const int64_t *ptr_y,
                            int64_t P, int64_t NX, int64_t NY, int32_t D, double sigma,
                            double *loss, double *Kxx, double *Kyy, double *Kxy, double *grad_x,
                            double *grad_y, double *grad_wx, double *grad_wy, double *grad_sigma,
                            void *workspace, size_t workspace_bytes, ra_stream_t stream);

/* Dense matrices of one pair (kde_gradients.py:32-36):
 * G[i][j] = exp(-|a_i - b_j|^2 / (2 sigma^2)) [n, m] and
 * diff[i][j][d] = a_i[d] - b_j[d] [n, m, D], float64; either output may be
 * NULL.  At most 2^36 entries. */
RA_API int ra_kde_exact_matrices_f64(const double *a, int64_t n, const double *b, int64_t m,
                                     int32_t D, double sigma, double *G, double *diff,
                                     ra_stream_t stream);

/* ---- pairwise-distance spectrum loss ------------------------------------ */
/* Replaces the per-graph loop of rapidalign/algorithms.py:54-90
 * (pairwise_distance_loss): per group g, the sorted distances of all point
 * pairs of the source group and of the target group, the shorter list padded
 * with zeros at its end, loss[g] = mean of the squared differences over the
 * longer length (NaN when both groups have < 2 points).
 *
 * A cloud: points [N, D] (float32), optional perm [N] (the point at grouped
 * position k is perm[k]; NULL = identity), ptr [G + 1] (grouped positions of
 * each group), pair_offsets [G + 1] (exclusive scan of n_g (n_g - 1) / 2),
 * all device arrays; num_pairs = pair_offsets[G] and max_group = the largest
 * n_g, both known to the host (at most 65536 points per group and
 * 2^31 - 1 pairs per cloud).  The backward reads the sorted distances the
 * forward left in the workspace. */
typedef struct ra_pdl_cloud {
  const float *points;
  const int64_t *perm;
  const int64_t *ptr;
  const int64_t *pair_offsets;
  int64_t num_pairs;
  int64_t max_group;
} ra_pdl_cloud;

RA_API size_t ra_pdl_workspace_bytes(int64_t G, int64_t pairs_src, int64_t pairs_tgt);
RA_API int ra_pdl_forward(const ra_pdl_cloud *src, const ra_pdl_cloud *tgt, int64_t G,
                          int32_t D, double *loss, void *workspace, size_t workspace_bytes,
                          ra_stream_t stream);
/* Adds d(sum_g grad_loss[g] loss[g]) / d points into grad_src / grad_tgt
 * (float32 [N, D], caller-zeroed; either may be NULL). */
RA_API int ra_pdl_backward(const ra_pdl_cloud *src, const ra_pdl_cloud *tgt, int64_t G,
                           int32_t D, const double *grad_loss, float *grad_src, float *grad_tgt,
                           void *workspace, size_t workspace_bytes, ra_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* RAPIDALIGN_B200_H */
