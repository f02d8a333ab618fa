/*
 * dq_abi.h -- C ABI of the dyn-quant B200 library (libdq_b200.so).
 *
 * Plain C: pointers, sizes and a status code; no CUDA or torch types.  Device
 * buffers are raw device pointers; FP16 values are IEEE binary16 bit patterns
 * (uint16_t); `stream` is a cudaStream_t passed as void* (NULL = legacy
 * default stream).  Every call is stream-ordered and asynchronous: it enqueues
 * work and returns; nothing allocates device memory and nothing synchronises.
 *
 * Each entry point names the reference interface it replaces (paths inside the
 * dyn-quant project).  The reference's launchers return void and check no CUDA
 * error (src/split_gemv.cu:160-198); here every call validates its arguments
 * and returns a dq_status_t, with the CUDA error of a failed launch available
 * from dq_last_cuda_error().
 *
 * Formats (bit-compatible with the reference, src/quant_format.cuh:12-38):
 *   packed   uint8  [d_out][d_in/2]   column 2j in bits 3:0 of byte j, 2j+1 in bits 7:4
 *   scales   f16    [d_out][d_in/128] per-group scale
 *   zeros    f16    [d_out][d_in/128] per-group zero-point; w = scale * (code - zero)
 *   fp16     f16    [d_out][d_in]     original weights, row-major (as the reference keeps them)
 *   fp16_cm  f16    [d_in][d_out]     the same weights column-major (the outlier-column
 *                                     mirror: one outlier column is d_out contiguous halves)
 * Alignment: packed, x, fp16, fp16_cm and w16 need 16-byte aligned pointers;
 * scales and zeros 2-byte.  d_in must be a positive multiple of 128.
 */
#ifndef DQ_ABI_H_
#define DQ_ABI_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define DQ_API __attribute__((visibility("default")))
#else
#define DQ_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum dq_status_t {
    DQ_OK = 0,
    DQ_ERR_INVALID_ARGUMENT = 1, /* null pointer where one is required, bad k */
    DQ_ERR_SHAPE = 2,            /* d_in not a positive multiple of 128, negative d_out, ... */
    DQ_ERR_ALIGNMENT = 3,        /* a pointer misses its required alignment */
    DQ_ERR_UNSUPPORTED = 4,      /* shape beyond what the kernel supports (see dq_max_d_in) */
    DQ_ERR_CUDA = 5,             /* a CUDA call failed: see dq_last_cuda_error() */
    DQ_ERR_WORKSPACE = 6         /* workspace missing or too small */
} dq_status_t;

/* Non-owning view of one quantized weight matrix (the reference's
 * QuantizedWeights, src/quant_format.cuh:12-23, plus two optional load-time
 * layouts).  At least one of fp16 / fp16_cm must be set for the split GEMV;
 * the column-major mirror is the fast path for outlier columns.  native, when
 * set (dq_build_native), is what the kernels stream instead of packed /
 * scales / zeros (which must still be valid and describe the same weights). */
typedef struct dq_weights_t {
    const uint8_t* packed;
    const uint16_t* scales;
    const uint16_t* zeros;
    const uint16_t* fp16;       /* row-major [d_out][d_in], may be NULL if fp16_cm is set */
    const uint16_t* fp16_cm;    /* column-major [d_in][d_out], may be NULL */
    const uint8_t* native;      /* unit layout from dq_build_native, 16-byte aligned, may be NULL */
    int32_t d_out;
    int32_t d_in;
} dq_weights_t;

/* Row-sharded split GEMV with the gather fused (dq_split_gemv_gather): one
 * process per GPU, every rank holding rows_per rows of the weights (the last
 * ranks zero-padded), the ranks' gather regions mapped into each other's
 * address space (dq_ipc_handle / dq_ipc_open).  region[rank] is this process's
 * own region, region[q] rank q's as mapped here. */
#define DQ_MAX_GATHER_RANKS 8
typedef struct dq_gather_t {
    int32_t rank;      /* this process, 0 <= rank < world */
    int32_t world;     /* ranks, 1 .. DQ_MAX_GATHER_RANKS */
    int32_t rows_per;  /* rows of every rank's slice, a multiple of 16 (= the local weights' d_out) */
    int32_t d_total;   /* rows of the full output, (world - 1) * rows_per < d_total <= world * rows_per */
    void* region[DQ_MAX_GATHER_RANKS];
} dq_gather_t;

/* Human-readable name of a status code (static string). */
DQ_API const char* dq_status_string(dq_status_t s);

/* The cudaError_t (as int) of the last call on this thread that returned
 * DQ_ERR_CUDA, or 0. */
DQ_API int dq_last_cuda_error(void);

/* Library version as 10000*major + 100*minor + patch. */
DQ_API int dq_version(void);

/* Largest d_in the single-pass GEMV kernels accept on this build (the
 * activation vector and its per-group tables live in shared memory). */
DQ_API int32_t dq_max_d_in(void);

/*
 * Quantize an FP16 weight matrix on the device, bit-exactly as
 * quantize_weights_host does on the host (src/quant_format.cuh:58-97):
 * per row and 128-column group, min/max -> scale = range/15 (1 if range <
 * 1e-8), zero = -min/scale, codes = clamp(trunc((v-min)/scale + 0.5), 0, 15).
 * Replaces: quantize_weights_host (src/quant_format.cuh:58), and the host
 * round trip of the torch binding (csrc/bindings.cpp:26-75).
 * w16: device [d_out][d_in] f16.  Outputs are caller-allocated device buffers.
 */
DQ_API dq_status_t dq_quantize(const uint16_t* w16, int32_t d_out, int32_t d_in, uint8_t* packed,
                        uint16_t* scales, uint16_t* zeros, void* stream);

/*
 * Build the column-major FP16 mirror fp16_cm[d_in][d_out] of w16[d_out][d_in].
 * No reference counterpart: the reference gathers outlier columns from the
 * row-major copy (src/split_gemv.cu:125,131).  Used by DynQuantLinear.load_weight.
 */
DQ_API dq_status_t dq_build_colmajor(const uint16_t* w16, int32_t d_out, int32_t d_in, uint16_t* fp16_cm,
                              void* stream);

/*
 * Native unit layout streamed by the batch-1 GEMV kernels with one bulk copy
 * per 16-row x 512-column unit: for each (16-row block, 4-group chunk), 4096
 * bytes of packed codes in the order the kernel's lanes read them, then 256
 * bytes of (scale bits | zero bits << 16) for 16 rows x 4 groups; zero-padded
 * past d_out and past the last group.  A reordering of the reference format
 * (src/quant_format.cuh:12-23), built once at load time; no reference
 * counterpart.  dq_native_bytes gives the size (0 for a bad shape).
 */
DQ_API size_t dq_native_bytes(int32_t d_out, int32_t d_in);
DQ_API dq_status_t dq_build_native(const uint8_t* packed, const uint16_t* scales, const uint16_t* zeros,
                                   int32_t d_out, int32_t d_in, uint8_t* native, void* stream);

/*
 * Workspace of the batch-1 GEMVs: device memory of at least
 * dq_workspace_bytes(d_out, d_in) bytes, 256-byte aligned, ZERO-FILLED before
 * its first use.  Its first 256 + 128 KiB hold a call counter, an arrival
 * counter and, per CTA, the partial row sums of the 16-row block that CTA
 * shares with the one before it, each tagged with the call's number so that a
 * sum left by an earlier call is never taken; then the counters of the other
 * kernels and, for rows of 24576 columns or more cut into column slabs, the
 * slabs' tagged partial row sums (8 bytes per row and slab after the first;
 * a smaller workspace runs such a call without slabs); the rest, which grows
 * with the shape, serves the streaming kernel (task queue and per-row-block
 * partial sums, DQ_STREAM=1) and the batched kernels.  Every
 * call leaves it ready for the next one, so one zero-filled workspace serves
 * any number of stream-ordered calls of any shape; after a call that reported
 * a device error (dq_read_device_error), reset it with dq_reset_workspace.
 * Calls that share a workspace must not overlap on the GPU.
 */
DQ_API size_t dq_workspace_bytes(int32_t d_out, int32_t d_in);

/*
 * Zero-fill a workspace on `stream` (an asynchronous memset of its
 * workspace_bytes, no allocation).  Needed only after
 * dq_read_device_error reported an error of a call that used the workspace:
 * such a call may leave a row block's arrival counter short.  No reference
 * counterpart.
 */
DQ_API dq_status_t dq_reset_workspace(void* workspace, size_t workspace_bytes, void* stream);

/*
 * Fused dynamic-precision GEMV, batch 1: y = W_split x.
 * Channel c is an outlier when |x_c - mean(x)| > outlier_k * std(x) (unbiased
 * variance floored at 1e-8, strict >), keeping at most d_in/16 outliers per
 * 32-column stripe class as the reference's warp capacity does
 * (src/outlier_detect.cuh:160-178).  Outlier columns use the FP16 weights, the
 * rest the INT4 codes; FP32 accumulation; y is rounded to FP16 once.
 * Enqueues one kernel, launched as a programmatic dependent of the preceding
 * work on the stream: it starts streaming weights early and reads x, y and
 * the workspace only once that work has completed.
 * Replaces: launch_split_gemv (src/split_gemv.cu:160-198, src/split_gemv.cuh:10).
 * x: device [d_in] f16, y: device [d_out] f16.
 */
DQ_API dq_status_t dq_split_gemv(const dq_weights_t* w, const uint16_t* x, uint16_t* y, float outlier_k,
                                 void* workspace, size_t workspace_bytes, void* stream);

/*
 * The split GEMV of dq_split_gemv with no workspace argument.  No counterpart
 * in the reference.
 * For callers that cannot allocate device memory at call time: runtime plugin
 * interfaces whose execute step must not allocate and pass no scratch buffer,
 * hosts with a device-memory budget fixed at start-up, C hosts that receive
 * device pointers from another runtime and have no allocator of their own.
 * The workspace is a 132 KiB static device array inside the library; every GPU
 * that loads the library holds it until the process exits.  A shape whose
 * workspace (dq_workspace_bytes) would exceed 132 KiB is rejected with
 * DQ_ERR_WORKSPACE (with the present kernels no shape does).  Arguments,
 * validation and results are otherwise those of dq_split_gemv.
 * The first call on each device (with that device current) looks up the
 * array's address and clears it on `stream`; make that first call before any
 * stream capture.  All calls on a device share the array, and each call leaves
 * it ready for the next (also after a device error: the partial sums carry
 * their call's number, so a late word of a call whose wait gave up is never
 * taken by a later call): calls whose GPU work overlaps (unordered streams,
 * or several host threads at once) race on it and give wrong results.
 * Allocates nothing: no cudaMalloc, cudaFree or allocating library routine.
 */
DQ_API dq_status_t dq_split_gemv_noalloc(const dq_weights_t* w, const uint16_t* x, uint16_t* y,
                                         float outlier_k, void* stream);

/*
 * Zero-fill dq_split_gemv_noalloc's static array on the current device, on
 * `stream` (an asynchronous memset, no allocation).  After a call that
 * reported a device error (dq_read_device_error: a bounded wait gave up) the
 * array holds that call's tagged partial sums and a completed-call count that
 * later calls still use correctly, so nothing needs resetting; a caller that
 * wants the array back in its first-call state (after a CUDA error it has
 * recovered from, say) calls this, ordered before the next no-alloc call.  No
 * counterpart in the reference.
 */
DQ_API dq_status_t dq_reset_noalloc_workspace(void* stream);

/*
 * Workspace of dq_split_gemv_batched for m vectors: at least
 * dq_workspace_bytes_batched(d_out, d_in, m) bytes, 256-byte aligned and
 * ZERO-FILLED before its first use.  It begins with the batch-1 region (so one
 * workspace serves both entry points and every shape it is large enough for),
 * then scratch that each call overwrites (masks, the outlier-only rows, the
 * x' tables, the outlier union and its activation table, per-slab partial
 * sums).  Calls that share a
 * workspace must not overlap on the GPU.  Every call leaves it ready for the
 * next one (after a device error: dq_reset_workspace).  0 on invalid shapes.
 */
DQ_API size_t dq_workspace_bytes_batched(int32_t d_out, int32_t d_in, int32_t m);

/*
 * Split GEMV of m activation vectors at once (1 <= m <= 16): for every i,
 * y[i] = the split GEMV of x[i] as dq_split_gemv computes it, with x[i]'s own
 * statistics and outlier mask (bit-identical to the batch-1 mask).  The INT4
 * weights are streamed once for all vectors; the FP16 weights of the union of
 * the m masks' columns are read once.  FP32 accumulation, y rounded to FP16
 * once; results are bit-reproducible run to run (fixed summation order), and
 * agree with m separate dq_split_gemv calls within FP32 rounding.
 * The reference has a batch-1 entry point only (launch_split_gemv,
 * src/split_gemv.cu:160-198); this is that computation per row of x.
 * Needs w->native (dq_build_native) and w->fp16_cm or w->fp16.
 * x: device [m][d_in] f16 (rows contiguous), y: device [m][d_out] f16.
 * Enqueues three kernels, each a programmatic dependent of its predecessor.
 */
DQ_API dq_status_t dq_split_gemv_batched(const dq_weights_t* w, const uint16_t* x, uint16_t* y, int32_t m,
                                         float outlier_k, void* workspace, size_t workspace_bytes,
                                         void* stream);

/*
 * Workspace of dq_split_gemv_batched_grouped: one region per problem, each
 * sized for m_max vectors (the largest m of the call).  0 on invalid
 * arguments (1 <= m_max <= 16, 1 <= groups <= 16).
 */
DQ_API size_t dq_workspace_bytes_batched_grouped(int32_t d_out, int32_t d_in, int32_t m_max, int32_t groups);

/*
 * `groups` batched split GEMVs of one shape in one set of launches: for every
 * problem e, y[e] = dq_split_gemv_batched(&w[e], x[e], m[e]).  Built for the
 * experts of a mixture-of-experts layer, each with the few tokens routed to
 * it: one launch streams every expert's weights, so the per-call latency of
 * the plan and of a short weight stream is paid once instead of per expert.
 * Each problem's results are bit-identical to its own dq_split_gemv_batched
 * call when m[e] and the call's largest m are both at most 8 or both above
 * 8; otherwise they agree within FP32 rounding (the call runs every problem
 * with the two-tile geometry, which cuts the INT4 sums into other slabs).
 * w: host array of `groups` weight descriptors of one shape, all with
 * native, and all with or all without fp16_cm; x, y: host arrays of device
 * pointers ([m[e]][d_in] and [m[e]][d_out] f16, 16-byte aligned); m: host
 * array, 1 <= m[e] <= 16; 1 <= groups <= 16.  No counterpart in the reference
 * (its entry point is batch 1).  Enqueues three kernels.
 */
DQ_API dq_status_t dq_split_gemv_batched_grouped(const dq_weights_t* w, const uint16_t* const* x,
                                                 uint16_t* const* y, const int32_t* m, int32_t groups,
                                                 float outlier_k, void* workspace, size_t workspace_bytes,
                                                 void* stream);

/*
 * Gated activation of a mixture-of-experts FFN (Mixtral-style
 * y = w2 (silu(w1 x) * (w3 x))): h = fp16(silu(a) * b) elementwise over n
 * values (n a multiple of 8), silu(v) = v / (1 + exp(-v)) in FP32.  No
 * counterpart in the reference (its MoE use is one split GEMV per token and
 * expert); the step between the batched GEMVs of an expert.
 */
DQ_API dq_status_t dq_silu_mul(const uint16_t* a, const uint16_t* b, uint16_t* h, int64_t n, void* stream);

/*
 * The same gated activation on the output of the fused gate/up projection
 * [w1; w3] (one split GEMV with both matrices stacked): ab is [rows][2d],
 * row r holding (w1 x_r, w3 x_r); h[r][j] = fp16(silu(ab[r][j]) * ab[r][d + j]),
 * h [rows][d] (d a multiple of 8).  No counterpart in the reference.
 */
DQ_API dq_status_t dq_silu_mul_pairs(const uint16_t* ab, uint16_t* h, int32_t rows, int32_t d, void* stream);

/*
 * Weighted combine of one expert's outputs: out[rows[i]][:] += weight[i] *
 * y[i][:] for i < m (y FP16 [m][d], out FP32 [tokens][d], d a multiple of 8,
 * the rows of one call distinct).  Stream-ordered calls accumulate the
 * experts in call order.  No counterpart in the reference.
 */
DQ_API dq_status_t dq_moe_combine(const uint16_t* y, const int32_t* rows, const float* weight, float* out,
                                  int32_t m, int32_t d, void* stream);

/*
 * Dense INT4 GEMV (no outlier handling): y = dequant(W) x.
 * Replaces: launch_int4_gemv (src/int4_gemv.cu:80-100, src/int4_gemv.cuh:9).
 * Only packed/scales/zeros (or native) of *w are read.
 */
DQ_API dq_status_t dq_int4_gemv(const dq_weights_t* w, const uint16_t* x, uint16_t* y, void* workspace,
                                size_t workspace_bytes, void* stream);

/*
 * FP16 dense GEMV with FP32 accumulation: y = W16 x.
 * Replaces: launch_reference_gemv (src/reference_gemv.cu:60-78, src/reference_gemv.cuh:10).
 */
DQ_API dq_status_t dq_reference_gemv(const uint16_t* w16, const uint16_t* x, uint16_t* y, int32_t d_out,
                              int32_t d_in, void* stream);

/*
 * Standalone outlier detector over x[d_in] with the statistics, threshold and
 * capacity rule the split GEMV uses (bit-identical to the mask the GEMV
 * applies).  Replaces: scan_outliers_block (src/outlier_detect.cuh:104-205),
 * which in the reference exists only inside the GEMV kernel.
 * Outputs (device, caller-allocated; any may be NULL):
 *   mask_words [d_in/32] uint32  bit (c % 32) of word c/32 set for outlier c
 *   indices    [d_in/4]  int32   outlier indices in the reference's list order
 *                                (stripe class 0 ascending, then 1, 2, 3)
 *   count      [1]       int32   number of outliers (<= d_in/4)
 *   stats      [4]       float   mean, threshold, unbiased variance, M2
 */
DQ_API dq_status_t dq_detect_outliers(const uint16_t* x, int32_t d_in, float outlier_k,
                               uint32_t* mask_words, int32_t* indices, int32_t* count,
                               float* stats, void* stream);

/*
 * Bytes of one rank's gather region for slices of rows_per rows (0 on a bad
 * size).  The region is device memory, 256-byte aligned, zero-filled once
 * before its first use, shared by all the calls of one weight matrix (every
 * rank making the same calls in the same order).
 */
DQ_API size_t dq_gather_region_bytes(int32_t rows_per);

/*
 * Row-sharded split GEMV with the all-gather fused into the kernel: this
 * rank's rows of y = the split GEMV of x (w->d_out == g->rows_per, native
 * layout and column-major mirror required), then the full y[d_total] on every
 * rank.  Every output row is stored in y and, over NVLink, in every other
 * rank's region, as one 32-bit word: the FP16 value in the low half and the
 * low 16 bits of the call's number in the high half (the region: a 256-byte
 * header holding u32 [calls completed], then two copies of the full output,
 * 8 x rows_per words each, for calls of parity 0 and 1).  Each CTA then reads
 * the same rows of every other rank's slice from this rank's own region as
 * soon as their words carry this call's tag (bounded wait, about a second:
 * on timeout bit 4 of the device error word is set and those rows are left
 * unwritten) and writes them into y.  No fences, flags or reads of another
 * rank's memory.  All ranks call it with the same shapes, in the same order;
 * y is this process's own buffer.  Replaces launch_split_gemv
 * (src/split_gemv.cu:160-198) on a slice of the rows plus the collective
 * that would follow it.
 */
DQ_API dq_status_t dq_split_gemv_gather(const dq_weights_t* w, const uint16_t* x, uint16_t* y, float outlier_k,
                                        void* workspace, size_t workspace_bytes, const dq_gather_t* g,
                                        void* stream);

/*
 * Device memory for gather regions and its interprocess mapping (CUDA IPC,
 * plain peer access: no multicast objects).  dq_ipc_handle writes the 64-byte
 * handle of a block from dq_device_alloc; dq_ipc_open maps another process's
 * block into this one (the same GPU node, peer access enabled on demand);
 * dq_ipc_close unmaps it.
 */
DQ_API dq_status_t dq_device_alloc(size_t bytes, void** ptr);
DQ_API dq_status_t dq_device_free(void* ptr);
DQ_API dq_status_t dq_ipc_handle(void* ptr, uint8_t handle[64]);
DQ_API dq_status_t dq_ipc_open(const uint8_t handle[64], void** ptr);
DQ_API dq_status_t dq_ipc_close(void* ptr);

/*
 * Device error word of this library on the current device: bit 0 is set by a
 * batch-1 kernel whose bounded wait for its own bulk copies gave up (the
 * kernel then drains its copies, skips the remaining work and returns; its
 * output is not valid), bit 1 by a batch-1 kernel whose bounded wait for a
 * neighbouring CTA's partial sums gave up, bit 4 by a gathering kernel whose
 * bounded wait for another rank's rows gave up, bit 5 by the streaming kernel
 * (DQ_STREAM=1) whose bounded wait for its own bulk copies gave up (it
 * carries on; its output is not valid), bit 8 by a batched kernel
 * whose bounded wait for its own bulk copies gave up.  Synchronous; clear != 0
 * resets the word.  No reference counterpart.
 */
DQ_API dq_status_t dq_read_device_error(uint32_t* word, int clear);

#ifdef __cplusplus
}
#endif

#endif /* DQ_ABI_H_ */
