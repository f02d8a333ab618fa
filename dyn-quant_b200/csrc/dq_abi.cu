// dq_abi.cu -- the extern "C" entry points of include/dq_abi.h: argument
// validation, error reporting, then the kernel launchers.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "dq_internal.h"

namespace dq {

namespace {
thread_local int t_last_cuda_error = 0;

constexpr int kMaxDev = 64;
int g_sm_count[kMaxDev];
int g_smem_optin[kMaxDev];

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline bool aligned2(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 1u) == 0; }

dq_status_t check_dims(int32_t d_out, int32_t d_in) {
    if (d_out < 0 || d_in <= 0 || d_in % 128 != 0) return DQ_ERR_SHAPE;
    return DQ_OK;
}
}  // namespace

void set_cuda_error(cudaError_t e) { t_last_cuda_error = static_cast<int>(e); }

dq_status_t device_info(DeviceInfo* out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) { set_cuda_error(e); return DQ_ERR_CUDA; }
    if (dev >= 0 && dev < kMaxDev) {
        int sm = __atomic_load_n(&g_sm_count[dev], __ATOMIC_ACQUIRE);
        if (sm > 0) {
            out->sm_count = sm;
            out->smem_optin = __atomic_load_n(&g_smem_optin[dev], __ATOMIC_ACQUIRE);
            return DQ_OK;
        }
    }
    int sm = 0, optin = 0;
    if ((e = cudaDeviceGetAttribute(&sm, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) != cudaSuccess) {
        set_cuda_error(e);
        return DQ_ERR_CUDA;
    }
    if (dev >= 0 && dev < kMaxDev) {
        __atomic_store_n(&g_smem_optin[dev], optin, __ATOMIC_RELEASE);
        __atomic_store_n(&g_sm_count[dev], sm, __ATOMIC_RELEASE);
    }
    out->sm_count = sm;
    out->smem_optin = optin;
    return DQ_OK;
}

}  // namespace dq

using namespace dq;

extern "C" {

const char* dq_status_string(dq_status_t s) {
    switch (s) {
        case DQ_OK: return "DQ_OK";
        case DQ_ERR_INVALID_ARGUMENT: return "DQ_ERR_INVALID_ARGUMENT";
        case DQ_ERR_SHAPE: return "DQ_ERR_SHAPE";
        case DQ_ERR_ALIGNMENT: return "DQ_ERR_ALIGNMENT";
        case DQ_ERR_UNSUPPORTED: return "DQ_ERR_UNSUPPORTED";
        case DQ_ERR_CUDA: return "DQ_ERR_CUDA";
        case DQ_ERR_WORKSPACE: return "DQ_ERR_WORKSPACE";
    }
    return "DQ_ERR_UNKNOWN";
}

int dq_last_cuda_error(void) { return t_last_cuda_error; }

int dq_version(void) { return 100; }  // 0.1.0

int32_t dq_max_d_in(void) { return kMaxDIn; }

dq_status_t dq_quantize(const uint16_t* w16, int32_t d_out, int32_t d_in, uint8_t* packed,
                        uint16_t* scales, uint16_t* zeros, void* stream) {
    dq_status_t st = check_dims(d_out, d_in);
    if (st != DQ_OK) return st;
    if (d_out == 0) return DQ_OK;
    if (!w16 || !packed || !scales || !zeros) return DQ_ERR_INVALID_ARGUMENT;
    if (!aligned16(w16) || !aligned16(packed) || !aligned2(scales) || !aligned2(zeros))
        return DQ_ERR_ALIGNMENT;
    return launch_quantize(w16, d_out, d_in, packed, scales, zeros, static_cast<cudaStream_t>(stream));
}

dq_status_t dq_build_colmajor(const uint16_t* w16, int32_t d_out, int32_t d_in, uint16_t* fp16_cm,
                              void* stream) {
    dq_status_t st = check_dims(d_out, d_in);
    if (st != DQ_OK) return st;
    if (d_out == 0) return DQ_OK;
    if (!w16 || !fp16_cm) return DQ_ERR_INVALID_ARGUMENT;
    if (!aligned16(w16) || !aligned2(fp16_cm)) return DQ_ERR_ALIGNMENT;
    return launch_colmajor(w16, d_out, d_in, fp16_cm, static_cast<cudaStream_t>(stream));
}

static dq_status_t check_weights(const dq_weights_t* w, const uint16_t* x, const uint16_t* y,
                                 bool need_fp16, const void* workspace, size_t workspace_bytes) {
    if (!w || !x || !y) return DQ_ERR_INVALID_ARGUMENT;
    dq_status_t st = check_dims(w->d_out, w->d_in);
    if (st != DQ_OK) return st;
    if (w->d_in > kMaxDIn) return DQ_ERR_UNSUPPORTED;
    if (w->d_out == 0) return DQ_OK;
    if (!w->packed || !w->scales || !w->zeros) return DQ_ERR_INVALID_ARGUMENT;
    if (need_fp16 && !w->fp16 && !w->fp16_cm) return DQ_ERR_INVALID_ARGUMENT;
    if (!aligned16(w->packed) || !aligned16(x) || !aligned2(y) || !aligned2(w->scales) ||
        !aligned2(w->zeros))
        return DQ_ERR_ALIGNMENT;
    if (need_fp16 && ((w->fp16 && !aligned16(w->fp16)) || (w->fp16_cm && !aligned16(w->fp16_cm))))
        return DQ_ERR_ALIGNMENT;
    if (w->native && !aligned16(w->native)) return DQ_ERR_ALIGNMENT;
    if (!workspace || workspace_bytes < ws_layout(w->d_out, w->d_in).total) return DQ_ERR_WORKSPACE;
    if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return DQ_ERR_ALIGNMENT;
    return DQ_OK;
}

size_t dq_native_bytes(int32_t d_out, int32_t d_in) {
    if (check_dims(d_out, d_in) != DQ_OK) return 0;
    return native_bytes(d_out, d_in);
}

dq_status_t dq_build_native(const uint8_t* packed, const uint16_t* scales, const uint16_t* zeros,
                            int32_t d_out, int32_t d_in, uint8_t* native, void* stream) {
    dq_status_t st = check_dims(d_out, d_in);
    if (st != DQ_OK) return st;
    if (d_out == 0) return DQ_OK;
    if (!packed || !scales || !zeros || !native) return DQ_ERR_INVALID_ARGUMENT;
    if (!aligned16(packed) || !aligned2(scales) || !aligned2(zeros) || !aligned16(native))
        return DQ_ERR_ALIGNMENT;
    return launch_build_native(packed, scales, zeros, d_out, d_in, native, static_cast<cudaStream_t>(stream));
}

dq_status_t dq_read_device_error(uint32_t* word, int clear) {
    if (!word) return DQ_ERR_INVALID_ARGUMENT;
    uint32_t b1 = 0, bg = 0, bs = 0;
    dq_status_t st = read_device_error(&b1, clear != 0);
    if (st != DQ_OK) return st;
    st = read_batched_error(&bg, clear != 0);
    if (st != DQ_OK) return st;
    st = read_stream_error(&bs, clear != 0);
    if (st != DQ_OK) return st;
    // streaming kernel: bit 0 of its word (its own copies) -> bit 5
    *word = b1 | (bg << 8) | ((bs & 1u) ? (1u << 5) : 0u);
    return DQ_OK;
}

dq_status_t dq_silu_mul(const uint16_t* a, const uint16_t* b, uint16_t* h, int64_t n, void* stream) {
    if (n < 0 || n % 8 != 0) return DQ_ERR_SHAPE;
    if (n == 0) return DQ_OK;
    if (!a || !b || !h) return DQ_ERR_INVALID_ARGUMENT;
    if (!aligned16(a) || !aligned16(b) || !aligned16(h)) return DQ_ERR_ALIGNMENT;
    return launch_silu_mul(a, b, h, 1, n, n, static_cast<cudaStream_t>(stream));
}

dq_status_t dq_silu_mul_pairs(const uint16_t* ab, uint16_t* h, int32_t rows, int32_t d, void* stream) {
    if (rows < 0 || d < 0 || d % 8 != 0) return DQ_ERR_SHAPE;
    if (rows == 0 || d == 0) return DQ_OK;
    if (!ab || !h) return DQ_ERR_INVALID_ARGUMENT;
    if (!aligned16(ab) || !aligned16(h)) return DQ_ERR_ALIGNMENT;
    return launch_silu_mul(ab, ab + d, h, rows, d, 2LL * d, static_cast<cudaStream_t>(stream));
}

dq_status_t dq_moe_combine(const uint16_t* y, const int32_t* rows, const float* weight, float* out, int32_t m,
                           int32_t d, void* stream) {
    if (m < 0 || d <= 0 || d % 8 != 0) return DQ_ERR_SHAPE;
    if (m == 0) return DQ_OK;
    if (!y || !rows || !weight || !out) return DQ_ERR_INVALID_ARGUMENT;
    if (!aligned16(y) || !aligned16(out) || (reinterpret_cast<uintptr_t>(rows) & 3u) ||
        (reinterpret_cast<uintptr_t>(weight) & 3u))
        return DQ_ERR_ALIGNMENT;
    return launch_combine(y, rows, weight, out, m, d, static_cast<cudaStream_t>(stream));
}

size_t dq_workspace_bytes_batched(int32_t d_out, int32_t d_in, int32_t m) {
    if (check_dims(d_out, d_in) != DQ_OK || m < 1 || m > kBgMaxM) return 0;
    return bg_ws(bg_geom(d_out, d_in, m), d_out, d_in).total;
}

dq_status_t dq_split_gemv_batched(const dq_weights_t* w, const uint16_t* x, uint16_t* y, int32_t m,
                                  float outlier_k, void* workspace, size_t workspace_bytes, void* stream) {
    if (m < 1 || m > kBgMaxM) return DQ_ERR_SHAPE;
    if (w && w->d_out == 0 && check_dims(w->d_out, w->d_in) == DQ_OK) return DQ_OK;
    dq_status_t st = check_weights(w, x, y, true, workspace, workspace_bytes);
    if (st != DQ_OK) return st;
    if (!w->native) return DQ_ERR_INVALID_ARGUMENT;
    if (workspace_bytes < bg_ws(bg_geom(w->d_out, w->d_in, m), w->d_out, w->d_in).total) return DQ_ERR_WORKSPACE;
    return launch_gemv_batched(*w, x, y, m, outlier_k, workspace, static_cast<cudaStream_t>(stream));
}

size_t dq_workspace_bytes_batched_grouped(int32_t d_out, int32_t d_in, int32_t m_max, int32_t groups) {
    if (check_dims(d_out, d_in) != DQ_OK || m_max < 1 || m_max > kBgMaxM || groups < 1 || groups > kBgMaxGroups)
        return 0;
    return batched_grouped_region(d_out, d_in, m_max) * static_cast<size_t>(groups);
}

dq_status_t dq_split_gemv_batched_grouped(const dq_weights_t* w, const uint16_t* const* x, uint16_t* const* y,
                                          const int32_t* m, int32_t groups, float outlier_k, void* workspace,
                                          size_t workspace_bytes, void* stream) {
    if (!w || !x || !y || !m) return DQ_ERR_INVALID_ARGUMENT;
    if (groups < 1 || groups > kBgMaxGroups) return DQ_ERR_SHAPE;
    int m_max = 0;
    for (int e = 0; e < groups; ++e) {
        if (m[e] < 1 || m[e] > kBgMaxM) return DQ_ERR_SHAPE;
        if (w[e].d_out != w[0].d_out || w[e].d_in != w[0].d_in) return DQ_ERR_SHAPE;
        if ((w[e].fp16_cm == nullptr) != (w[0].fp16_cm == nullptr)) return DQ_ERR_INVALID_ARGUMENT;
        if (m[e] > m_max) m_max = m[e];
    }
    if (w[0].d_out == 0 && check_dims(w[0].d_out, w[0].d_in) == DQ_OK) return DQ_OK;
    const size_t need = dq_workspace_bytes_batched_grouped(w[0].d_out, w[0].d_in, m_max, groups);
    for (int e = 0; e < groups; ++e) {
        const dq_status_t st = check_weights(&w[e], x[e], y[e], true, workspace, workspace_bytes);
        if (st != DQ_OK) return st;
        if (!w[e].native) return DQ_ERR_INVALID_ARGUMENT;
    }
    if (need == 0 || workspace_bytes < need) return DQ_ERR_WORKSPACE;
    return launch_gemv_batched_grouped(w, x, y, m, groups, outlier_k, workspace, static_cast<cudaStream_t>(stream));
}

size_t dq_workspace_bytes(int32_t d_out, int32_t d_in) {
    if (check_dims(d_out, d_in) != DQ_OK) return 0;
    const size_t a = stream_ws(d_out, d_in).total, b = b1_workspace_bytes(d_out, d_in);
    return a > b ? a : b;
}

dq_status_t dq_reset_workspace(void* workspace, size_t workspace_bytes, void* stream) {
    if (!workspace) return DQ_ERR_INVALID_ARGUMENT;
    // All of it: the counters at the head and the tagged words behind them
    // (a reset restarts the call tags, so no word of an earlier call may stay).
    const cudaError_t e = cudaMemsetAsync(workspace, 0, workspace_bytes, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) { set_cuda_error(e); return DQ_ERR_CUDA; }
    return DQ_OK;
}

// The split / INT4 GEMV runs the batch-1 kernel of dq_gemv.cu, which is the
// faster of the two on B200 at every Llama-2 shape measured (the fused
// gather always does).  With DQ_STREAM=1 in the environment (read once) the
// streaming kernel (dq_stream.cu) serves the plain calls it supports instead
// (native layout, column-major mirror for the split GEMV), for timing the
// two against each other.
static bool stream_requested() {
    static const bool on = [] {
        const char* s = std::getenv("DQ_STREAM");
        return s && s[0] == '1';
    }();
    return on;
}

static bool use_stream(const dq_weights_t& w, bool split, size_t workspace_bytes) {
    return stream_requested() && stream_supported(w, split) && stream_geom(w.d_out, w.d_in).n_rb <= kStreamMaxRb &&
           workspace_bytes >= stream_ws(w.d_out, w.d_in).total;
}

dq_status_t dq_split_gemv(const dq_weights_t* w, const uint16_t* x, uint16_t* y, float outlier_k,
                          void* workspace, size_t workspace_bytes, void* stream) {
    if (w && w->d_out == 0 && check_dims(w->d_out, w->d_in) == DQ_OK) return DQ_OK;
    dq_status_t st = check_weights(w, x, y, true, workspace, workspace_bytes);
    if (st != DQ_OK) return st;
    if (use_stream(*w, true, workspace_bytes))
        return launch_gemv_stream(*w, x, y, outlier_k, true, workspace, static_cast<cudaStream_t>(stream));
    return launch_gemv_b1(*w, x, y, outlier_k, true, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

size_t dq_gather_region_bytes(int32_t rows_per) {
    if (rows_per <= 0 || rows_per % 16 != 0) return 0;
    return gather_layout(rows_per).total;
}

dq_status_t dq_split_gemv_gather(const dq_weights_t* w, const uint16_t* x, uint16_t* y, float outlier_k,
                                 void* workspace, size_t workspace_bytes, const dq_gather_t* g, void* stream) {
    if (!g) return DQ_ERR_INVALID_ARGUMENT;
    if (g->world < 1 || g->world > kMaxGatherRanks || g->rank < 0 || g->rank >= g->world) return DQ_ERR_INVALID_ARGUMENT;
    if (g->rows_per <= 0 || g->rows_per % 16 != 0) return DQ_ERR_SHAPE;
    const long long full = static_cast<long long>(g->world) * g->rows_per;
    if (g->d_total > full || g->d_total <= full - g->rows_per) return DQ_ERR_SHAPE;
    for (int q = 0; q < g->world; ++q) {
        if (!g->region[q]) return DQ_ERR_INVALID_ARGUMENT;
        if ((reinterpret_cast<uintptr_t>(g->region[q]) & 255u) != 0) return DQ_ERR_ALIGNMENT;
    }
    dq_status_t st = check_weights(w, x, y, true, workspace, workspace_bytes);
    if (st != DQ_OK) return st;
    if (w->d_out != g->rows_per) return DQ_ERR_SHAPE;
    if (!w->native || !w->fp16_cm || !stream_supported(*w, true)) return DQ_ERR_INVALID_ARGUMENT;
    if (stream_geom(w->d_out, w->d_in).n_rb > kStreamMaxRb) return DQ_ERR_UNSUPPORTED;
    if (workspace_bytes < stream_ws(w->d_out, w->d_in).total) return DQ_ERR_WORKSPACE;
    return launch_gemv_b1_gather(*w, x, y, outlier_k, workspace, workspace_bytes, *g, static_cast<cudaStream_t>(stream));
}

dq_status_t dq_device_alloc(size_t bytes, void** ptr) {
    if (!ptr || bytes == 0) return DQ_ERR_INVALID_ARGUMENT;
    const cudaError_t e = cudaMalloc(ptr, bytes);
    if (e != cudaSuccess) { *ptr = nullptr; set_cuda_error(e); return DQ_ERR_CUDA; }
    return DQ_OK;
}

dq_status_t dq_device_free(void* ptr) {
    if (!ptr) return DQ_OK;
    const cudaError_t e = cudaFree(ptr);
    if (e != cudaSuccess) { set_cuda_error(e); return DQ_ERR_CUDA; }
    return DQ_OK;
}

dq_status_t dq_ipc_handle(void* ptr, uint8_t handle[64]) {
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
    if (!ptr || !handle) return DQ_ERR_INVALID_ARGUMENT;
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, ptr);
    if (e != cudaSuccess) { set_cuda_error(e); return DQ_ERR_CUDA; }
    memcpy(handle, &h, sizeof(h));
    return DQ_OK;
}

dq_status_t dq_ipc_open(const uint8_t handle[64], void** ptr) {
    if (!handle || !ptr) return DQ_ERR_INVALID_ARGUMENT;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) { *ptr = nullptr; set_cuda_error(e); return DQ_ERR_CUDA; }
    return DQ_OK;
}

dq_status_t dq_ipc_close(void* ptr) {
    if (!ptr) return DQ_OK;
    const cudaError_t e = cudaIpcCloseMemHandle(ptr);
    if (e != cudaSuccess) { set_cuda_error(e); return DQ_ERR_CUDA; }
    return DQ_OK;
}

dq_status_t dq_int4_gemv(const dq_weights_t* w, const uint16_t* x, uint16_t* y, void* workspace,
                         size_t workspace_bytes, void* stream) {
    if (w && w->d_out == 0 && check_dims(w->d_out, w->d_in) == DQ_OK) return DQ_OK;
    dq_status_t st = check_weights(w, x, y, false, workspace, workspace_bytes);
    if (st != DQ_OK) return st;
    if (use_stream(*w, false, workspace_bytes))
        return launch_gemv_stream(*w, x, y, 0.f, false, workspace, static_cast<cudaStream_t>(stream));
    return launch_gemv_b1(*w, x, y, 0.f, false, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

dq_status_t dq_reference_gemv(const uint16_t* w16, const uint16_t* x, uint16_t* y, int32_t d_out,
                              int32_t d_in, void* stream) {
    if (!w16 || !x || !y) return DQ_ERR_INVALID_ARGUMENT;
    dq_status_t st = check_dims(d_out, d_in);
    if (st != DQ_OK) return st;
    if (d_in > kMaxDIn) return DQ_ERR_UNSUPPORTED;
    if (d_out == 0) return DQ_OK;
    if (!aligned16(w16) || !aligned16(x) || !aligned2(y)) return DQ_ERR_ALIGNMENT;
    return launch_reference_gemv(w16, x, y, d_out, d_in, static_cast<cudaStream_t>(stream));
}

dq_status_t dq_detect_outliers(const uint16_t* x, int32_t d_in, float outlier_k,
                               uint32_t* mask_words, int32_t* indices, int32_t* count,
                               float* stats, void* stream) {
    if (!x) return DQ_ERR_INVALID_ARGUMENT;
    if (d_in <= 0 || d_in % 128 != 0) return DQ_ERR_SHAPE;
    if (d_in > kMaxDIn) return DQ_ERR_UNSUPPORTED;
    if (!aligned16(x)) return DQ_ERR_ALIGNMENT;
    return launch_detect(x, d_in, outlier_k, mask_words, indices, count, stats,
                         static_cast<cudaStream_t>(stream));
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Split GEMV without a caller-provided workspace.
//
// Some callers cannot allocate device memory when they call the GEMV: plugin
// interfaces of inference runtimes whose execute step must not allocate and
// hands over no scratch buffer, hosts that reserve a fixed device-memory
// budget at start-up and may not grow it afterwards, and C hosts that only
// receive device pointers from another runtime and have no allocator of their
// own.  For them the split GEMV's workspace is this file-scope device array.
// It is static device memory of the library's module: every GPU that loads
// the library holds these kStaticScratchBytes until the process exits.
//
// In host code g_dq_static_scratch is only a host-side stand-in for the
// symbol, not a device address; the device address comes from
// cudaGetSymbolAddress, looked up once per device (with that device current)
// on the first call made there.
// ---------------------------------------------------------------------------
namespace {

constexpr size_t kStaticScratchBytes = 132 * 1024;  // workspace of grids up to kMaxCtas CTAs
static_assert(kStaticScratchBytes >= 256 + sizeof(unsigned long long) * 16 * dq::kMaxCtas,
              "static scratch smaller than the split GEMV workspace");

static __device__ __align__(256) unsigned char g_dq_static_scratch[kStaticScratchBytes];

void* g_static_scratch_ptr[kMaxDev];  // device address per ordinal, set once
std::mutex g_static_scratch_mu;

// Device address of the static scratch on the current device.  The first call
// on a device looks it up and clears the array on `stream`: the workspace
// starts from zeros, and every call (also one whose bounded waits gave up)
// leaves it ready for the next call.
dq_status_t static_scratch(void** out, cudaStream_t stream) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) { set_cuda_error(e); return DQ_ERR_CUDA; }
    if (dev < 0 || dev >= kMaxDev) return DQ_ERR_UNSUPPORTED;
    void* p = __atomic_load_n(&g_static_scratch_ptr[dev], __ATOMIC_ACQUIRE);
    if (!p) {
        std::lock_guard<std::mutex> lock(g_static_scratch_mu);
        p = g_static_scratch_ptr[dev];
        if (!p) {
            e = cudaGetSymbolAddress(&p, g_dq_static_scratch);
            if (e != cudaSuccess) { set_cuda_error(e); return DQ_ERR_CUDA; }
            e = cudaMemsetAsync(p, 0, kStaticScratchBytes, stream);
            if (e != cudaSuccess) { set_cuda_error(e); return DQ_ERR_CUDA; }
            __atomic_store_n(&g_static_scratch_ptr[dev], p, __ATOMIC_RELEASE);
        }
    }
    *out = p;
    return DQ_OK;
}

}  // namespace

extern "C" dq_status_t dq_reset_noalloc_workspace(void* stream) {
    void* ws = nullptr;
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    dq_status_t st = static_scratch(&ws, s);  // (a first call clears the whole array already)
    if (st != DQ_OK) return st;
    const cudaError_t e = cudaMemsetAsync(ws, 0, kStaticScratchBytes, s);
    if (e != cudaSuccess) { set_cuda_error(e); return DQ_ERR_CUDA; }
    return DQ_OK;
}

extern "C" dq_status_t dq_split_gemv_noalloc(const dq_weights_t* w, const uint16_t* x, uint16_t* y,
                                             float outlier_k, void* stream) {
    if (w && w->d_out == 0 && check_dims(w->d_out, w->d_in) == DQ_OK) return DQ_OK;
    if (!w) return DQ_ERR_INVALID_ARGUMENT;
    dq_status_t st = check_dims(w->d_out, w->d_in);
    if (st != DQ_OK) return st;
    if (ws_layout(w->d_out, w->d_in).total > kStaticScratchBytes) return DQ_ERR_WORKSPACE;
    // Validate everything but the workspace before any CUDA call; a non-null,
    // 256-byte aligned stand-in passes the workspace checks, which the static
    // array meets by construction.
    st = check_weights(w, x, y, true, reinterpret_cast<const void*>(uintptr_t{256}), kStaticScratchBytes);
    if (st != DQ_OK) return st;
    void* ws = nullptr;
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    if ((st = static_scratch(&ws, s)) != DQ_OK) return st;
    return launch_gemv_b1(*w, x, y, outlier_k, true, ws, kStaticScratchBytes, s);
}
