/*
 * dq_reference_api.hpp -- the reference's C++ host API, header-only, on top of
 * the C ABI of include/dq_abi.h.
 *
 * Same names, signatures and conventions as dyn-quant's
 *   src/quant_format.cuh:12-23, 58-124   QuantizedWeights, quantize_weights_host,
 *                                        free_quantized_weights
 *   src/split_gemv.cuh:10-18             launch_split_gemv
 *   src/int4_gemv.cuh:9-16               launch_int4_gemv
 *   src/reference_gemv.cuh:10-17         launch_reference_gemv
 * so that C++ code written against the reference compiles unchanged when it
 * includes this header instead of the reference's headers and links
 * libdq_b200.so.  As in the reference, the launchers return void and are
 * stream-ordered; the status of the last call on this thread is available
 * from dq_ref_last_status() (the reference reports no errors at all).
 *
 * Differences in mechanism, not in results:
 *  - quantize_weights_host uploads the FP16 matrix and quantizes it on the GPU
 *    (bit-identical to the reference's host loop) instead of on the CPU.
 *  - On the first GEMV call for a given QuantizedWeights, the shim builds the
 *    two load-time layouts the fast kernels stream (dq_build_native,
 *    dq_build_colmajor) and keeps them until free_quantized_weights.  Weights
 *    changed in place after that first call must be re-registered by freeing
 *    and re-quantizing (or by calling dq_ref_forget(W)).
 *  - Each device gets one zero-filled GEMV workspace, allocated on first use.
 *    Calls on one device from several host threads or unordered streams must
 *    not overlap, as with any shared workspace.
 */
#ifndef DQ_REFERENCE_API_HPP_
#define DQ_REFERENCE_API_HPP_

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>
#include <unordered_map>

#include "dq_abi.h"

static constexpr int GROUP_SIZE = 128;

struct QuantizedWeights {
    uint8_t* packed;         // [d_out][d_in/2], column 2j in bits 3:0 of byte j
    __half* scales;          // [d_out][d_in/GROUP_SIZE]
    __half* zeros;           // [d_out][d_in/GROUP_SIZE]
    __half* fp16_weights;    // [d_out][d_in], row-major
    int d_out;
    int d_in;
};

namespace dq_ref_detail {

inline dq_status_t& last_status() {
    thread_local dq_status_t s = DQ_OK;
    return s;
}

struct Layouts {
    uint8_t* native = nullptr;
    uint16_t* fp16_cm = nullptr;
};

inline std::mutex& mu() {
    static std::mutex m;
    return m;
}
inline std::unordered_map<const void*, Layouts>& layouts() {
    static std::unordered_map<const void*, Layouts> m;
    return m;
}

// Zero-filled workspace of the current device (allocated once, kept).
inline void* workspace(size_t need) {
    static void* ws[64] = {};
    static size_t bytes[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lock(mu());
    if (bytes[dev] < need) {
        if (ws[dev]) cudaFree(ws[dev]);
        ws[dev] = nullptr;
        bytes[dev] = 0;
        if (cudaMalloc(&ws[dev], need) != cudaSuccess) return nullptr;
        if (cudaMemset(ws[dev], 0, need) != cudaSuccess) return nullptr;
        bytes[dev] = need;
    }
    return ws[dev];
}

inline Layouts layouts_for(const QuantizedWeights& W, cudaStream_t stream) {
    {
        std::lock_guard<std::mutex> lock(mu());
        auto it = layouts().find(W.packed);
        if (it != layouts().end()) return it->second;
    }
    Layouts L;
    const size_t nb = dq_native_bytes(W.d_out, W.d_in);
    if (nb && cudaMalloc(&L.native, nb) == cudaSuccess)
        if (dq_build_native(W.packed, reinterpret_cast<const uint16_t*>(W.scales),
                            reinterpret_cast<const uint16_t*>(W.zeros), W.d_out, W.d_in, L.native,
                            stream) != DQ_OK) {
            cudaFree(L.native);
            L.native = nullptr;
        }
    const size_t cm = static_cast<size_t>(W.d_out) * W.d_in * sizeof(uint16_t);
    if (W.fp16_weights && cm && cudaMalloc(&L.fp16_cm, cm) == cudaSuccess)
        if (dq_build_colmajor(reinterpret_cast<const uint16_t*>(W.fp16_weights), W.d_out, W.d_in, L.fp16_cm,
                              stream) != DQ_OK) {
            cudaFree(L.fp16_cm);
            L.fp16_cm = nullptr;
        }
    std::lock_guard<std::mutex> lock(mu());
    layouts()[W.packed] = L;
    return L;
}

inline dq_weights_t view(const QuantizedWeights& W, const Layouts& L) {
    dq_weights_t w;
    w.packed = W.packed;
    w.scales = reinterpret_cast<const uint16_t*>(W.scales);
    w.zeros = reinterpret_cast<const uint16_t*>(W.zeros);
    w.fp16 = reinterpret_cast<const uint16_t*>(W.fp16_weights);
    w.fp16_cm = L.fp16_cm;
    w.native = L.native;
    w.d_out = W.d_out;
    w.d_in = W.d_in;
    return w;
}

}  // namespace dq_ref_detail

// Status of the last call of this header's API on this thread.
inline dq_status_t dq_ref_last_status() { return dq_ref_detail::last_status(); }

// Drops the cached fast layouts of W (call after changing W's arrays in place).
inline void dq_ref_forget(const QuantizedWeights& W) {
    dq_ref_detail::Layouts L;
    {
        std::lock_guard<std::mutex> lock(dq_ref_detail::mu());
        auto it = dq_ref_detail::layouts().find(W.packed);
        if (it == dq_ref_detail::layouts().end()) return;
        L = it->second;
        dq_ref_detail::layouts().erase(it);
    }
    cudaDeviceSynchronize();
    if (L.native) cudaFree(L.native);
    if (L.fp16_cm) cudaFree(L.fp16_cm);
}

// src/quant_format.cuh:58-111: quantize a host FP16 [d_out][d_in] matrix; the
// returned device arrays are owned by the caller (free_quantized_weights).
inline QuantizedWeights quantize_weights_host(const __half* host_fp16, int d_out, int d_in) {
    QuantizedWeights q{nullptr, nullptr, nullptr, nullptr, d_out, d_in};
    const size_t n = static_cast<size_t>(d_out) * d_in;
    const size_t ng = static_cast<size_t>(d_out) * (d_in / GROUP_SIZE);
    dq_status_t st = DQ_ERR_CUDA;
    if (cudaMalloc(&q.packed, n / 2) == cudaSuccess && cudaMalloc(&q.scales, ng * sizeof(__half)) == cudaSuccess &&
        cudaMalloc(&q.zeros, ng * sizeof(__half)) == cudaSuccess &&
        cudaMalloc(&q.fp16_weights, n * sizeof(__half)) == cudaSuccess &&
        cudaMemcpy(q.fp16_weights, host_fp16, n * sizeof(__half), cudaMemcpyHostToDevice) == cudaSuccess) {
        st = dq_quantize(reinterpret_cast<const uint16_t*>(q.fp16_weights), d_out, d_in, q.packed,
                         reinterpret_cast<uint16_t*>(q.scales), reinterpret_cast<uint16_t*>(q.zeros), nullptr);
        if (st == DQ_OK && cudaDeviceSynchronize() != cudaSuccess) st = DQ_ERR_CUDA;
    }
    dq_ref_detail::last_status() = st;
    return q;
}

// src/quant_format.cuh:118-123
inline void free_quantized_weights(QuantizedWeights& q) {
    dq_ref_forget(q);
    cudaFree(q.packed);
    cudaFree(q.scales);
    cudaFree(q.zeros);
    cudaFree(q.fp16_weights);
}

// src/split_gemv.cuh:10-18
inline void launch_split_gemv(const QuantizedWeights& W, const __half* x, __half* y, int d_out, int d_in,
                              float outlier_k, cudaStream_t stream = 0) {
    QuantizedWeights v = W;
    v.d_out = d_out;
    v.d_in = d_in;
    const dq_ref_detail::Layouts L = dq_ref_detail::layouts_for(v, stream);
    const dq_weights_t w = dq_ref_detail::view(v, L);
    const size_t need = dq_workspace_bytes(d_out, d_in);
    void* ws = dq_ref_detail::workspace(need);
    dq_ref_detail::last_status() =
        ws ? dq_split_gemv(&w, reinterpret_cast<const uint16_t*>(x), reinterpret_cast<uint16_t*>(y), outlier_k, ws,
                           need, stream)
           : DQ_ERR_CUDA;
}

// src/int4_gemv.cuh:9-16
inline void launch_int4_gemv(const QuantizedWeights& W, const __half* x, __half* y, int d_out, int d_in,
                             cudaStream_t stream = 0) {
    QuantizedWeights v = W;
    v.d_out = d_out;
    v.d_in = d_in;
    const dq_ref_detail::Layouts L = dq_ref_detail::layouts_for(v, stream);
    const dq_weights_t w = dq_ref_detail::view(v, L);
    const size_t need = dq_workspace_bytes(d_out, d_in);
    void* ws = dq_ref_detail::workspace(need);
    dq_ref_detail::last_status() =
        ws ? dq_int4_gemv(&w, reinterpret_cast<const uint16_t*>(x), reinterpret_cast<uint16_t*>(y), ws, need, stream)
           : DQ_ERR_CUDA;
}

// src/reference_gemv.cuh:10-17
inline void launch_reference_gemv(const __half* W_fp16, const __half* x, __half* y, int d_out, int d_in,
                                  cudaStream_t stream = 0) {
    dq_ref_detail::last_status() =
        dq_reference_gemv(reinterpret_cast<const uint16_t*>(W_fp16), reinterpret_cast<const uint16_t*>(x),
                          reinterpret_cast<uint16_t*>(y), d_out, d_in, stream);
}

#endif  // DQ_REFERENCE_API_HPP_
