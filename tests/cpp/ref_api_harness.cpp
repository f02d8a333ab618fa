// Test harness for include/dq_reference_api.hpp: C entry points that drive the
// reference-signature C++ API (quantize_weights_host, launch_*_gemv,
// free_quantized_weights) so that a pytest can call them through ctypes.
// Built by tests/test_gpu_ref_api.py with g++ against libdq_b200.so.
#include "dq_reference_api.hpp"

extern "C" int refapi_run(const uint16_t* host_w, int d_out, int d_in, const uint16_t* x_dev, float k,
                          uint16_t* y_split, uint16_t* y_int4, uint16_t* y_ref, uint8_t* packed_out,
                          int reps) {
    QuantizedWeights W = quantize_weights_host(reinterpret_cast<const __half*>(host_w), d_out, d_in);
    if (dq_ref_last_status() != DQ_OK) return 100 + dq_ref_last_status();
    for (int r = 0; r < reps; ++r) {
        launch_split_gemv(W, reinterpret_cast<const __half*>(x_dev), reinterpret_cast<__half*>(y_split), d_out, d_in,
                          k);
        if (dq_ref_last_status() != DQ_OK) return 200 + dq_ref_last_status();
    }
    launch_int4_gemv(W, reinterpret_cast<const __half*>(x_dev), reinterpret_cast<__half*>(y_int4), d_out, d_in);
    if (dq_ref_last_status() != DQ_OK) return 300 + dq_ref_last_status();
    launch_reference_gemv(W.fp16_weights, reinterpret_cast<const __half*>(x_dev), reinterpret_cast<__half*>(y_ref),
                          d_out, d_in);
    if (dq_ref_last_status() != DQ_OK) return 400 + dq_ref_last_status();
    if (cudaMemcpy(packed_out, W.packed, static_cast<size_t>(d_out) * d_in / 2, cudaMemcpyDeviceToHost) != cudaSuccess)
        return 500;
    free_quantized_weights(W);
    return cudaDeviceSynchronize() == cudaSuccess ? 0 : 600;
}
