// ref_gpu_harness.cu -- C entry points into the reference's own GPU kernels.
//
// TEST INFRASTRUCTURE ONLY (oracle side).  oracle/build_oracle.py compiles
// this file together with the reference's src/{split,int4,reference}_gemv.cu
// for sm_100a, with the reference's own flags (-O3 -use_fast_math
// --expt-relaxed-constexpr), into oracle/_ref/libdqref_gpu.so, which is never
// committed.  The reference does not compile as shipped; the build works on a
// scratch copy outside the repository with three minimal patches:
//   P1 src/quant_format.cuh:26   pack_int4 gains __host__ (host quantizer calls it)
//   P2 src/outlier_detect.cuh:108 int* smem_warp_mean -> float* (what its comment says)
//   P3 src/split_gemv.cu:190     cudaFuncSetAttribute(MaxDynamicSharedMemorySize)
//                                before the launch (needed when 2*d_in+580 > 48 KB)
// Nothing else changes.  In particular the s_packed staging of
// src/split_gemv.cu:85-93 is left as written: it stages rows 0..1 of each
// 4-row block only, so rows with row % 4 in {2, 3} read shared memory that is
// never written, and their outputs are not meaningful.
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "quant_format.cuh"
#include "outlier_detect.cuh"
#include "split_gemv.cuh"
#include "int4_gemv.cuh"
#include "reference_gemv.cuh"

static QuantizedWeights make_view(const uint8_t* packed, const void* scales, const void* zeros,
                                  const void* fp16_w, int d_out, int d_in) {
    QuantizedWeights q;
    q.packed = const_cast<uint8_t*>(packed);
    q.scales = reinterpret_cast<__half*>(const_cast<void*>(scales));
    q.zeros = reinterpret_cast<__half*>(const_cast<void*>(zeros));
    q.fp16_weights = reinterpret_cast<__half*>(const_cast<void*>(fp16_w));
    q.d_out = d_out;
    q.d_in = d_in;
    return q;
}

extern "C" int dqref_split_gemv(const uint8_t* packed, const void* scales, const void* zeros,
                                const void* fp16_w, const void* x, void* y, int d_out, int d_in,
                                float k, void* stream) {
    QuantizedWeights q = make_view(packed, scales, zeros, fp16_w, d_out, d_in);
    launch_split_gemv(q, static_cast<const __half*>(x), static_cast<__half*>(y), d_out, d_in, k,
                      static_cast<cudaStream_t>(stream));
    return static_cast<int>(cudaGetLastError());
}

extern "C" int dqref_int4_gemv(const uint8_t* packed, const void* scales, const void* zeros,
                               const void* x, void* y, int d_out, int d_in, void* stream) {
    QuantizedWeights q = make_view(packed, scales, zeros, nullptr, d_out, d_in);
    launch_int4_gemv(q, static_cast<const __half*>(x), static_cast<__half*>(y), d_out, d_in,
                     static_cast<cudaStream_t>(stream));
    return static_cast<int>(cudaGetLastError());
}

extern "C" int dqref_reference_gemv(const void* w, const void* x, void* y, int d_out, int d_in,
                                    void* stream) {
    launch_reference_gemv(static_cast<const __half*>(w), static_cast<const __half*>(x),
                          static_cast<__half*>(y), d_out, d_in, static_cast<cudaStream_t>(stream));
    return static_cast<int>(cudaGetLastError());
}

// One 128-thread block runs the reference's scan_outliers_block with the same
// shared-memory carve and capacity as split_gemv_kernel (src/split_gemv.cu:46-64),
// then exports the index list, the count and the merged Welford state.
__global__ void dqref_detect_kernel(const __half* x, int n, float k, int capacity,
                                    int* indices, int* count, float* stats) {
    extern __shared__ char smem[];
    const int num_warps = 4;
    float* smem_warp_mean = reinterpret_cast<float*>(smem);
    float* smem_warp_M2 = smem_warp_mean + num_warps;
    int* smem_warp_count = reinterpret_cast<int*>(smem_warp_M2 + num_warps);
    int* smem_warp_ocounts = smem_warp_count + num_warps;
    int* outlier_count = smem_warp_ocounts + num_warps;
    int* outlier_indices = outlier_count + 1;
    int* scratch = outlier_indices + capacity;
    if (threadIdx.x == 0) *outlier_count = 0;
    __syncthreads();
    scan_outliers_block(x, n, k, smem_warp_mean, smem_warp_M2, smem_warp_count, smem_warp_ocounts,
                        outlier_indices, outlier_count, scratch, capacity);
    const int c = *outlier_count;
    for (int i = threadIdx.x; i < c; i += blockDim.x) indices[i] = outlier_indices[i];
    if (threadIdx.x == 0) {
        *count = c;
        float mean = smem_warp_mean[0];
        float m2 = smem_warp_M2[0];
        int cnt = smem_warp_count[0];
        float var = (cnt > 1) ? m2 / static_cast<float>(cnt - 1) : 0.f;
        stats[0] = mean;
        stats[1] = k * sqrtf(fmaxf(var, 1e-8f));
        stats[2] = var;
        stats[3] = m2;
    }
}

extern "C" int dqref_detect(const void* x, int n, float k, int* indices, int* count, float* stats,
                            void* stream) {
    const int capacity = n / 4;
    size_t smem = 4 * sizeof(float) * 2 + 4 * sizeof(int) * 2 + sizeof(int) +
                  2 * static_cast<size_t>(capacity) * sizeof(int);
    cudaFuncSetAttribute(dqref_detect_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(smem));
    dqref_detect_kernel<<<1, 128, smem, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const __half*>(x), n, k, capacity, indices, count, stats);
    return static_cast<int>(cudaGetLastError());
}
