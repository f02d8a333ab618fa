// dq_moe.cu -- the elementwise steps around the split GEMVs of a mixture-of-
// experts FFN (Mixtral-style: y = w2 (silu(w1 x) * (w3 x)), top-k routing):
// the gated activation and the weighted combine of the experts' outputs.
// Both are memory-bound and tiny next to the GEMVs; 16-byte accesses.
#include "dq_common.cuh"
#include "dq_internal.h"

namespace dq {

namespace {

__device__ __forceinline__ uint32_t word_of_u4(const uint4& v, int i) {
    return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}

// h = fp16(silu(a) * b) with silu(v) = v / (1 + exp(-v)), FP32 arithmetic,
// over rows of d8 pieces of 8 values: a and b rows ld8 pieces apart, h rows
// contiguous.
__global__ void silu_mul_kernel(const uint16_t* __restrict__ a, const uint16_t* __restrict__ b,
                                uint16_t* __restrict__ h, long long rows, long long d8, long long ld8) {
    const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    pdl_launch_dependents();
    pdl_wait();
    if (i >= rows * d8) return;
    const long long r = i / d8, src = r * ld8 + (i - r * d8);
    const uint4 va = ldcg_v4(a + 8 * src), vb = ldcg_v4(b + 8 * src);
    uint32_t out[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const uint32_t wa = word_of_u4(va, k), wb = word_of_u4(vb, k);
        float r[2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const float x = h2f_bits(j ? hi16(wa) : lo16(wa));
            const float g = h2f_bits(j ? hi16(wb) : lo16(wb));
            r[j] = __fdiv_rn(x, 1.0f + expf(-x)) * g;
        }
        out[k] = pack_h2(__half_as_ushort(__float2half_rn(r[0])), __half_as_ushort(__float2half_rn(r[1])));
    }
    *reinterpret_cast<uint4*>(h + 8 * i) = make_uint4(out[0], out[1], out[2], out[3]);
}

// out[rows[i]][:] += weight[i] * y[i][:] (FP32 out, FP16 y), rows distinct
// within one call.
__global__ void combine_kernel(const uint16_t* __restrict__ y, const int32_t* __restrict__ rows,
                               const float* __restrict__ weight, float* __restrict__ out, int m, int d8) {
    const int i = blockIdx.y;
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    pdl_launch_dependents();
    pdl_wait();
    if (i >= m || c >= d8) return;
    const int r = rows[i];
    const float wt = weight[i];
    const uint4 v = ldcg_v4(y + (static_cast<size_t>(i) * d8 + c) * 8);
    float* o = out + (static_cast<size_t>(r) * d8 + c) * 8;
    float4 o0 = *reinterpret_cast<float4*>(o), o1 = *reinterpret_cast<float4*>(o + 4);
    o0.x = fmaf(wt, h2f_bits(lo16(v.x)), o0.x);
    o0.y = fmaf(wt, h2f_bits(hi16(v.x)), o0.y);
    o0.z = fmaf(wt, h2f_bits(lo16(v.y)), o0.z);
    o0.w = fmaf(wt, h2f_bits(hi16(v.y)), o0.w);
    o1.x = fmaf(wt, h2f_bits(lo16(v.z)), o1.x);
    o1.y = fmaf(wt, h2f_bits(hi16(v.z)), o1.y);
    o1.z = fmaf(wt, h2f_bits(lo16(v.w)), o1.z);
    o1.w = fmaf(wt, h2f_bits(hi16(v.w)), o1.w);
    *reinterpret_cast<float4*>(o) = o0;
    *reinterpret_cast<float4*>(o + 4) = o1;
}

template <class K, class... A>
dq_status_t launch_pdl_plain(K kernel, dim3 grid, int threads, cudaStream_t stream, A... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, args...);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) { set_cuda_error(e); return DQ_ERR_CUDA; }
    return DQ_OK;
}

}  // namespace

dq_status_t launch_silu_mul(const uint16_t* a, const uint16_t* b, uint16_t* h, long long rows, long long d,
                            long long ld, cudaStream_t stream) {
    const long long n8 = rows * (d / 8);
    if (n8 == 0) return DQ_OK;
    const int threads = 256;
    const long long blocks = (n8 + threads - 1) / threads;
    return launch_pdl_plain(silu_mul_kernel, dim3(static_cast<unsigned>(blocks)), threads, stream, a, b, h, rows,
                            d / 8, ld / 8);
}

dq_status_t launch_combine(const uint16_t* y, const int32_t* rows, const float* weight, float* out, int m, int d,
                           cudaStream_t stream) {
    if (m == 0) return DQ_OK;
    const int d8 = d / 8, threads = 128;
    return launch_pdl_plain(combine_kernel, dim3((d8 + threads - 1) / threads, m), threads, stream, y, rows, weight,
                            out, m, d8);
}

}  // namespace dq
