// dq_internal.h -- host-side interface between the C ABI (dq_abi.cu) and the
// kernel translation units.  Not installed; include/dq_abi.h is the public API.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/dq_abi.h"

namespace dq {

// Shared-memory plan of the single-pass GEMV kernels for a given d_in and
// row-blocks-per-CTA bound.  Identical on host (sizing) and device (carving).
struct SmemLayout {
    int sx, bsm, mask, xp, goff, list, part, misc, total;
};

__host__ __device__ inline int align16(int v) { return (v + 15) & ~15; }

__host__ __device__ inline SmemLayout smem_layout(int d_in, int nrb_max, int nw, bool split) {
    const int G = d_in / 128;
    SmemLayout L;
    int off = 0;
    L.sx = off;   off += align16(2 * d_in);             // raw x, f16
    L.bsm = off;  off += G * 256;                       // MMA B fragments, f16 (token 0)
    L.mask = off; off += align16(d_in / 8);             // outlier bitmask bytes
    L.xp = off;   off += align16(4 * G);                // per-group sum of non-outlier x, f32
    L.goff = off; off += align16(4 * (G + 1));          // per-group outlier list offsets
    L.list = off; off += split ? align16(d_in) : 0;     // outlier columns (<= d_in/4 int32)
    L.part = off; off += nrb_max * nw * 16 * 4;         // per-warp row partial sums
    L.misc = off; off += 256;                           // reduction scratch + stats + stripe counts
    L.total = off;
    return L;
}

// Device facts cached per ordinal.
struct DeviceInfo {
    int sm_count;
    int smem_optin;
};
dq_status_t device_info(DeviceInfo* out);

void set_cuda_error(cudaError_t e);

// Kernel launchers (arguments already validated by the C ABI layer).
dq_status_t launch_gemv_m1(const dq_weights_t& w, const uint16_t* x, uint16_t* y, float k,
                           bool split, cudaStream_t stream);
dq_status_t launch_reference_gemv(const uint16_t* w16, const uint16_t* x, uint16_t* y, int d_out,
                                  int d_in, cudaStream_t stream);
dq_status_t launch_detect(const uint16_t* x, int d_in, float k, uint32_t* mask_words,
                          int32_t* indices, int32_t* count, float* stats, cudaStream_t stream);
dq_status_t launch_quantize(const uint16_t* w16, int d_out, int d_in, uint8_t* packed,
                            uint16_t* scales, uint16_t* zeros, cudaStream_t stream);
dq_status_t launch_colmajor(const uint16_t* w16, int d_out, int d_in, uint16_t* cm,
                            cudaStream_t stream);

// Largest d_in the single-pass kernels accept.
constexpr int kMaxDIn = 32768;
// Threads per CTA of the single-pass kernels (the detector uses the same count
// so its mask is bit-identical to the one the GEMV applies).
constexpr int kGemvWarps = 16;

}  // namespace dq
