// dq_internal.h -- host-side interface between the C ABI (dq_abi.cu) and the
// kernel translation units.  Not installed; include/dq_abi.h is the public API.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/dq_abi.h"

namespace dq {

// Geometry of the batch-1 split / INT4 kernel (shared by host sizing and
// device carving).
constexpr int kB1Warps = 8;                          // warps per CTA (one CTA per SM)
constexpr int kB1Threads = kB1Warps * 32;
constexpr int kB1Stages = 3;                         // bulk-copy ring stages per warp
constexpr int kB1ChunkGroups = 4;                    // 128-column groups per unit
constexpr int kB1UnitPacked = 4096;                  // packed INT4 of one unit (16 rows x 512 columns)
constexpr int kB1StageSZ = 256;                      // 16 rows x 4 groups x (scale, zero)
constexpr int kB1UnitBytes = kB1UnitPacked + kB1StageSZ;  // one unit of the native layout
constexpr int kB1RowPitch = 272;                     // reference layout: smem bytes per weight row
constexpr int kB1OutlierSlots = 16;                  // FP16 outlier columns staged per unit
constexpr int kB1StageOutliers = kB1UnitBytes;       // offset of the outlier slots in a stage
constexpr int kB1StageBytes = kB1UnitBytes + kB1OutlierSlots * 32;
constexpr int kPlanThreads = 1024;                   // threads of the activation-plan kernel
constexpr int kMaxCtas = 1024;                       // bound on the GEMV grid (workspace sizing)

__host__ __device__ inline int align16(int v) { return (v + 15) & ~15; }

// Activation plan: everything the GEMV needs to know about x, computed once
// per call by the plan kernel.  Same layout in the plan kernel's shared memory,
// in the workspace, and (its first copy_bytes) in each GEMV CTA's shared memory.
struct PlanLayout {
    int bsm;    // MMA B fragments of x' (outliers zeroed): 2*d_in bytes
    int xp;     // per group float4 (1024 * sum x' even cols, 1024 * sum odd cols, sum x', 0)
    int goff;   // per-group outlier list offsets, G+1 ints
    int list;   // outliers: column | FP16 bits of x << 16, capacity d_in/4
    int copy_bytes;
    int mask;   // outlier bitmask, d_in/8 bytes
    int stats;  // mean, thresh, var, M2 (float), count (int)
    int total;
};

__host__ __device__ inline PlanLayout plan_layout(int d_in) {
    const int G = d_in / 128;
    PlanLayout P;
    int off = 0;
    P.bsm = off;  off += 2 * d_in;
    P.xp = off;   off += 16 * G;
    P.goff = off; off += align16(4 * (G + 1));
    P.list = off; off += align16(4 * (d_in / 4));
    P.copy_bytes = off;
    P.mask = off; off += align16(d_in / 8);
    P.stats = off; off += 32;
    P.total = off;
    return P;
}

// Workspace of a batch-1 GEMV call: the plan, two partial-row-sum slots per
// CTA for row blocks shared with a neighbouring CTA, and one arrival counter
// per row block (zero before first use; every call leaves them zero).
struct WsLayout {
    size_t plan, fix, cnt, total;
};

inline size_t align256(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

inline WsLayout ws_layout(int d_out, int d_in) {
    WsLayout W;
    W.plan = 0;
    W.fix = align256(static_cast<size_t>(plan_layout(d_in).total));
    W.cnt = W.fix + align256(static_cast<size_t>(kMaxCtas) * 2 * 16 * sizeof(float));
    const size_t n_rb = (static_cast<size_t>(d_out) + 15) / 16;
    W.total = W.cnt + align256(n_rb * sizeof(unsigned int));
    return W;
}

// Shared-memory plan of the batch-1 GEMV kernel.
struct GemvSmem {
    int ring, bars, plan, part, misc, total;
};

__host__ __device__ inline GemvSmem gemv_smem(int d_in, int nrb_max) {
    GemvSmem S;
    int off = 0;
    S.ring = off; off += kB1Warps * kB1Stages * kB1StageBytes;
    S.bars = off; off += align16((kB1Warps * kB1Stages + 1) * 8);
    S.plan = off; off += plan_layout(d_in).copy_bytes;
    S.part = off; off += nrb_max * kB1Warps * 16 * 4;
    S.misc = off; off += 64;
    S.total = off;
    return S;
}

// Bytes of the native unit layout the batch-1 kernel streams with one bulk
// copy per unit: [row-block][4-group chunk] blocks of kB1UnitBytes.
inline size_t native_bytes(int d_out, int d_in) {
    const size_t n_rb = (static_cast<size_t>(d_out) + 15) / 16;
    const size_t nc = (static_cast<size_t>(d_in / 128) + kB1ChunkGroups - 1) / kB1ChunkGroups;
    return n_rb * nc * kB1UnitBytes;
}

// Device facts cached per ordinal.
struct DeviceInfo {
    int sm_count;
    int smem_optin;
};
dq_status_t device_info(DeviceInfo* out);

void set_cuda_error(cudaError_t e);

// Kernel launchers (arguments already validated by the C ABI layer).
dq_status_t launch_gemv_b1(const dq_weights_t& w, const uint16_t* x, uint16_t* y, float k,
                           bool split, void* workspace, cudaStream_t stream);
dq_status_t launch_build_native(const uint8_t* packed, const uint16_t* scales, const uint16_t* zeros,
                                int d_out, int d_in, uint8_t* out, cudaStream_t stream);
dq_status_t read_device_error(uint32_t* word, bool clear);
dq_status_t launch_reference_gemv(const uint16_t* w16, const uint16_t* x, uint16_t* y, int d_out,
                                  int d_in, cudaStream_t stream);
dq_status_t launch_detect(const uint16_t* x, int d_in, float k, uint32_t* mask_words,
                          int32_t* indices, int32_t* count, float* stats, cudaStream_t stream);
dq_status_t launch_quantize(const uint16_t* w16, int d_out, int d_in, uint8_t* packed,
                            uint16_t* scales, uint16_t* zeros, cudaStream_t stream);
dq_status_t launch_colmajor(const uint16_t* w16, int d_out, int d_in, uint16_t* cm,
                            cudaStream_t stream);

// Largest d_in the single-pass kernels accept (x, its B fragments and the
// outlier list live in shared memory next to the weight rings).
constexpr int kMaxDIn = 30720;

}  // namespace dq
